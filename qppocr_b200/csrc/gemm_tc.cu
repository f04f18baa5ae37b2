// Dense convolution / linear layers on the 5th-generation tensor cores.
//
// Replaces the reference's sgemm family (qppocr-kernels gemm.rs:223-589,
// conv.rs:264-460 1x1 path, conv.rs:553-637 implicit GEMM, conv.rs:856-901
// conv1x1_nhwc, shape.rs:568-698 constant-B matmul).
//
//   D[128 x BN] tile in TMEM  =  sum_k  A[128 x 32] (smem)  *  B[BN x 32]^T (smem)
//
// * A (activations, NHWC rows) and B (weights, [N][K] = ONNX Conv layout,
//   K-major) are staged by TMA with 128-byte swizzle into a STAGES-deep ring.
// * One elected lane issues tcgen05.mma kind::tf32 (M=128, N=BN, K=8); the
//   accumulator lives in TMEM and never touches registers during the K loop.
// * Operands are rounded to tf32 to nearest (the tensor core itself would
//   truncate, biasing every product toward zero): B at load time, A on chip
//   by four converter warps between the TMA landing and the MMA.
// * MATH_3XTF32 (fp32-accurate mode): B arrives pre-split (hi = rn(B),
//   lo = rn(B - hi)); A is split the same way on chip; each k-step issues
//   lo*hi + hi*lo + hi*hi.  The tensor core's fp32 accumulation drifts toward
//   zero with K, so partial sums over CH k-blocks are promoted into fp32
//   registers with IEEE round-to-nearest adds (TMEM is drained per chunk).
// * Persistent: one CTA per SM walks output tiles round-robin; TMA, A
//   conversion and MMA run ahead across tiles while the epilogue drains the
//   other of two TMEM accumulators.
// * Epilogue: warps 4-7 read their 32 TMEM lanes (tcgen05.ld 32x32b), add bias,
//   apply the fused activation, add the residual (optionally through a
//   nearest-upsample index map) and store fp32 rows.
// * A_MODE 2 (k x k, stride 1, output rows >= 64 wide): a tile is one output
//   row of 128 pixels; per (kernel row, 32-channel block) one TMA box brings a
//   128 + kw - 1 pixel halo row, and tap kx reads it shifted by kx rows (a
//   descriptor start kx * 128 bytes in; the 128-byte swizzle is a function of
//   the absolute shared-memory address, so the shifted view reads the rows
//   the TMA wrote, with base offset 0), so each input pixel crosses L2 -> SM
//   once per kernel row instead of once per tap.
// * A_MODE 1 (k x k, stride 1 conv): the A tile is a 4-D TMA box
//   [1][TH][TW][32ch] of the NHWC input shifted by the tap offset; rows and
//   columns outside the image are zero-filled by TMA, which is exactly the
//   conv's zero padding.  k order is tap-major then channel.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "tc_epilogue.cuh"

namespace qpc {

namespace {


// A_MODE 2 (halo row): one output row of 128 pixels per tile; the A stage is a
// 128 + kw - 1 pixel halo row (136 rows reserved, 17 KB) and B holds the kw
// taps of one kernel row, room for MAX_KW_HALO taps.  The host routes only
// kernels with kw <= MAX_KW_HALO here: the B box is kw taps deep.
constexpr int MAX_KW_HALO = 3;
constexpr int HALO_ROWS = 136;
constexpr int HALO_BYTES = HALO_ROWS * BK * 4;
static_assert(BM + MAX_KW_HALO - 1 <= HALO_ROWS, "halo row does not fit its buffer");

// A_MODE 7 (CTC head, A resident): the stages hold B only; the row block's
// A, up to HEAD_RES_KB k-blocks, sits in RES bytes after them.
constexpr int HEAD_RES_KB = 5;
template <int BN, bool SPLIT, int A_MODE>
struct Smem {
  static constexpr int A_BYTES = A_MODE == 7 ? 0 : (A_MODE == 2 ? HALO_BYTES : A_TILE_BYTES);
  static constexpr int B_TILE = BN * BK * 4;
  static constexpr int B_BYTES = (A_MODE == 2 ? MAX_KW_HALO : 1) * B_TILE;
  static constexpr int STAGE = A_BYTES + B_BYTES + (SPLIT ? (A_BYTES + B_BYTES) : 0);
  static constexpr int RES = A_MODE == 7 ? HEAD_RES_KB * A_TILE_BYTES : 0;
};

// CTC head (A_MODE 6, 7).  Tile schedule: CTA b owns the contiguous tiles
// [head_lo(b), head_lo(b + 1)) of the row-major tile order (so a row block's
// column tiles reach it in ascending order, one row block after the other),
// and its epilogue group g takes the CTA's tiles g, g + NGRP, ... as in the
// strided schedule.  Each group keeps one running (max, argmax, sum exp) per
// row over its tiles of a row block and leaves it in the partials slot of
// its first tile there.
__device__ __forceinline__ int head_lo(int b, int T, int W) { return (int)((int64_t)b * T / W); }

// Tile of slot k of this CTA, or -1 past its last tile.
template <bool HEAD>
__device__ __forceinline__ int cta_tile(int k, int T) {
  if constexpr (HEAD) {
    const int t = head_lo((int)blockIdx.x, T, (int)gridDim.x) + k;
    return t < head_lo((int)blockIdx.x + 1, T, (int)gridDim.x) ? t : -1;
  } else {
    const int64_t t = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
    return t < T ? (int)t : -1;
  }
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x (MUFU; subnormal results flush to zero).  exp(x) is taken as
// 2^(x log2 e): the head only sums these terms for the softmax denominator.
__device__ __forceinline__ float exp2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// One row's running softmax state over the columns merged so far.
struct HeadRun {
  float m;  // first strict maximum of logit + bias
  float s;  // sum of exp(l - m)
  int mi;   // its column
};

// Merges one tile's columns into `hr`, in 32-column chunks.  Per chunk: bias
// (loaded before the TMEM read so the two latencies overlap), padding
// columns -> -inf, the chunk max (three-input max tree), its first column (a
// descending select scan: the lowest column holding the max, as an ascending
// scan with a strict compare keeps), then sum exp(l - max).  Chunks and
// tiles arrive in ascending column order, so `cm > hr.m` keeps the first
// maximum across them too.
template <int BN, class Fetch>
__device__ __forceinline__ void head_tile(const GemmArgs& args, int n0, HeadRun& hr, Fetch&& fetch) {
  const float* bias = args.epi.bias;
#pragma unroll 1
  for (int cc = 0; cc < BN; cc += 32) {
    const int c0 = n0 + cc;
    if (c0 >= args.N) break;
    const int valid = args.N - c0;  // columns >= valid are padding
    float4 b[8];
    if (bias) {
      const float4* b4 = reinterpret_cast<const float4*>(bias + c0);
      if (valid >= 32) {
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] = __ldg(b4 + j);
      } else {  // the head's last chunk: stay inside the bias array
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          b[j].x = 4 * j < valid ? __ldg(bias + c0 + 4 * j) : 0.f;
          b[j].y = 4 * j + 1 < valid ? __ldg(bias + c0 + 4 * j + 1) : 0.f;
          b[j].z = 4 * j + 2 < valid ? __ldg(bias + c0 + 4 * j + 2) : 0.f;
          b[j].w = 4 * j + 3 < valid ? __ldg(bias + c0 + 4 * j + 3) : 0.f;
        }
      }
    }
    float v[32];
    fetch(cc, v);
    if (bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] = __fadd_rn(v[4 * j], b[j].x);
        v[4 * j + 1] = __fadd_rn(v[4 * j + 1], b[j].y);
        v[4 * j + 2] = __fadd_rn(v[4 * j + 2], b[j].z);
        v[4 * j + 3] = __fadd_rn(v[4 * j + 3], b[j].w);
      }
    }
    if (valid < 32)
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j >= valid) v[j] = -INFINITY;
    float t[11];
#pragma unroll
    for (int j = 0; j < 10; ++j) t[j] = max3f(v[3 * j], v[3 * j + 1], v[3 * j + 2]);
    t[10] = fmaxf(v[30], v[31]);
    const float cm = max3f(max3f(t[0], t[1], t[2]), max3f(t[3], t[4], t[5]),
                           max3f(t[6], t[7], fmaxf(t[8], fmaxf(t[9], t[10]))));
    int cj = 31;
#pragma unroll
    for (int j = 30; j >= 0; --j) cj = v[j] == cm ? j : cj;
    const float cmL = cm * kLog2e;
    float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      p0 += exp2_ftz(fmaf(v[j], kLog2e, -cmL));
      p1 += exp2_ftz(fmaf(v[j + 1], kLog2e, -cmL));
      p2 += exp2_ftz(fmaf(v[j + 2], kLog2e, -cmL));
      p3 += exp2_ftz(fmaf(v[j + 3], kLog2e, -cmL));
    }
    const float cs = (p0 + p1) + (p2 + p3);
    if (cm > hr.m) {
      hr.s = hr.s * exp2_ftz((hr.m - cm) * kLog2e) + cs;
      hr.m = cm;
      hr.mi = c0 + cj;
    } else {
      hr.s += cs * exp2_ftz((cm - hr.m) * kLog2e);
    }
  }
}

// ConvT pair epilogue for one tile (A_MODE 4: up to 32 channels between the
// layers, A_MODE 5: up to 24; launch_convt_pair): row r is input pixel
// `orow` of the first ConvT and its 128 columns are that layer's outputs for
// the sub-pixels s = 2 dy + dx, 32 columns each.  Per sub-pixel: + BN shift
// (the scale is folded into the filter), act1, then the second ConvT's four
// outputs sum_m z[m] * w2[m][ey][ex] (m ascending, fma from 0) and act2.
// The pixel's 4 x 4 output block leaves as four 16-byte row segments (a
// warp's 32 pixels write 512 contiguous bytes per output row).  `pc` (shift,
// w2) sits in the kernel parameters.
template <int PM, class Consts, class Fetch>
__device__ __forceinline__ void pair_tile(const GemmArgs& args, int64_t orow, const Consts& pc, Fetch&& fetch) {
  const GemmEpilogue& e = args.epi;
  const int64_t ow = 4 * (int64_t)e.pair_w;
  float* dst = nullptr;
  if (orow >= 0) {
    const int64_t hw = (int64_t)e.pair_h * e.pair_w;
    const int64_t img = orow / hw;
    const int rem = (int)(orow - img * hw);
    const int y = rem / e.pair_w, x = rem - y * e.pair_w;
    dst = e.out + ((img * 4 * e.pair_h + 4 * y) * ow + 4 * x);
  }
#pragma unroll
  for (int dy = 0; dy < 2; ++dy) {
    float o[8];  // output rows 4y + 2 dy + ey, columns 4x + 2 dx + ex: [ey][2 dx + ex]
#pragma unroll
    for (int dx = 0; dx < 2; ++dx) {
      const int s = 2 * dy + dx;
      float v[32];
      fetch(32 * s, v);  // warp-collective
#pragma unroll
      for (int j = 0; j < PM; ++j) v[j] = __fadd_rn(v[j], pc.shift[32 * s + j]);
      apply_act_n(v, e.act);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int m = 0; m < PM; ++m) {
        a0 = __fmaf_rn(v[m], pc.w2[m][0], a0);
        a1 = __fmaf_rn(v[m], pc.w2[m][1], a1);
        a2 = __fmaf_rn(v[m], pc.w2[m][2], a2);
        a3 = __fmaf_rn(v[m], pc.w2[m][3], a3);
      }
      o[2 * dx] = a0;
      o[2 * dx + 1] = a1;
      o[4 + 2 * dx] = a2;
      o[4 + 2 * dx + 1] = a3;
    }
    apply_act_n(o, e.pair_act);
    if (dst) {
      *reinterpret_cast<float4*>(dst + (2 * dy) * ow) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(dst + (2 * dy + 1) * ow) = make_float4(o[4], o[5], o[6], o[7]);
    }
  }
}

// Warp roles: w0 TMA producer, w1 MMA issuer, w2-3 convert A, then 4-warp
// epilogue groups that take tiles round-robin (their serial TMEM -> smem ->
// TMA-store chains overlap).  TF32 runs 4 groups for 32-column N tiles,
// where a tile carries little work and the chain's latency sets the pace, and
// 2 otherwise; 3xTF32 keeps one group, whose registers hold the promoted
// accumulator.
// The ConvT pair mode (A_MODE 4/5) runs 4 groups: its epilogue is arithmetic
// (a second layer per row), and it stages no output in shared memory.  The
// CTC head (A_MODE 6, 7) stages nothing either; it runs HEAD_GROUPS groups.
constexpr int HEAD_GROUPS = 2;
template <int BN, bool SPLIT, int A_MODE = 0>
struct Roles {
  static constexpr int EPI_GROUPS =
      SPLIT ? 1 : ((A_MODE == 6 || A_MODE == 7) ? HEAD_GROUPS : ((BN <= 32 || A_MODE >= 4) ? 4 : 2));
  static constexpr int THREADS = 128 + 128 * EPI_GROUPS;
  static constexpr int STAGING = A_MODE >= 4 ? 0 : EPI_GROUPS * 2 * OUT_STAGE_BYTES;
};

// Per-mode constants passed by value in the kernel parameters (constant
// bank), so an unrolled epilogue reads them as instruction operands.
struct NoConsts {
  int unused;
};
struct PairConsts {
  float shift[128];  // first ConvT's BN shift per column (its scale is folded into B), zero on padding
  float w2[32][4];   // second ConvT [m][2 ey + ex], zero rows past M
};
template <int A_MODE>
struct ModeConsts {
  using type = NoConsts;
};
template <>
struct ModeConsts<4> {
  using type = PairConsts;
};
template <>
struct ModeConsts<5> {
  using type = PairConsts;
};
// TMEM accumulators: 8 for 32-column tiles, 4 up to 128 columns, 2 otherwise
// (the MMA runs ahead of the epilogue groups by NBUF - groups tiles);
// 3xTF32 ping-pongs 2 chunk buffers.
template <int BN, bool SPLIT>
struct Accs {
  static constexpr int NBUF = SPLIT ? 2 : (BN <= 32 ? 8 : (BN <= 128 ? 4 : 2));
};
constexpr int CH = 1;             // k-blocks per promotion chunk (3xTF32)

// Persistent, warp-specialised tcgen05 GEMM.  Each CTA walks tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...; the TMA ring, the A conversion and
// the MMAs run ahead across tile boundaries while the epilogue warps drain the
// previous tile from the other TMEM accumulator.
template <int BN, int STAGES, bool SPLIT, int A_MODE>
__global__ void __launch_bounds__(Roles<BN, SPLIT, A_MODE>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmOut,
                   const GemmArgs args, const __grid_constant__ typename ModeConsts<A_MODE>::type mc) {
  using SM = Smem<BN, SPLIT, A_MODE>;
  // A_MODE 3: rows mode (0) with the per-image channel gate applied to A;
  // A_MODE 4/5: rows mode with the ConvT pair epilogue (pair_tile);
  // A_MODE 6: rows mode with the CTC head epilogue (head_tile);
  // A_MODE 7: the same with the row block's A resident in shared memory
  // (tf32-rounded by its producer; loaded once per row block, B streams)
  constexpr int AM = (A_MODE == 3 || A_MODE >= 4) ? 0 : A_MODE;
  constexpr bool GATED = A_MODE == 3;
  constexpr bool PAIR = A_MODE == 4 || A_MODE == 5;
  constexpr bool HEAD = A_MODE == 6 || A_MODE == 7;
  constexpr bool ARES = A_MODE == 7;
  constexpr int PAIR_M = A_MODE == 5 ? 24 : 32;
  constexpr int NBUF = Accs<BN, SPLIT>::NBUF;
  constexpr int NGRP = Roles<BN, SPLIT, A_MODE>::EPI_GROUPS;
  static_assert(NBUF % NGRP == 0, "each accumulator must belong to one epilogue group");
  // A stored tf32-rounded by its producer (rows mode, no gate or split): the
  // converters have nothing to do, and the MMA thread takes each stage from
  // the TMA barrier directly.
  const bool conv_skip = ARES || (AM == 0 && !GATED && !SPLIT && !PAIR && args.epi.a_rounded != 0);
  constexpr uint32_t TMEM_COLS = (NBUF * BN < 32) ? 32 : NBUF * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t conv_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[NBUF];
  __shared__ __align__(8) uint64_t acc_empty[NBUF];
  __shared__ __align__(8) uint64_t a_full;   // ARES: the row block's A landed
  __shared__ __align__(8) uint64_t a_empty;  // ARES: the MMAs on the previous A completed
  __shared__ uint32_t tmem_base_slot;
  __shared__ int64_t s_rrow[NGRP][BM];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = (args.N + BN - 1) / BN;
  const int total_tiles = args.m_tiles * n_tiles;
  const int nkb = args.nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], 64);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&a_full, 1);
    mbar_init(&a_empty, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    if (SPLIT) prefetch_tensormap(&tmBlo);
    if (args.tma_store) prefetch_tensormap(&tmOut);
  }
  uint8_t* out_stage = smem + STAGES * SM::STAGE;  // 2 x 16 KB, 1024-aligned
  uint8_t* a_res = out_stage + Roles<BN, SPLIT, A_MODE>::STAGING;  // ARES: SM::RES bytes
  if (warp == 0) {
    tmem_alloc(&tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      const uint32_t a_bytes = AM == 2 ? (uint32_t)(BM + args.kw - 1) * BK * 4
                                       : (AM == 0 ? (uint32_t)(BM * args.bkw * 4) : A_TILE_BYTES);
      const uint32_t b_bytes = AM == 2 ? args.kw * SM::B_TILE : (AM == 0 ? (uint32_t)(BN * args.bkw * 4) : SM::B_TILE);
      const uint32_t bytes = ARES ? b_bytes : (SPLIT ? (a_bytes + 2 * b_bytes) : (a_bytes + b_bytes));
      uint32_t it = 0, a_loads = 0;
      int a_mblk = -1;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int tile = cta_tile<HEAD>(k, total_tiles);
        if (tile < 0) break;
        const TileCoord tc = tile_coord(args, tile, n_tiles, BN);
        if constexpr (ARES) {
          if (tc.m_blk != a_mblk) {  // the row block's A, once the MMAs on the last one are done
            if (a_loads > 0 && !mbar_wait(&a_empty, (a_loads - 1) & 1u, args.err)) { ok = false; break; }
            mbar_arrive_expect_tx(&a_full, (uint32_t)nkb * a_bytes);
            for (int kb = 0; kb < nkb; ++kb)
              tma_load_2d(a_res + kb * A_TILE_BYTES, &tmA, &a_full, kb * args.bkw, tc.m_blk * BM);
            ++a_loads;
            a_mblk = tc.m_blk;
          }
        }
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.err)) { ok = false; break; }
          uint8_t* st = smem + s * SM::STAGE;
          mbar_arrive_expect_tx(&full_bar[s], bytes);
          if (ARES) {
            tma_load_2d(st, &tmB, &full_bar[s], kb * args.bkw, tc.n0);
          } else if (AM == 0) {
            tma_load_2d(st, &tmA, &full_bar[s], kb * args.bkw, tc.m_blk * BM);
            tma_load_2d(st + SM::A_BYTES, &tmB, &full_bar[s], kb * args.bkw, tc.n0);
            if (SPLIT) tma_load_2d(st + 2 * SM::A_BYTES + SM::B_BYTES, &tmBlo, &full_bar[s], kb * args.bkw, tc.n0);
          } else if (AM == 2) {
            // halo row of input row oy + ky - ph, columns ox0 - pw .. ox0 - pw + 128 + kw - 2
            const int ky = kb / args.cblocks, cb = kb % args.cblocks;
            tma_load_4d(st, &tmA, &full_bar[s], cb * BK, tc.ox0 - args.pw, tc.oy0 + ky - args.ph, tc.img);
            tma_load_4d(st + SM::A_BYTES, &tmB, &full_bar[s], cb * BK, tc.n0, ky * args.kw, 0);
            if (SPLIT)
              tma_load_4d(st + 2 * SM::A_BYTES + SM::B_BYTES, &tmBlo, &full_bar[s], cb * BK, tc.n0, ky * args.kw, 0);
          } else {
            const int tap = kb / args.cblocks, cb = kb % args.cblocks;
            const int ky = tap / args.kw, kx = tap % args.kw;
            tma_load_4d(st, &tmA, &full_bar[s], cb * BK, tc.ox0 + kx - args.pw, tc.oy0 + ky - args.ph, tc.img);
            tma_load_4d(st + SM::A_BYTES, &tmB, &full_bar[s], cb * BK, tc.n0, tap, 0);
            if (SPLIT)
              tma_load_4d(st + 2 * SM::A_BYTES + SM::B_BYTES, &tmBlo, &full_bar[s], cb * BK, tc.n0, tap, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      uint32_t it = 0, acc_i = 0;  // acc_i: accumulator fills (tiles, or chunks in 3xTF32)
      uint32_t a_uses = 0;
      int a_mblk = -1;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int tile = cta_tile<HEAD>(k, total_tiles);
        if (tile < 0) break;
        if constexpr (ARES) {
          const int m_blk = tile / n_tiles;
          if (m_blk != a_mblk) {
            // a_empty completes once every MMA issued so far (those reading
            // the previous A) has; then wait for this row block's A
            if (a_uses > 0) mma_commit(&a_empty);
            if (!mbar_wait(&a_full, a_uses & 1u, args.err)) { ok = false; break; }
            ++a_uses;
            a_mblk = m_blk;
          }
        }
        for (int kb = 0; kb < nkb && ok; ++kb, ++it) {
          const bool first = SPLIT ? (kb % CH) == 0 : kb == 0;
          const uint32_t buf = acc_i % NBUF;
          if (first && acc_i >= (uint32_t)NBUF) {
            if (!mbar_wait(&acc_empty[buf], ((acc_i / NBUF) - 1) & 1u, args.err)) {
              ok = false;
              break;
            }
            tc_fence_after();  // the epilogue's TMEM reads of this accumulator come first
          }
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          // Operand stages need no tcgen05 fence: the mbarrier wait orders the
          // TMA writes and the converters' (proxy-fenced) writes before the MMAs,
          // and a fence per stage would stall this thread on the MMAs in flight.
          if (!mbar_wait(conv_skip ? &full_bar[s] : &conv_bar[s], ph, args.err)) { ok = false; break; }
          const uint32_t d_tmem = tmem_d + buf * BN;
          const uint32_t a_addr = ARES ? smem_u32(a_res + kb * A_TILE_BYTES) : smem_u32(smem + s * SM::STAGE);
          const uint32_t b_addr = ARES ? smem_u32(smem + s * SM::STAGE) : a_addr + SM::A_BYTES;
          const uint32_t alo_addr = b_addr + SM::B_BYTES;
          const uint32_t blo_addr = alo_addr + SM::A_BYTES;
          // AM 2: tap kx of this kernel row is the halo shifted by kx rows
          const int ntap = AM == 2 ? args.kw : 1;
          const int ksteps = AM == 0 ? args.bkw / 8 : BK / 8;
          for (int kx = 0; kx < ntap; ++kx) {
            const uint32_t a_off = (uint32_t)kx * 128u, b_off = (uint32_t)kx * SM::B_TILE;
#pragma unroll
            for (int ks = 0; ks < BK / 8; ++ks) {
              if (ks >= ksteps) break;
              const uint32_t acc = (!first || kx > 0 || ks > 0) ? 1u : 0u;
              const uint64_t ad = sw128_kmajor_desc(a_addr + a_off + ks * 32);
              const uint64_t bd = sw128_kmajor_desc(b_addr + b_off + ks * 32);
              if (SPLIT) {
                const uint64_t alo = sw128_kmajor_desc(alo_addr + a_off + ks * 32);
                const uint64_t blo = sw128_kmajor_desc(blo_addr + b_off + ks * 32);
                mma_tf32(d_tmem, alo, bd, idesc, acc);
                mma_tf32(d_tmem, ad, blo, idesc, 1u);
                mma_tf32(d_tmem, ad, bd, idesc, 1u);
              } else {
                mma_tf32(d_tmem, ad, bd, idesc, acc);
              }
            }
          }
          mma_commit(&empty_bar[s]);  // frees the stage once these MMAs have read it
          const bool last = SPLIT ? ((kb % CH) == CH - 1 || kb == nkb - 1) : kb == nkb - 1;
          if (last) {
            mma_commit(&acc_full[buf]);
            ++acc_i;
          }
        }
      }
    }
  } else if (warp < 4) {
    // ---------------- converters: round A to tf32 (nearest) in place; in
    // 3xTF32 also write lo = rn(A - hi).  Elementwise, so the swizzle is moot.
    const int t = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = true;
    const float* gate = GATED ? args.epi.a_gate : nullptr;
    const int ghw = GATED ? args.epi.a_gate_rows : 1;
    const int64_t img_last = GATED ? (args.M - 1) / ghw : 0;
    for (int k = 0; ok && !conv_skip; ++k) {
      const int tile = cta_tile<HEAD>(k, total_tiles);
      if (tile < 0) break;
      // image of this tile's first row and that row's place in it (rows are
      // consecutive pixels, so a row's image is img0 + the number of image
      // boundaries crossed, at most one when an image has >= 128 rows)
      const int64_t row0 = (int64_t)(tile / n_tiles) * BM;
      const int64_t img0 = GATED ? row0 / ghw : 0;
      const int r0 = GATED ? (int)(row0 - img0 * ghw) : 0;
      const int64_t img1 = GATED ? min(img0 + 1, img_last) : 0;
      // Chunk i = t + 64 j is row (t >> 3) + 8 j, channel quad (t & 7) ^ ((t >> 3) & 7):
      // the same quad for all of this thread's chunks, so with >= 128-row
      // images only two gate values (this image's, the next one's) occur,
      // the next one's from tile row rsw on.  They do not depend on the
      // stage's data: each stage's pair is loaded one stage ahead.
      const int quad = ((t & 7) ^ ((t >> 3) & 7)) << 2;
      const int rsw = GATED ? ghw - r0 : 0;
      auto gate_pair = [&](int kb, float4& ga, float4& gb) {
        ga = make_float4(0.f, 0.f, 0.f, 0.f);
        gb = ga;
        const int ch = kb * args.bkw + quad;
        if (ch < args.K) {
          ga = __ldg(reinterpret_cast<const float4*>(gate + img0 * (int64_t)args.K + ch));
          gb = __ldg(reinterpret_cast<const float4*>(gate + img1 * (int64_t)args.K + ch));
        }
      };
      float4 ga_next = make_float4(0.f, 0.f, 0.f, 0.f), gb_next = ga_next;
      if (GATED && ghw >= BM) gate_pair(0, ga_next, gb_next);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        const float4 ga = ga_next, gb = gb_next;
        if (GATED && ghw >= BM && kb + 1 < nkb) gate_pair(kb + 1, ga_next, gb_next);
        if (!mbar_wait(&full_bar[s], ph, args.err)) { ok = false; break; }
        float4* a = reinterpret_cast<float4*>(smem + s * SM::STAGE);
        float4* lo = reinterpret_cast<float4*>(smem + s * SM::STAGE + SM::A_BYTES + SM::B_BYTES);
        // (A rounded by its producer in rows mode: conv_skip, no converters)
        const int n4 = AM == 2 ? (BM + args.kw - 1) * (BK / 4) : A_TILE_BYTES / 16;
        if (GATED && ghw >= BM) {
          // rows past M and channels past K hold TMA zero fill (or, past a
          // 24-wide k-block, bytes no MMA reads): no bounds checks needed
#pragma unroll 4
          for (int i = t; i < n4; i += 64) {
            float4 v = a[i];
            const float4 g4 = (i >> 3) >= rsw ? gb : ga;
            v.x = __fmul_rn(v.x, g4.x);
            v.y = __fmul_rn(v.y, g4.y);
            v.z = __fmul_rn(v.z, g4.z);
            v.w = __fmul_rn(v.w, g4.w);
            float4 h;
            h.x = tf32_rna(v.x);
            h.y = tf32_rna(v.y);
            h.z = tf32_rna(v.z);
            h.w = tf32_rna(v.w);
            a[i] = h;
            if (SPLIT) {
              float4 l;
              l.x = tf32_rna(__fsub_rn(v.x, h.x));
              l.y = tf32_rna(__fsub_rn(v.y, h.y));
              l.z = tf32_rna(__fsub_rn(v.z, h.z));
              l.w = tf32_rna(__fsub_rn(v.w, h.w));
              lo[i] = l;
            }
          }
        } else {
#pragma unroll 4
        for (int i = t; i < n4; i += 64) {
          float4 v = a[i];
          if (GATED) {
            // logical (row, channel quad) of swizzled 16-byte chunk i; images
            // of fewer than 128 rows: the row's own image's gate
            const int row = i >> 3, c4 = (i & 7) ^ (row & 7);
            const int ch = kb * args.bkw + c4 * 4;
            if (row0 + row < args.M && ch < args.K) {
              const int64_t img = img0 + (r0 + row) / ghw;
              const float4 g4 = __ldg(reinterpret_cast<const float4*>(gate + img * (int64_t)args.K + ch));
              v.x = __fmul_rn(v.x, g4.x);
              v.y = __fmul_rn(v.y, g4.y);
              v.z = __fmul_rn(v.z, g4.z);
              v.w = __fmul_rn(v.w, g4.w);
            }
          }
          float4 h;
          h.x = tf32_rna(v.x);
          h.y = tf32_rna(v.y);
          h.z = tf32_rna(v.z);
          h.w = tf32_rna(v.w);
          a[i] = h;
          if (SPLIT) {
            float4 l;
            l.x = tf32_rna(__fsub_rn(v.x, h.x));
            l.y = tf32_rna(__fsub_rn(v.y, h.y));
            l.z = tf32_rna(__fsub_rn(v.z, h.z));
            l.w = tf32_rna(__fsub_rn(v.w, h.w));
            lo[i] = l;
          }
        }
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv_bar[s]);
      }
    }
  } else {
    // ---------------- epilogue groups (warps 4-7, 8-11): TMEM lane quarter
    // q = warp % 4; group `grp` takes local tiles grp, grp + NGRP, ...
    const int q = warp & 3;
    const int grp = (warp - 4) >> 2;
    const int r = q * 32 + lane;
    const int gt = threadIdx.x - 128 - grp * 128;  // thread index within the group
    const uint32_t lane_base = tmem_d + ((uint32_t)(q * 32) << 16);
    const GemmEpilogue& e = args.epi;
    uint8_t* my_stage = out_stage + grp * 2 * OUT_STAGE_BYTES;
    uint32_t acc_i = grp, chunk_ctr = 0;
    bool ok = true;
    float accr[SPLIT ? BN : 1];
    bool first_tile = true;
    // Head: this group's tiles of the CTA's range, and the running state of
    // row r of the row block in hand (written to partials[slot][row] when the
    // row block changes and at the end; slot = the group's first column tile
    // in that row block)
    int t_first = blockIdx.x + grp * gridDim.x, t_end = total_tiles, t_step = NGRP * gridDim.x;
    HeadRun hr{-INFINITY, 0.f, 0};
    int head_mblk = -1, head_slot = 0;
    auto head_flush = [&]() {
      const int64_t row = (int64_t)head_mblk * BM + r;
      if (row < args.M)
        e.partials[(int64_t)head_slot * args.M + row] = make_float4(hr.m, __uint_as_float((unsigned)hr.mi), hr.s, 0.f);
    };
    if constexpr (HEAD) {
      t_first = head_lo((int)blockIdx.x, total_tiles, (int)gridDim.x) + grp;
      t_end = head_lo((int)blockIdx.x + 1, total_tiles, (int)gridDim.x);
      t_step = NGRP;
    }
    for (int tile = t_first; tile < t_end && ok; tile += t_step) {
      const TileCoord tc = tile_coord(args, tile, n_tiles, BN);
      const RowMap rm = row_map<AM>(args, tc.m_blk, tc.img, tc.oy0, tc.ox0, r);
      const int64_t orow = rm.orow, rrow = rm.orow >= 0 ? rm.rrow : -1;
      if constexpr (HEAD) {
        if (tc.m_blk != head_mblk) {
          if (head_mblk >= 0) head_flush();
          head_mblk = tc.m_blk;
          head_slot = tc.n0 / BN;
          hr = HeadRun{-INFINITY, 0.f, 0};
        }
        // this tile's bias lines into L1 while its MMAs finish
        if (e.bias && lane < BN / 32 && tc.n0 + 32 * lane < args.N) prefetch_l1(e.bias + tc.n0 + 32 * lane);
      }
      if (!HEAD && !SPLIT && NGRP <= 2 && e.residual) {
        // Residual lines of this group's next tile (and, first, of this one)
        // into L2 while the MMAs run, so the per-chunk loads hit L2.
        auto prefetch = [&](const TileCoord& pc, int64_t prow) {
          if (prow < 0) return;
          const float* rp = e.residual + prow * e.ldr + pc.n0;
#pragma unroll
          for (int c = 0; c < BN; c += 32)
            if (pc.n0 + c < args.N) prefetch_l2(rp + c);
        };
        if (first_tile) prefetch(tc, rrow);
        const int nt = tile + NGRP * gridDim.x;
        if (nt < total_tiles) {
          const TileCoord nc = tile_coord(args, nt, n_tiles, BN);
          const RowMap nm = row_map<AM>(args, nc.m_blk, nc.img, nc.oy0, nc.ox0, r);
          prefetch(nc, nm.orow >= 0 ? nm.rrow : -1);
        }
        first_tile = false;
      }
      if (!SPLIT) {
        const uint32_t buf = acc_i % NBUF;
        if (!mbar_wait(&acc_full[buf], (acc_i / NBUF) & 1u, args.err)) { ok = false; break; }
        tc_fence_after();
        auto fetch = [&](int c, float (&v)[32]) {
          uint32_t a[16], b[16];
          tmem_ld16_nowait(lane_base + buf * BN + c, a);
          tmem_ld16_nowait(lane_base + buf * BN + c + 16, b);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = __uint_as_float(a[j]);
            v[16 + j] = __uint_as_float(b[j]);
          }
        };
        if constexpr (PAIR) {
          pair_tile<PAIR_M>(args, orow, mc, fetch);
        } else if constexpr (HEAD) {
          head_tile<BN>(args, tc.n0, hr, fetch);
        } else if (args.tma_store) {
          store_tile<BN, AM>(args, &tmOut, my_stage, s_rrow[grp], 1 + grp, chunk_ctr, tc.m_blk, tc.n0, tc.img,
                             tc.oy0, tc.ox0, r, gt, fetch);
        } else {
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            if (tc.n0 + c >= args.N) break;
            float v[16];
            tmem_ld16(lane_base + buf * BN + c, v);  // warp-collective
            if (orow >= 0) epilogue_store<BN>(args, v, orow, rrow, tc.n0 + c);
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        acc_i += NGRP;
      } else {
#pragma unroll
        for (int j = 0; j < BN; ++j) accr[j % (SPLIT ? BN : 1)] = 0.f;
        const int nchunks = (nkb + CH - 1) / CH;
        for (int ck = 0; ck < nchunks; ++ck) {
          // promotion: TMEM partial sum of this chunk -> fp32 registers (RN adds)
          const uint32_t buf = acc_i % NBUF;
          if (!mbar_wait(&acc_full[buf], (acc_i / NBUF) & 1u, args.err)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c0 = 0; c0 < (SPLIT ? BN : 16); c0 += 16) {
            uint32_t v[16];
            tmem_ld16_nowait(lane_base + buf * BN + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              accr[(c0 + j) % (SPLIT ? BN : 1)] =
                  __fadd_rn(accr[(c0 + j) % (SPLIT ? BN : 1)], __uint_as_float(v[j]));
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);
          ++acc_i;
        }
        if (!ok) break;
        auto fetch = [&](int c, float (&v)[32]) {
#pragma unroll
          for (int cb = 0; cb < BN; cb += 32)
            if (cb == c)
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = accr[(cb + j) % (SPLIT ? BN : 1)];
        };
        if constexpr (PAIR) {
          pair_tile<PAIR_M>(args, orow, mc, fetch);
        } else if constexpr (HEAD) {
          head_tile<BN>(args, tc.n0, hr, fetch);
        } else if (args.tma_store) {
          store_tile<BN, AM>(args, &tmOut, my_stage, s_rrow[grp], 1 + grp, chunk_ctr, tc.m_blk, tc.n0, tc.img,
                             tc.oy0, tc.ox0, r, gt, fetch);
        } else {
#pragma unroll
          for (int c = 0; c < BN; c += 16) {
            if (tc.n0 + c < args.N && orow >= 0) {
              float v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = accr[(c + j) % (SPLIT ? BN : 1)];
              epilogue_store<BN>(args, v, orow, rrow, tc.n0 + c);
            }
          }
        }
      }
    }
    if constexpr (HEAD) {
      if (ok && head_mblk >= 0) head_flush();
    }
  }
  if (args.tma_store && threadIdx.x >= 128 && ((threadIdx.x - 128) & 127) == 0)
    bulk_wait_group<0>();  // each epilogue group's stores out of smem before exit
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, TMEM_COLS);
}

// Row-band implicit GEMM for k x k stride-1 convs (kw <= MAX_KW_HALO, one
// column tile of N <= BN output channels, TF32).  A tile is RB output rows of
// 128 pixels.  The whole filter (taps x channel blocks x BN x 32 floats,
// tf32-rounded on the host) is loaded into shared memory once per CTA, and
// the ring streams only input halo rows: stage (j, cb) is input row
// oy0 - ph + j, channels cb*32..cb*32+31, columns ox0 - pw .. ox0 - pw + 128
// + kw - 2.  Every staged row feeds each of the kh output rows it touches
// (output row i = j - ky, all kw taps as shifted views), so an input pixel
// crosses L2 -> SM (RB + kh - 1) / RB times per output row instead of kh
// times, and no weights are restaged.  Accumulators: RB x BN TMEM columns per
// tile, two tiles in flight.  Warps: w0 TMA, w1 MMA, w2-3 tf32 rounding of A,
// w4-7 epilogue (one 128-pixel row chunk at a time through store_tile).
template <int BN, int STAGES, int RB>
__global__ void __launch_bounds__(256, 1)
    conv_band_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmOut, const GemmArgs args, int w_bytes) {
  constexpr int B_TILE = BN * BK * 4;
  constexpr uint32_t TMEM_COLS = 2 * RB * BN;
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512, "band accumulators do not fit TMEM");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t conv_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t w_full;
  __shared__ uint32_t tmem_base_slot;
  __shared__ int64_t s_rrow[BM];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = args.m_tiles;
  const int kw = args.kw, kh = args.taps / args.kw, cblocks = args.cblocks;
  const int nkb = (RB + kh - 1) * cblocks;
  uint8_t* wsm = smem;                   // resident filter
  uint8_t* ring = smem + w_bytes;        // STAGES x HALO_BYTES
  uint8_t* out_stage = ring + STAGES * HALO_BYTES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], 64);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&w_full, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmW);
    if (args.tma_store) prefetch_tensormap(&tmOut);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: the filter once, then halo rows
      mbar_arrive_expect_tx(&w_full, (uint32_t)w_bytes);
      for (int tap = 0; tap < args.taps; ++tap)
        for (int cb = 0; cb < cblocks; ++cb)
          tma_load_4d(wsm + (tap * cblocks + cb) * B_TILE, &tmW, &w_full, cb * BK, 0, tap, 0);
      const uint32_t a_bytes = (uint32_t)(BM + kw - 1) * BK * 4;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const TileCoord tc = tile_coord(args, tile, 1, BN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int j = kb / cblocks, cb = kb % cblocks;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], a_bytes);
          tma_load_4d(ring + s * HALO_BYTES, &tmA, &full_bar[s], cb * BK, tc.ox0 - args.pw,
                      tc.oy0 - args.ph + j, tc.img);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      bool ok = mbar_wait(&w_full, 0, args.err);
      const uint32_t w_addr = smem_u32(wsm);
      uint32_t it = 0, acc_i = 0;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++acc_i) {
        const TileCoord tc = tile_coord(args, tile, 1, BN);
        const int rows = min(RB, args.oh - tc.oy0);
        const uint32_t buf = acc_i & 1u;
        if (acc_i >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((acc_i >> 1) - 1) & 1u, args.err)) break;
          tc_fence_after();  // the epilogue's TMEM reads of this accumulator come first
        }
        const uint32_t d_base = tmem_d + buf * (RB * BN);
        for (int kb = 0; kb < nkb && ok; ++kb, ++it) {
          const int j = kb / cblocks, cb = kb % cblocks;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&conv_bar[s], ph, args.err)) { ok = false; break; }
          const uint32_t a_addr = smem_u32(ring + s * HALO_BYTES);
          for (int ky = 0; ky < kh; ++ky) {
            const int i = j - ky;  // output row of this tile fed by kernel row ky
            if (i < 0 || i >= rows) continue;
            const uint32_t d = d_base + i * BN;
            for (int kx = 0; kx < kw; ++kx) {
              const uint32_t b_addr = w_addr + ((ky * kw + kx) * cblocks + cb) * B_TILE;
#pragma unroll
              for (int ks = 0; ks < BK / 8; ++ks) {
                const uint32_t acc = (ky | cb | kx | ks) ? 1u : 0u;
                mma_tf32(d, sw128_kmajor_desc(a_addr + kx * 128 + ks * 32),
                         sw128_kmajor_desc(b_addr + ks * 32), idesc, acc);
              }
            }
          }
          mma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 4) {
    // ---------------- converters: round the halo row to tf32 (nearest) in place
    const int t = threadIdx.x - 64;
    const int n4 = (BM + kw - 1) * (BK / 4);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!mbar_wait(&full_bar[s], ph, args.err)) { ok = false; break; }
        float4* a = reinterpret_cast<float4*>(ring + s * HALO_BYTES);
#pragma unroll 4
        for (int i = t; i < n4; i += 64) {
          const float4 v = a[i];
          a[i] = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv_bar[s]);
      }
    }
  } else {
    // ---------------- epilogue (warps 4-7): TMEM lane r = pixel ox0 + r
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int gt = threadIdx.x - 128;
    const uint32_t lane_base = tmem_d + ((uint32_t)(q * 32) << 16);
    uint32_t acc_i = 0, chunk_ctr = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++acc_i) {
      const TileCoord tc = tile_coord(args, tile, 1, BN);
      const int rows = min(RB, args.oh - tc.oy0);
      const uint32_t buf = acc_i & 1u;
      if (!mbar_wait(&acc_full[buf], (acc_i >> 1) & 1u, args.err)) break;
      tc_fence_after();
      for (int i = 0; i < rows; ++i) {
        const uint32_t col0 = buf * (RB * BN) + i * BN;
        auto fetch = [&](int c, float (&v)[32]) {
          uint32_t a[16], b[16];
          tmem_ld16_nowait(lane_base + col0 + c, a);
          tmem_ld16_nowait(lane_base + col0 + c + 16, b);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            v[jj] = __uint_as_float(a[jj]);
            v[16 + jj] = __uint_as_float(b[jj]);
          }
        };
        if (args.tma_store) {
          store_tile<BN, 1>(args, &tmOut, out_stage, s_rrow, 1, chunk_ctr, 0, 0, tc.img, tc.oy0 + i, tc.ox0,
                            r, gt, fetch);
        } else {
          const RowMap m = row_map<1>(args, 0, tc.img, tc.oy0 + i, tc.ox0, r);
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            if (c >= args.N) break;
            float v[16];
            tmem_ld16(lane_base + col0 + c, v);  // warp-collective
            if (m.orow >= 0) epilogue_store<BN>(args, v, m.orow, m.rrow, c);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  if (args.tma_store && threadIdx.x == 128) bulk_wait_group<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, TMEM_COLS);
}

// Tap-folded row-band implicit GEMM for k x k stride-1 convs with M <= 32
// output channels (TF32).  A 128 x N x 8 TF32 MMA with a small N costs about
// as much as a wide one (its issue, not its arithmetic, sets the pace), so
// the kw taps of one kernel row go into N: B rows are (kx, m) pairs (NF =
// kw*M rounded up to 16) and one MMA over an unshifted 128-pixel input row j
// produces, for every input pixel p, all kw tap products P[p][kx][m] of
// kernel row ky = j - i for output row i.  Output pixel t of the tile is
// sum_kx P[t + kx][kx][m]: the epilogue takes slice kx = 0 from its own TMEM
// lane and slices kx >= 1 from lanes t + kx through shared memory, so a tile
// row yields TWO = 128 - (kw - 1) outputs.
// The kernel rows go into N as well: the filter sits in shared memory as
// [cblocks][kh][NF] with ky descending, and accumulator i (output row i of
// the tile) occupies TMEM columns [i*NF, (i+1)*NF), so kernel rows hi..lo of
// input row j - feeding output rows j-hi..j-lo - are one contiguous run of B
// rows and one of D columns: a single MMA with N = (hi-lo+1)*NF per k-step.
// Each accumulator element still receives its k-slices in the same order
// (input row, channel block, k-step) as with one MMA per kernel row.
// Accumulator i sums ky and channels on the tensor core; the kx slices are
// added in fp32 (slice 0, then 1, then 2) in the epilogue.
// Warps: w0 TMA, w1 MMA, w2-3 tf32 rounding of A, w4-7 epilogue.
//
// MMAs of one staged input row j (channel block cb) for kernel rows LO..HI
// of a 3-row kernel with 3*NF <= 256, straight-line: a runtime loop around
// MMA issue, closed by a commit, was measured to slow every MMA in it
// several-fold.  An output row's first contribution (ky = 0, cb = 0, k-step 0)
// initialises its accumulator, so that k-step is split: row j alone with
// accumulate off, rows j-HI..j-1 with it on.
// Descriptors are built once per kernel: a swizzled K-major descriptor of
// address x + off is the one of x plus off / 16 (the address field holds
// x / 16, and shared addresses stay below 256 KB), so the issue thread only
// adds constants.  ids[n - 1]: instruction descriptor for N = n * NF.
template <int LO, int HI>
__device__ __forceinline__ void fold_issue(uint32_t d_base, int j, uint32_t nf, uint64_t a_desc, uint64_t b_cb,
                                           bool first_cb, const uint32_t (&ids)[3]) {
  const uint32_t d_lo = d_base + (uint32_t)(j - HI) * nf;  // accumulator of output row j - HI
  const uint64_t b_lo = b_cb + (uint64_t)((2 - HI) * nf * 8u);  // B rows of kernel row HI (descending)
#pragma unroll
  for (int ks = 0; ks < BK / 8; ++ks) {
    const uint64_t ad = a_desc + (uint64_t)(ks * 2);
    if (LO == 0 && ks == 0 && first_cb) {
      mma_tf32(d_base + (uint32_t)j * nf, ad, b_cb + (uint64_t)(2u * nf * 8u), ids[0], 0u);
      if (HI >= 1) mma_tf32(d_lo, ad, b_lo, ids[HI >= 1 ? HI - 1 : 0], 1u);
    } else {
      mma_tf32(d_lo, ad, b_lo + (uint64_t)(ks * 2), ids[HI - LO], 1u);
    }
  }
}

// The same for any kernel height, in runs of at most 256 / NF kernel rows.
__device__ __forceinline__ void fold_issue_rt(uint32_t d_base, int j, uint32_t nf, uint64_t a_desc, uint64_t b_cb,
                                              int kh, int lo, int hi, bool first_cb) {
  const int maxr = 256 / (int)nf;
  for (int ks = 0; ks < BK / 8; ++ks) {
    const uint64_t ad = a_desc + (uint64_t)(ks * 2);
    int bottom = lo;
    if (lo == 0 && ks == 0 && first_cb) {
      mma_tf32(d_base + (uint32_t)j * nf, ad, b_cb + (uint64_t)((kh - 1) * nf * 8u), idesc_tf32(BM, (int)nf), 0u);
      bottom = 1;
    }
    for (int c_hi = hi; c_hi >= bottom;) {
      const int c_lo = max(bottom, c_hi - maxr + 1);
      mma_tf32(d_base + (uint32_t)(j - c_hi) * nf, ad, b_cb + (uint64_t)((kh - 1 - c_hi) * nf * 8u + ks * 2),
               idesc_tf32(BM, (c_hi - c_lo + 1) * (int)nf), 1u);
      c_hi = c_lo - 1;
    }
  }
}

// MT > 0: the conv has MT output channels and a kw = 3 kernel, known at
// compile time, so the epilogue's exchange offsets are constants, its
// shared-memory loads are issued as one batch and the bias sits in registers
// (added after the slice sums, where the store would add it).  MT == 0: the
// same arithmetic with runtime sizes.
template <int STAGES, int MT>
__global__ void __launch_bounds__(256, 1)
    conv_fold_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmOut, const GemmArgs args, int w_bytes, int nf,
                     int rb) {
  constexpr int MAXNF = 96;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t conv_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t w_full;
  __shared__ uint32_t tmem_base_slot;
  __shared__ int64_t s_rrow[BM];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = args.m_tiles;
  const int kw = args.kw, kh = args.taps / args.kw, cblocks = args.cblocks, M = args.N;
  const int nkb = (rb + kh - 1) * cblocks;
  const int xst = (kw - 1) * M + 1;                       // exchange row stride (odd)
  const bool a_pre = args.epi.a_rounded != 0;
  uint8_t* wsm = smem;                                    // [kh][cblocks] x NF x 128 B
  uint8_t* ring = smem + w_bytes;                         // STAGES x 16 KB
  float* exch = reinterpret_cast<float*>(ring + STAGES * A_TILE_BYTES);  // 128 x xst
  uint8_t* out_stage = reinterpret_cast<uint8_t*>(exch) +
                       ((BM * xst * 4 + 1023) / 1024) * 1024;            // 2 x 16 KB
  const uint32_t tmem_cols = 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], 64);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&w_full, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmW);
    if (args.tma_store) prefetch_tensormap(&tmOut);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: the folded filter once, then input rows
      mbar_arrive_expect_tx(&w_full, (uint32_t)w_bytes);
      for (int ky = 0; ky < kh; ++ky)
        for (int cb = 0; cb < cblocks; ++cb)
          tma_load_4d(wsm + (cb * kh + (kh - 1 - ky)) * nf * 128, &tmW, &w_full, cb * BK, 0, ky, 0);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const TileCoord tc = tile_coord(args, tile, 1, 32);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int j = kb / cblocks, cb = kb % cblocks;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], A_TILE_BYTES);
          tma_load_4d(ring + s * A_TILE_BYTES, &tmA, &full_bar[s], cb * BK, tc.ox0 - args.pw,
                      tc.oy0 - args.ph + j, tc.img);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = idesc_tf32(BM, nf);
      bool ok = mbar_wait(&w_full, 0, args.err);
      const uint64_t w_desc = sw128_kmajor_desc(smem_u32(wsm));
      const uint64_t ring_desc = sw128_kmajor_desc(smem_u32(ring));
      const uint32_t ids[3] = {idesc_tf32(BM, nf), 2 * nf <= 256 ? idesc_tf32(BM, 2 * nf) : 0u,
                               3 * nf <= 256 ? idesc_tf32(BM, 3 * nf) : 0u};
      uint32_t it = 0, acc_i = 0;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++acc_i) {
        const TileCoord tc = tile_coord(args, tile, 1, 32);
        const int rows = min(rb, args.oh - tc.oy0);
        const uint32_t buf = acc_i & 1u;
        if (acc_i >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((acc_i >> 1) - 1) & 1u, args.err)) break;
          tc_fence_after();  // the epilogue's TMEM reads of this accumulator come first
        }
        const uint32_t d_base = tmem_d + buf * (uint32_t)(rb * nf);
        int j = 0, cb = 0;  // input row of the tile, channel block
        for (int kb = 0; kb < nkb && ok; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          // A rounded by its producer: straight from the TMA barrier
          if (!mbar_wait(a_pre ? &full_bar[s] : &conv_bar[s], ph, args.err)) { ok = false; break; }
          const uint64_t a_desc = ring_desc + (uint64_t)(s * (A_TILE_BYTES >> 4));
          const uint64_t b_cb = w_desc + (uint64_t)((cb * kh) * nf * 8u);  // [kh][NF] block of cb
          // kernel rows ky with output row j - ky inside the tile: lo..hi
          const int lo = max(0, j - (rows - 1)), hi = min(kh - 1, j);
          if (kh == 3 && 3 * nf <= 256) {
            switch (lo * 4 + hi) {
              case 0: fold_issue<0, 0>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              case 1: fold_issue<0, 1>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              case 2: fold_issue<0, 2>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              case 5: fold_issue<1, 1>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              case 6: fold_issue<1, 2>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              case 10: fold_issue<2, 2>(d_base, j, nf, a_desc, b_cb, cb == 0, ids); break;
              default: break;  // lo > hi: no output row of this tile uses input row j
            }
          } else if (lo <= hi) {
            fold_issue_rt(d_base, j, nf, a_desc, b_cb, kh, lo, hi, cb == 0);
          }
          mma_commit(&empty_bar[s]);
          if (++cb == cblocks) {
            cb = 0;
            ++j;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 4) {
    // ---------------- converters: round the input row to tf32 (nearest) in
    // place; idle when the producer stored A rounded
    const int t = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = !a_pre;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!mbar_wait(&full_bar[s], ph, args.err)) { ok = false; break; }
        float4* a = reinterpret_cast<float4*>(ring + s * A_TILE_BYTES);
#pragma unroll 4
        for (int i = t; i < A_TILE_BYTES / 16; i += 64) {
          const float4 v = a[i];
          a[i] = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv_bar[s]);
      }
    }
  } else {
    // ---------------- epilogue (warps 4-7): TMEM lane r = input pixel ox0 - pw + r,
    // which is also output pixel ox0 + r's kx = 0 slice
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int gt = threadIdx.x - 128;
    const uint32_t lane_base = tmem_d + ((uint32_t)(q * 32) << 16);
    const int r1 = min(r + 1, BM - 1), r2 = min(r + 2, BM - 1);  // rows >= TWO are not stored
    uint32_t acc_i = 0, chunk_ctr = 0;
    const bool has_bias = args.epi.bias != nullptr;
    float bias_r[MT > 0 ? MT : 1];
#pragma unroll
    for (int m = 0; m < (MT > 0 ? MT : 1); ++m) bias_r[m] = (MT > 0 && has_bias) ? __ldg(args.epi.bias + m) : 0.f;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++acc_i) {
      const TileCoord tc = tile_coord(args, tile, 1, 32);
      const int rows = min(rb, args.oh - tc.oy0);
      const uint32_t buf = acc_i & 1u;
      if (!mbar_wait(&acc_full[buf], (acc_i >> 1) & 1u, args.err)) break;
      tc_fence_after();
      for (int i = 0; i < rows; ++i) {
        const uint32_t col0 = buf * (uint32_t)(rb * nf) + i * nf;
        uint32_t raw[MAXNF / 16][16];
#pragma unroll
        for (int c = 0; c < MAXNF / 16; ++c)
          if (c * 16 < nf) tmem_ld16_nowait(lane_base + col0 + c * 16, raw[c]);
        tmem_ld_wait();
        float row[MAXNF];
#pragma unroll
        for (int c = 0; c < MAXNF; ++c) row[c] = __uint_as_float(raw[c / 16][c % 16]);
        named_bar_sync(2, 128);  // the previous row's readers are done with `exch`
#pragma unroll
        for (int c = 0; c < MAXNF; ++c)
          if (c >= M && c < kw * M) exch[r * xst + (c - M)] = row[c];
        named_bar_sync(2, 128);
        auto fetch = [&](int cc, float (&v)[32]) {
          if constexpr (MT > 0) {
            constexpr int XST = 2 * MT + 1;
            const float* e1 = exch + r1 * XST;
            const float* e2 = exch + r2 * XST + MT;
            float s1[MT], s2[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              s1[m] = e1[m];
              s2[m] = e2[m];
            }
#pragma unroll
            for (int m = 0; m < 32; ++m) {
              float o = 0.f;
              if (m < MT) {
                o = __fadd_rn(__fadd_rn(row[m], s1[m]), s2[m]);
                if (has_bias && args.tma_store) o = __fadd_rn(o, bias_r[m]);  // else epilogue_store adds it
              }
              v[m] = o;
            }
          } else {
#pragma unroll
            for (int m = 0; m < 32; ++m) {
              float o = 0.f;
              if (m < M) {
                o = row[m];
                if (kw > 1) o = __fadd_rn(o, exch[r1 * xst + m]);
                if (kw > 2) o = __fadd_rn(o, exch[r2 * xst + M + m]);
              }
              v[m] = o;
            }
          }
        };
        if (args.tma_store) {
          if constexpr (MT > 0)
            store_tile<32, 1, true, false>(args, &tmOut, out_stage, s_rrow, 1, chunk_ctr, 0, 0, tc.img, tc.oy0 + i,
                                           tc.ox0, r, gt, fetch);
          else
            store_tile<32, 1>(args, &tmOut, out_stage, s_rrow, 1, chunk_ctr, 0, 0, tc.img, tc.oy0 + i, tc.ox0,
                              r, gt, fetch);
        } else {
          const RowMap m = row_map<1>(args, 0, tc.img, tc.oy0 + i, tc.ox0, r);
          float v[32];
          fetch(0, v);
          if (m.orow >= 0 && r < args.tw) {
            float v16[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v16[jj] = v[jj];
            epilogue_store<32>(args, v16, m.orow, m.rrow, 0);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v16[jj] = v[16 + jj];
            if (M > 16) epilogue_store<32>(args, v16, m.orow, m.rrow, 16);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  if (args.tma_store && threadIdx.x == 128) bulk_wait_group<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, tmem_cols);
}

// ----------------------------------------------------------- host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box) {
  return make_tensor_map(map, base, rank, dims, strides, box, true);
}

}  // namespace

// fp32 tensor map, zero fill out of bounds.
bool make_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides[i];
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base),
                  gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

int sm_count() { return current_sm_count(); }

// Ring depth: as many stages as fit next to the output staging buffers and
// the 1 KB alignment slack in 224 KB of dynamic shared memory (the 227 KB
// per-block limit less up to 3 KB of static barriers and row caches), at
// most 8.  An instantiation with room for fewer than 2 stages is not built.
template <int BN, bool SPLIT, int A_MODE>
constexpr int stages_raw() {
  return (224 * 1024 - Roles<BN, SPLIT, A_MODE>::STAGING - Smem<BN, SPLIT, A_MODE>::RES - 1024) /
         Smem<BN, SPLIT, A_MODE>::STAGE;
}
template <int BN, bool SPLIT, int A_MODE>
constexpr int stages_for() {
  return stages_raw<BN, SPLIT, A_MODE>() > 8 ? 8 : stages_raw<BN, SPLIT, A_MODE>();
}

template <int BN, bool SPLIT, int A_MODE>
cudaError_t run_kernel(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& blo,
                       const CUtensorMap& out, const GemmArgs& args, int tiles, cudaStream_t st,
                       const typename ModeConsts<A_MODE>::type& mc = {}) {
  if constexpr (stages_raw<BN, SPLIT, A_MODE>() < 2) {
    return cudaErrorInvalidValue;
  } else {
  constexpr int STAGES = stages_for<BN, SPLIT, A_MODE>();
  auto kern = gemm_tc_kernel<BN, STAGES, SPLIT, A_MODE>;
  const int smem = STAGES * Smem<BN, SPLIT, A_MODE>::STAGE + Roles<BN, SPLIT, A_MODE>::STAGING +
                   Smem<BN, SPLIT, A_MODE>::RES + 1024;
  if (cudaError_t e = ensure_dyn_smem((const void*)kern, smem); e != cudaSuccess) return e;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, Roles<BN, SPLIT, A_MODE>::THREADS, smem, st>>>(a, b, blo, out, args, mc);
  return cudaGetLastError();
  }
}

template <int A_MODE>
cudaError_t dispatch(int bn, bool split, const CUtensorMap& a, const CUtensorMap& b,
                     const CUtensorMap& blo, const CUtensorMap& out, GemmArgs args, int grid_m,
                     cudaStream_t st) {
  args.m_tiles = grid_m;
  const int tiles = grid_m * ((args.N + bn - 1) / bn);
  if (!split) {
    switch (bn) {
      case 32: return run_kernel<32, false, A_MODE>(a, b, blo, out, args, tiles, st);
      case 64: return run_kernel<64, false, A_MODE>(a, b, blo, out, args, tiles, st);
      case 128: return run_kernel<128, false, A_MODE>(a, b, blo, out, args, tiles, st);
      default: return run_kernel<256, false, A_MODE>(a, b, blo, out, args, tiles, st);
    }
  }
  switch (bn) {
    case 32: return run_kernel<32, true, A_MODE>(a, b, blo, out, args, tiles, st);
    case 64: return run_kernel<64, true, A_MODE>(a, b, blo, out, args, tiles, st);
    default: return run_kernel<128, true, A_MODE>(a, b, blo, out, args, tiles, st);
  }
}

// Row-band conv: STAGES halo rows in the ring next to the resident filter and
// one epilogue group's two output staging buffers.
constexpr int BAND_STAGES = 4;
constexpr int BAND_RB = 4;
constexpr int BAND_W_MAX = 224 * 1024 - BAND_STAGES * HALO_BYTES - 2 * OUT_STAGE_BYTES - 1024;

template <int BN>
cudaError_t run_band(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& out,
                     const GemmArgs& args, int w_bytes, cudaStream_t st) {
  auto kern = conv_band_kernel<BN, BAND_STAGES, BAND_RB>;
  const int smem = w_bytes + BAND_STAGES * HALO_BYTES + 2 * OUT_STAGE_BYTES + 1024;
  if (w_bytes > BAND_W_MAX) return cudaErrorInvalidValue;
  if (cudaError_t e = ensure_dyn_smem((const void*)kern, smem); e != cudaSuccess) return e;
  const int grid = args.m_tiles < sm_count() ? args.m_tiles : sm_count();
  kern<<<grid, 256, smem, st>>>(a, w, out, args, w_bytes);
  return cudaGetLastError();
}

// Tap-folded conv: shared-memory layout and limits.
constexpr int FOLD_STAGES = 4;
int fold_nf(const ConvGeom& g) { return ((g.kw * g.m + 15) / 16) * 16; }
int fold_smem(const ConvGeom& g, int* w_bytes_out) {
  const int cblocks = (g.c + BK - 1) / BK;
  const int w_bytes = g.kh * cblocks * fold_nf(g) * 128;
  const int xst = (g.kw - 1) * g.m + 1;
  const int exch = ((BM * xst * 4 + 1023) / 1024) * 1024;
  if (w_bytes_out) *w_bytes_out = w_bytes;
  return w_bytes + FOLD_STAGES * A_TILE_BYTES + exch + 2 * OUT_STAGE_BYTES + 1024;
}

// k-block width of a rows-mode GEMM: 32 floats (one 128-byte swizzle row),
// or 24 when K is a multiple of 24 but not of 32, so that every TMA box ends
// at the tensor's edge (a box overrunning the inner dimension was measured
// several times slower in the kernel's ring).
int k_block_width(int K) { return (K % 32 != 0 && K % 24 == 0) ? 24 : BK; }

// Output tile width: the smallest N tile that covers N with the least padding
// (3xTF32 keeps its promoted accumulator in registers: at most 128 columns).
int pick_bn(int n, bool split) {
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128 || split) return 128;
  // Wider: minimise padded columns, prefer 256 on ties (fewer A re-reads).
  const int c128 = ((n + 127) / 128) * 128, c256 = ((n + 255) / 256) * 256;
  return c256 <= c128 ? 256 : 128;
}

// CTC head tile width: 256 columns whenever N allows in TF32.  A head k-block
// (24 or 32 floats) carries only 3-4 MMAs, and each pipeline stage costs a
// fixed few hundred cycles of barrier round trip whatever its size, so the
// wider tile doubles the math per stage.  3xTF32 keeps its 128-column limit.
int head_bn(int n, bool split) { return (!split && n > 128) ? 256 : pick_bn(n, split); }

}  // namespace

bool conv_fold_ok(const ConvGeom& g) {
  return g.sh == 1 && g.sw == 1 && (g.c % 4) == 0 && g.kw <= 3 && g.kh <= 7 && g.m <= 32 &&
         g.ow >= 48 && fold_smem(g, nullptr) <= 224 * 1024;
}

int gemm_tc_col_tiles(int N, int math) {
  const int bn = head_bn(N, math == MATH_3XTF32);
  return (N + bn - 1) / bn;
}

namespace {
// Largest CTA b with head_lo(b) <= t: the CTA holding tile t.
__device__ __forceinline__ int head_cta_of(int t, int T, int W) {
  return (int)((((int64_t)t + 1) * W + T - 1) / T) - 1;
}

// Per row: the partials of the (CTA, epilogue group) pairs that covered its
// row block.  A pair's partial is the first maximum over its columns there,
// and the pairs' columns interleave, so the merge keeps the larger value and,
// on equal values, the lower column: the first maximum over all columns.
template <int NGRP>
__global__ void argmax_combine_kernel(const float4* __restrict__ partials, int n_tiles, int64_t M, int W,
                                      float* __restrict__ pairs) {
  const int T = (int)((M + BM - 1) / BM) * n_tiles;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < M;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int t0 = (int)(r / BM) * n_tiles, t1 = t0 + n_tiles;
    const int b0 = head_cta_of(t0, T, W), b1 = head_cta_of(t1 - 1, T, W);
    float best = -INFINITY;
    unsigned idx = 0xffffffffu;
    float4 p[8];  // this row's partials (at most 8 per CTA span, re-read beyond)
    int np = 0;
    for (int b = b0; b <= b1; ++b) {
      const int lo = head_lo(b, T, W);
      const int s0 = max(lo, t0), s1 = min(head_lo(b + 1, T, W), t1);
#pragma unroll
      for (int g = 0; g < NGRP; ++g) {
        const int first = s0 + ((g - (s0 - lo)) % NGRP + NGRP) % NGRP;
        if (first >= s1) continue;
        const float4 q = partials[(int64_t)(first - t0) * M + r];
        const unsigned qi = __float_as_uint(q.y);
        if (q.x > best || (q.x == best && qi < idx)) {
          best = q.x;
          idx = qi;
        }
        if (np < 8) p[np] = q;
        ++np;
      }
    }
    float s = 0.f;
    if (np <= 8) {
      for (int i = 0; i < np; ++i) s += p[i].z * exp2_ftz((p[i].x - best) * kLog2e);
    } else {
      for (int b = b0; b <= b1; ++b) {
        const int lo = head_lo(b, T, W);
        const int s0 = max(lo, t0), s1 = min(head_lo(b + 1, T, W), t1);
        for (int g = 0; g < NGRP; ++g) {
          const int first = s0 + ((g - (s0 - lo)) % NGRP + NGRP) % NGRP;
          if (first >= s1) continue;
          const float4 q = partials[(int64_t)(first - t0) * M + r];
          s += q.z * exp2_ftz((q.x - best) * kLog2e);
        }
      }
    }
    pairs[2 * r] = 1.0f / s;
    pairs[2 * r + 1] = __uint_as_float(idx);
  }
}
}  // namespace

int head_workers(int64_t M, int n_tiles, int math) {
  (void)math;
  const int64_t T = ((M + BM - 1) / BM) * n_tiles;
  return T < sm_count() ? (int)T : sm_count();  // run_kernel's grid: one tile range per CTA
}

cudaError_t launch_argmax_combine(const float4* partials, int n_tiles, int64_t M, int math, float* pairs,
                                  cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  const int W = head_workers(M, n_tiles, math);
  int64_t blocks = (M + 63) / 64;  // 64-row blocks: a rec batch's 10,240 rows cover every SM
  if (math == MATH_3XTF32)
    argmax_combine_kernel<1><<<(unsigned)blocks, 64, 0, st>>>(partials, n_tiles, M, W, pairs);
  else
    argmax_combine_kernel<HEAD_GROUPS><<<(unsigned)blocks, 64, 0, st>>>(partials, n_tiles, M, W, pairs);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const float* a, int64_t M, int K, int lda, const float* b,
                           const float* b_lo, int N, const GemmEpilogue& epi, int math,
                           unsigned int* err, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((K & 3) || (lda & 3) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (reinterpret_cast<uintptr_t>(b) & 15))
    return cudaErrorInvalidValue;
  const bool split = math == MATH_3XTF32;
  if (split && !b_lo) return cudaErrorInvalidValue;
  int bn = epi.partials ? head_bn(N, split) : pick_bn(N, split);
  // A grid with fewer tiles than SMs (the rec linears: 80 row blocks) leaves
  // SMs idle while each CTA runs its one long tile alone: halve the tile width
  // (down to 64 columns) until every SM has work and both epilogue groups of
  // a CTA can run at once.  The column split changes no output element's
  // arithmetic.
  if (!epi.partials)
    while (bn > 64 && ((M + BM - 1) / BM) * ((N + bn - 1) / bn) < sm_count()) bn /= 2;
  const int bkw = k_block_width(K);
  CUtensorMap ma, mb, mblo;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lda * 4};
    const uint32_t box[2] = {(uint32_t)bkw, BM};
    if (!make_map(&ma, a, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K * 4};
    const uint32_t box[2] = {(uint32_t)bkw, (uint32_t)bn};
    if (!make_map(&mb, b, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (split && !make_map(&mblo, b_lo, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (!split) mblo = mb;
  }
  GemmArgs args{};
  args.M = (int)M;
  args.N = N;
  args.K = K;
  args.bkw = bkw;
  args.nkb = (K + bkw - 1) / bkw;
  args.epi = epi;
  args.err = err;
  CUtensorMap mo = ma;
  const float* obase = epi.out + epi.col_off;
  if (!epi.partials && (N % 4) == 0 && (epi.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(obase) & 15) == 0 &&
      (!epi.residual || ((epi.ldr % 4) == 0 && (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0))) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)epi.ldo * 4};
    const uint32_t box[2] = {32, BM};
    args.tma_store = make_map(&mo, obase, 2, dims, strides, box) ? 1 : 0;
  }
  const int grid_m = (int)((M + BM - 1) / BM);
  if (epi.partials) {  // CTC head: no gate, nothing stored
    if (epi.a_gate) return cudaErrorInvalidValue;
    if (!split && epi.a_rounded && args.nkb <= HEAD_RES_KB) {
      // A rounded by its producer and small enough to stay resident per row block
      args.m_tiles = grid_m;
      const int tiles = grid_m * ((N + bn - 1) / bn);
      switch (bn) {
        case 32: return run_kernel<32, false, 7>(ma, mb, mblo, mo, args, tiles, st);
        case 64: return run_kernel<64, false, 7>(ma, mb, mblo, mo, args, tiles, st);
        case 128: return run_kernel<128, false, 7>(ma, mb, mblo, mo, args, tiles, st);
        default: return run_kernel<256, false, 7>(ma, mb, mblo, mo, args, tiles, st);
      }
    }
    return dispatch<6>(bn, split, ma, mb, mblo, mo, args, grid_m, st);
  }
  if (epi.a_gate) return dispatch<3>(bn, split, ma, mb, mblo, mo, args, grid_m, st);
  return dispatch<0>(bn, split, ma, mb, mblo, mo, args, grid_m, st);
}

cudaError_t launch_convt_pair(const float* x, int n, int h, int w, int c, int m1, const float* b1,
                              const float* b1_lo, const float* consts, const ActParams& act1,
                              const ActParams& act2, float* out, int math, unsigned int* err,
                              cudaStream_t st) {
  if (m1 <= 0 || m1 > 32) return cudaErrorInvalidValue;
  const int64_t M = (int64_t)n * h * w;
  if (M <= 0) return cudaSuccess;
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (c <= 0 || (c & 3) || M > (int64_t)0x7fffffff || !consts || !err || misaligned(x) || misaligned(b1) ||
      misaligned(out))
    return cudaErrorInvalidValue;
  PairConsts pc;
  std::memcpy(pc.shift, consts, sizeof(pc.shift));
  std::memcpy(pc.w2, consts + 128, sizeof(pc.w2));
  const bool split = math == MATH_3XTF32;
  if (split && (!b1_lo || misaligned(b1_lo))) return cudaErrorInvalidValue;
  const int bkw = k_block_width(c);
  CUtensorMap ma, mb, mblo;
  {
    const uint64_t dims[2] = {(uint64_t)c, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)c * 4};
    const uint32_t box[2] = {(uint32_t)bkw, BM};
    if (!make_map(&ma, x, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {(uint64_t)c, 128};
    const uint64_t strides[1] = {(uint64_t)c * 4};
    const uint32_t box[2] = {(uint32_t)bkw, 128};
    if (!make_map(&mb, b1, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (split && !make_map(&mblo, b1_lo, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (!split) mblo = mb;
  }
  GemmArgs args{};
  args.M = (int)M;
  args.N = 128;
  args.K = c;
  args.bkw = bkw;
  args.nkb = (c + bkw - 1) / bkw;
  args.err = err;
  args.tma_store = 0;
  args.epi.out = out;
  args.epi.act = act1;
  args.epi.pair_h = h;
  args.epi.pair_w = w;
  args.epi.pair_act = act2;
  const int grid_m = (int)((M + BM - 1) / BM);
  args.m_tiles = grid_m;
  if (m1 <= 24)
    return split ? run_kernel<128, true, 5>(ma, mb, mblo, ma, args, grid_m, st, pc)
                 : run_kernel<128, false, 5>(ma, mb, mblo, ma, args, grid_m, st, pc);
  return split ? run_kernel<128, true, 4>(ma, mb, mblo, ma, args, grid_m, st, pc)
               : run_kernel<128, false, 4>(ma, mb, mblo, ma, args, grid_m, st, pc);
}

cudaError_t launch_conv_tc(const float* x, const ConvGeom& g, const float* wk, const float* wk_lo,
                           const GemmEpilogue& epi, int math, unsigned int* err,
                           cudaStream_t st, const float* wk_fold) {
  if (g.sh != 1 || g.sw != 1 || (g.c & 3)) return cudaErrorInvalidValue;
  const bool split = math == MATH_3XTF32;
  if (split && !wk_lo) return cudaErrorInvalidValue;
  if (!split && wk_fold && conv_fold_ok(g)) {
    // Tap-folded kernel: TWO = 128 - (kw - 1) output pixels per tile row.
    const int nf = fold_nf(g);
    const int two = BM - (g.kw - 1);
    const int rb = std::min(4, 256 / nf);
    int w_bytes = 0;
    const int smem = fold_smem(g, &w_bytes);
    CUtensorMap ma, mw, mo;
    {
      const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
      const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4,
                                   (uint64_t)g.c * g.w * g.h * 4};
      const uint32_t box[4] = {BK, BM, 1, 1};
      if (!make_map(&ma, x, 4, dims, strides, box)) return cudaErrorInvalidValue;
    }
    {
      const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)nf, (uint64_t)g.kh, 1};
      const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * nf * 4, (uint64_t)g.c * nf * g.kh * 4};
      const uint32_t box[4] = {BK, (uint32_t)nf, 1, 1};
      if (!make_map(&mw, wk_fold, 4, dims, strides, box)) return cudaErrorInvalidValue;
    }
    GemmArgs args{};
    args.N = g.m;
    args.K = g.c * g.kh * g.kw;
    args.M = g.n * g.oh * g.ow;
    args.cblocks = (g.c + BK - 1) / BK;
    args.taps = g.kh * g.kw;
    args.kw = g.kw;
    args.ph = g.ph;
    args.pw = g.pw;
    args.oh = g.oh;
    args.ow = g.ow;
    args.tw = two;
    args.th = rb;
    args.tiles_x = (g.ow + two - 1) / two;
    args.tiles_y = (g.oh + rb - 1) / rb;
    args.m_tiles = g.n * args.tiles_x * args.tiles_y;
    args.epi = epi;
    args.err = err;
    mo = ma;
    const float* obase = epi.out + epi.col_off;
    if ((g.m % 4) == 0 && (epi.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(obase) & 15) == 0 &&
        (!epi.residual || ((epi.ldr % 4) == 0 && (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0))) {
      const uint64_t dims[4] = {(uint64_t)g.m, (uint64_t)g.ow, (uint64_t)g.oh, (uint64_t)g.n};
      const uint64_t strides[3] = {(uint64_t)epi.ldo * 4, (uint64_t)epi.ldo * g.ow * 4,
                                   (uint64_t)epi.ldo * g.ow * g.oh * 4};
      const uint32_t box[4] = {32, (uint32_t)two, 1, 1};
      args.tma_store = make_map(&mo, obase, 4, dims, strides, box) ? 1 : 0;
    }
    auto kern = (g.m == 24 && g.kw == 3) ? conv_fold_kernel<FOLD_STAGES, 24> : conv_fold_kernel<FOLD_STAGES, 0>;
    if (cudaError_t e = ensure_dyn_smem((const void*)kern, smem); e != cudaSuccess) return e;
    const int grid = args.m_tiles < sm_count() ? args.m_tiles : sm_count();
    kern<<<grid, 256, smem, st>>>(ma, mw, mo, args, w_bytes, nf, rb);
    return cudaGetLastError();
  }
  // Row-band mode: TF32, rows at least 64 wide, kernels at most MAX_KW_HALO
  // wide, one column tile, and a filter that fits in shared memory.
  {
    const int bn = pick_bn(g.m, false);
    const int cblocks = (g.c + BK - 1) / BK;
    const int64_t w_bytes = (int64_t)g.kh * g.kw * cblocks * bn * BK * 4;
    if (!split && g.ow >= 64 && g.kw <= MAX_KW_HALO && g.m <= 64 && w_bytes <= BAND_W_MAX) {
      CUtensorMap ma, mw, mo;
      {
        const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
        const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4,
                                     (uint64_t)g.c * g.w * g.h * 4};
        const uint32_t box[4] = {BK, (uint32_t)(BM + g.kw - 1), 1, 1};
        if (!make_map(&ma, x, 4, dims, strides, box)) return cudaErrorInvalidValue;
      }
      {
        const int taps = g.kh * g.kw;
        const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.m, (uint64_t)taps, 1};
        const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.m * 4,
                                     (uint64_t)g.c * g.m * taps * 4};
        const uint32_t box[4] = {BK, (uint32_t)bn, 1, 1};
        if (!make_map(&mw, wk, 4, dims, strides, box)) return cudaErrorInvalidValue;
      }
      GemmArgs args{};
      args.N = g.m;
      args.K = g.c * g.kh * g.kw;
      args.M = g.n * g.oh * g.ow;
      args.cblocks = cblocks;
      args.taps = g.kh * g.kw;
      args.kw = g.kw;
      args.ph = g.ph;
      args.pw = g.pw;
      args.oh = g.oh;
      args.ow = g.ow;
      args.tw = BM;
      args.th = BAND_RB;
      args.tiles_x = (g.ow + BM - 1) / BM;
      args.tiles_y = (g.oh + BAND_RB - 1) / BAND_RB;
      args.m_tiles = g.n * args.tiles_x * args.tiles_y;
      args.epi = epi;
      args.err = err;
      mo = ma;
      const float* obase = epi.out + epi.col_off;
      if ((g.m % 4) == 0 && (epi.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(obase) & 15) == 0 &&
          (!epi.residual || ((epi.ldr % 4) == 0 && (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0))) {
        const uint64_t dims[4] = {(uint64_t)g.m, (uint64_t)g.ow, (uint64_t)g.oh, (uint64_t)g.n};
        const uint64_t strides[3] = {(uint64_t)epi.ldo * 4, (uint64_t)epi.ldo * g.ow * 4,
                                     (uint64_t)epi.ldo * g.ow * g.oh * 4};
        const uint32_t box[4] = {32, (uint32_t)BM, 1, 1};
        args.tma_store = make_map(&mo, obase, 4, dims, strides, box) ? 1 : 0;
      }
      if (bn == 32) return run_band<32>(ma, mw, mo, args, (int)w_bytes, st);
      return run_band<64>(ma, mw, mo, args, (int)w_bytes, st);
    }
  }
  // Halo-row mode (A_MODE 2) for rows at least 64 wide and kernels at most
  // MAX_KW_HALO wide: one 128-pixel output row per tile, each input pixel
  // staged once per kernel row.
  const bool halo = g.ow >= 64 && g.kw <= MAX_KW_HALO && g.m <= (split ? 64 : 128);
  // Tile shape TH x TW = 128 output pixels; choose TW to waste the fewest.
  int best_tw = 16;
  int64_t best_cost = INT64_MAX;
  for (int tw = 8; tw <= 128; tw *= 2) {
    const int th = 128 / tw;
    const int64_t cost = (int64_t)((g.ow + tw - 1) / tw) * tw * ((g.oh + th - 1) / th) * th;
    if (cost < best_cost) { best_cost = cost; best_tw = tw; }
  }
  const int tw = halo ? 128 : best_tw, th = halo ? 1 : 128 / tw;
  const int bn = pick_bn(g.m, split);
  CUtensorMap ma, mb, mblo;
  {
    const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4,
                                 (uint64_t)g.c * g.w * g.h * 4};
    const uint32_t box[4] = {BK, (uint32_t)(halo ? tw + g.kw - 1 : tw), (uint32_t)th, 1};
    if (!make_map(&ma, x, 4, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const int taps = g.kh * g.kw;
    const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.m, (uint64_t)taps, 1};
    const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.m * 4,
                                 (uint64_t)g.c * g.m * taps * 4};
    const uint32_t box[4] = {BK, (uint32_t)bn, (uint32_t)(halo ? g.kw : 1), 1};
    if (!make_map(&mb, wk, 4, dims, strides, box)) return cudaErrorInvalidValue;
    if (split && !make_map(&mblo, wk_lo, 4, dims, strides, box)) return cudaErrorInvalidValue;
    if (!split) mblo = mb;
  }
  GemmArgs args{};
  args.N = g.m;
  args.K = g.c * g.kh * g.kw;
  args.M = g.n * g.oh * g.ow;
  args.cblocks = (g.c + BK - 1) / BK;
  args.taps = g.kh * g.kw;
  args.nkb = (halo ? g.kh : args.taps) * args.cblocks;
  args.kw = g.kw;
  args.ph = g.ph;
  args.pw = g.pw;
  args.oh = g.oh;
  args.ow = g.ow;
  args.tw = tw;
  args.th = th;
  args.tiles_x = (g.ow + tw - 1) / tw;
  args.tiles_y = (g.oh + th - 1) / th;
  args.epi = epi;
  args.err = err;
  CUtensorMap mo = ma;
  const float* obase = epi.out + epi.col_off;
  if ((g.m % 4) == 0 && (epi.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(obase) & 15) == 0 &&
      (!epi.residual || ((epi.ldr % 4) == 0 && (reinterpret_cast<uintptr_t>(epi.residual) & 15) == 0))) {
    const uint64_t dims[4] = {(uint64_t)g.m, (uint64_t)g.ow, (uint64_t)g.oh, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)epi.ldo * 4, (uint64_t)epi.ldo * g.ow * 4,
                                 (uint64_t)epi.ldo * g.ow * g.oh * 4};
    const uint32_t box[4] = {32, (uint32_t)tw, (uint32_t)th, 1};
    args.tma_store = make_map(&mo, obase, 4, dims, strides, box) ? 1 : 0;
  }
  const int grid_m = g.n * args.tiles_x * args.tiles_y;
  if (halo) return dispatch<2>(bn, split, ma, mb, mblo, mo, args, grid_m, st);
  return dispatch<1>(bn, split, ma, mb, mblo, mo, args, grid_m, st);
}

}  // namespace qpc
