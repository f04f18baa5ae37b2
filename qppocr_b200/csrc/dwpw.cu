// Fused depthwise-separable block on the 5th-generation tensor cores:
//
//   y = act2( pw( act1( dw(x) + b1 ) ) + b2 )
//
// a depthwise k x k conv (k = 3 or 5, stride 1 or 2) whose only consumer is a
// pointwise 1x1 conv - the PP-LCNet block of the det / cls backbones.  The
// reference runs them as two passes over memory (conv2d_res_into's depthwise
// branch, crates/qppocr-kernels/src/conv.rs:461-505 with the plane kernel
// :45-71, then the 1x1 path conv.rs:264-460 -> sgemm), as its GPU plan does
// (crates/qppocr-gpu/src/plan.rs:1573-1637).  Here the depthwise output never
// leaves the SM: it is computed into shared memory, rounded to tf32, and fed
// to tcgen05.mma as the A operand of the pointwise GEMM.
//
// Tile: 8 x 16 output pixels = the 128 rows of one MMA; the K loop walks the
// input channels in blocks of CW = 32 (one 128-byte swizzle row).
//   warp 0     TMA producer of input windows: per (tile, channel block)
//              ((8-1)s+k) x ((16-1)s+k) pixels x 32 channels (zero fill =
//              the conv's zero padding).
//   warp 2     TMA producer of pointwise filter blocks [BN][32] (tf32-rounded
//              at load time): loaded once and kept when the whole filter is
//              small, else streamed through a ring on this separate thread.
//   warp 1     MMA issuer (one lane): D[128 x BN] (TMEM) += A * B^T.
//   warps 4-7  epilogue: TMEM -> + b2 -> act2 -> swizzled staging -> TMA store
//              (per-thread row stores cost one L1 transaction per row and
//              16 bytes: several times slower than the bulk store).
//   warps 8-23 depthwise, two groups of 8 warps taking alternate (tile,
//              channel block) steps: lane = channel, each thread a 4 x 4
//              block of output pixels of its channel.  Input rows are
//              streamed once each into registers and every tap that reads
//              them is applied, so per output the chain is the reference's:
//              acc = 0, fma over ky outer / kx inner, + b1, act1
//              (bit-identical to the unfused depthwise kernel), then tf32
//              rounding to nearest (what the unfused GEMM applies to its A
//              operand) into the A stage in the 128-byte-swizzled K-major
//              layout the MMA reads.
// Rings: input windows (XS), A stages (AS), filter blocks (BS, or resident);
// TMEM holds 4 accumulators (2 for 256-channel outputs) so the epilogue of
// one tile overlaps the next tiles' MMAs.  The depthwise filter sits in
// shared memory when it fits, else it is read through L1.
// Every wait is bounded (mbar_wait): a wait that runs out raises the device
// error word and the CTA drains and returns.
#include "kernels.h"
#include "tc_epilogue.cuh"

namespace qpc {

namespace {

constexpr int DW_TH = 8, DW_TW = 16;  // output tile (rows x columns) = 128 pixels
constexpr int DW_COMPUTE = 256;       // depthwise threads (8 warps)
constexpr int DW_SMEM_BUDGET = 226 * 1024;
constexpr int DW_B_RESIDENT_MAX = 64 * 1024;  // whole pointwise filter kept in shared memory up to this size

// Thread layout: warps 0-3 control (window producer, MMA, filter producer),
// then NGRP epilogue groups of 4 warps, then the 8 depthwise warps.
template <int NGRP>
struct DwRoles {
  static constexpr int EPI0 = 4, DW0 = 4 + 4 * NGRP;
  static constexpr int THREADS = 32 * DW0 + DW_COMPUTE;
};

// Depthwise work split: a thread makes 2 adjacent channels (one float2, so
// every multiply-add is a packed two-lane fma) of a BY x BX block of output
// pixels; 16 channel pairs x 16 blocks = one 32-channel block of the tile.
template <int K, int S>
struct DwpwGeo {
  static constexpr int CW = 32;
  static constexpr int IH = (DW_TH - 1) * S + K;
  static constexpr int IW = (DW_TW - 1) * S + K;
  static constexpr int X_BYTES = ((IH * IW * CW * 4 + 1023) / 1024) * 1024;
  static constexpr int BY = 4, BX = 2;
  static constexpr int BLOCKS_X = DW_TW / BX;
  static constexpr int ROWS = (BY - 1) * S + K;         // input rows one thread block reads
  static constexpr int COLS = (BX - 1) * S + K;
  static_assert((DW_COMPUTE / (CW / 2)) * BY * BX == DW_TH * DW_TW, "blocks must tile the output tile");
};

struct DwpwArgs {
  GemmArgs g;             // the pointwise GEMM: M = n*oh*ow, N = Cout, K = C, 4-D tile geometry, epilogue
  const float* dw_w;      // [k*k][C] tap-major (global)
  const float* dw_bias;   // [C] or null
  ActParams dw_act;
  int C;
  int xs, as, bs;         // ring depths (bs == 0: the whole filter is resident, one block per channel block)
  int b_off, x_off, stg_off, w_off;  // byte offsets in dynamic shared memory (w_off < 0: filter read via L1)
};

// TMEM accumulators: as many as fit 512 columns, at most 4.
template <int BN>
struct DwAcc {
  static constexpr int NBUF = BN <= 128 ? 4 : 2;
};

template <int K, int S, int BN, int NGRP>
__global__ void __launch_bounds__(DwRoles<NGRP>::THREADS, 1)
    dwpw_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmOut, const DwpwArgs a) {
  using G = DwpwGeo<K, S>;
  using R = DwRoles<NGRP>;
  constexpr int CW = G::CW;
  constexpr int DW_NBUF = DwAcc<BN>::NBUF;
  constexpr uint32_t TMEM_COLS = DW_NBUF * BN < 32 ? 32 : DW_NBUF * BN;
  constexpr uint32_t B_BYTES = BN * 128;  // one [BN][32] filter block, 128-byte rows
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t x_full[4], x_empty[4], a_full[4], a_empty[4], b_full[4], b_empty[4];
  __shared__ __align__(8) uint64_t acc_full[DW_NBUF], acc_empty[DW_NBUF];
  __shared__ uint32_t tmem_slot;

  const GemmArgs& args = a.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.C / CW;
  const int total_tiles = args.m_tiles;
  const bool b_resident = a.bs == 0;
  uint8_t* a_ring = smem;                               // AS x 16 KB
  uint8_t* b_ring = smem + a.b_off;                     // BS x B_BYTES, or nkb x B_BYTES resident
  uint8_t* x_ring = smem + a.x_off;                     // XS x X_BYTES
  uint8_t* stg = smem + a.stg_off;                      // NGRP x 2 x 16 KB output staging

  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], DW_COMPUTE / 32);  // one arrival per depthwise warp
      mbar_init(&a_full[s], DW_COMPUTE / 32);
      mbar_init(&a_empty[s], 1);
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < DW_NBUF; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    fence_barrier_init();
    prefetch_tensormap(&tmX);
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmOut);
  }
  if (a.w_off >= 0) {  // depthwise filter [k*k][C] and bias [C] resident in shared memory
    float* w_s = reinterpret_cast<float*>(smem + a.w_off);
    for (int i = threadIdx.x; i < K * K * a.C; i += R::THREADS) w_s[i] = __ldg(a.dw_w + i);
    for (int i = threadIdx.x; i < a.C; i += R::THREADS)
      w_s[K * K * a.C + i] = a.dw_bias ? __ldg(a.dw_bias + i) : 0.0f;
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: input windows
      const uint32_t xbytes = (uint32_t)(G::IH * G::IW * CW * 4);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const TileCoord tc = tile_coord(args, tile, 1, BN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sx = it % a.xs;
          if (!mbar_wait(&x_empty[sx], ((it / a.xs) & 1u) ^ 1u, args.err)) { ok = false; break; }
          fence_proxy_async_smem();  // the depthwise warps' reads of this window before the new load
          mbar_arrive_expect_tx(&x_full[sx], xbytes);
          tma_load_4d(x_ring + sx * G::X_BYTES, &tmX, &x_full[sx], kb * CW, tc.ox0 * S - args.pw,
                      tc.oy0 * S - args.ph, tc.img);
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---------------- TMA producer: pointwise filter blocks (own thread, so
      // a window waiting for its buffer never holds back the filter stream)
      if (b_resident) {
        mbar_arrive_expect_tx(&b_full[0], (uint32_t)nkb * B_BYTES);
        for (int kb = 0; kb < nkb; ++kb) tma_load_2d(b_ring + kb * B_BYTES, &tmW, &b_full[0], kb * CW, 0);
      } else {
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
          for (int kb = 0; kb < nkb; ++kb, ++it) {
            const int sb = it % a.bs;
            if (!mbar_wait(&b_empty[sb], ((it / a.bs) & 1u) ^ 1u, args.err)) { ok = false; break; }
            mbar_arrive_expect_tx(&b_full[sb], B_BYTES);
            tma_load_2d(b_ring + sb * B_BYTES, &tmW, &b_full[sb], kb * CW, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      uint32_t it = 0, acc_i = 0;
      bool ok = !b_resident || mbar_wait(&b_full[0], 0, args.err);
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++acc_i) {
        const uint32_t buf = acc_i % DW_NBUF;
        if (acc_i >= (uint32_t)DW_NBUF) {
          if (!mbar_wait(&acc_empty[buf], ((acc_i / DW_NBUF) - 1) & 1u, args.err)) { ok = false; break; }
          tc_fence_after();
        }
        const uint32_t d_tmem = tmem_d + buf * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int sa = it % a.as;
          const int sb = b_resident ? kb : (int)(it % a.bs);
          if (!mbar_wait(&a_full[sa], (it / a.as) & 1u, args.err)) { ok = false; break; }
          if (!b_resident && !mbar_wait(&b_full[sb], (it / a.bs) & 1u, args.err)) { ok = false; break; }
          const uint32_t a_addr = smem_u32(a_ring + sa * A_TILE_BYTES);
          const uint32_t b_addr = smem_u32(b_ring + sb * B_BYTES);
#pragma unroll
          for (int ks = 0; ks < CW / 8; ++ks)
            mma_tf32(d_tmem, sw128_kmajor_desc(a_addr + ks * 32), sw128_kmajor_desc(b_addr + ks * 32), idesc,
                     (kb > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&a_empty[sa]);
          if (!b_resident) mma_commit(&b_empty[sb]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else if (warp >= R::EPI0 && warp < R::DW0) {
    // ---------------- epilogue groups: TMEM lane quarter q = warp % 4; group
    // `grp` takes the CTA's tiles grp, grp + NGRP, ... (their serial
    // TMEM -> staging -> TMA-store chains overlap)
    const int q = warp & 3;
    const int grp = (warp - R::EPI0) >> 2;
    const int r = q * 32 + lane;
    const int gt = threadIdx.x - 32 * R::EPI0 - grp * 128;
    const uint32_t lane_base = tmem_d + ((uint32_t)(q * 32) << 16);
    uint8_t* my_stg = stg + grp * 2 * OUT_STAGE_BYTES;
    uint32_t acc_i = grp, chunk_ctr = 0;
    for (int tile = blockIdx.x + grp * gridDim.x; tile < total_tiles; tile += NGRP * gridDim.x, acc_i += NGRP) {
      const TileCoord tc = tile_coord(args, tile, 1, BN);
      const uint32_t buf = acc_i % DW_NBUF;
      if (!mbar_wait(&acc_full[buf], (acc_i / DW_NBUF) & 1u, args.err)) break;
      tc_fence_after();
      auto fetch = [&](int c, float (&v)[32]) {
        uint32_t x0[16], x1[16];
        tmem_ld16_nowait(lane_base + buf * BN + c, x0);
        tmem_ld16_nowait(lane_base + buf * BN + c + 16, x1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __uint_as_float(x0[j]);
          v[16 + j] = __uint_as_float(x1[j]);
        }
      };
      store_tile<BN, 1, false>(args, &tmOut, my_stg, nullptr, 1 + grp, chunk_ctr, tc.m_blk, tc.n0, tc.img, tc.oy0,
                               tc.ox0, r, gt, fetch);
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    if (gt == 0) bulk_wait_group<0>();  // the last stores out of shared memory before exit
  } else if (warp >= R::DW0) {
    // ---------------- depthwise
    const int gt = threadIdx.x - 32 * R::DW0;
    const int cp = gt & 15;                        // channel pair within the block
    const int blk = gt >> 4;                       // pixel block of the tile
    const int by = blk / G::BLOCKS_X, bx = blk % G::BLOCKS_X;
    const int py0 = by * G::BY, px0 = bx * G::BX;  // block origin in the output tile
    const float* w_s = a.w_off >= 0 ? reinterpret_cast<const float*>(smem + a.w_off) : nullptr;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int c = kb * CW + 2 * cp;
        float2 wr[K * K];
#pragma unroll
        for (int t = 0; t < K * K; ++t)
          wr[t] = w_s ? *reinterpret_cast<const float2*>(w_s + t * a.C + c)
                      : __ldg(reinterpret_cast<const float2*>(a.dw_w + t * a.C + c));
        const float2 b1 = w_s ? *reinterpret_cast<const float2*>(w_s + K * K * a.C + c)
                              : (a.dw_bias ? __ldg(reinterpret_cast<const float2*>(a.dw_bias + c))
                                           : make_float2(0.f, 0.f));
        const int sx = it % a.xs;
        if (!mbar_wait(&x_full[sx], (it / a.xs) & 1u, args.err)) { ok = false; break; }
        const float* xw = reinterpret_cast<const float*>(x_ring + sx * G::X_BYTES) +
                          ((py0 * S) * G::IW + px0 * S) * CW + 2 * cp;
        float2 acc[G::BY][G::BX];
#pragma unroll
        for (int oy = 0; oy < G::BY; ++oy)
#pragma unroll
          for (int ox = 0; ox < G::BX; ++ox) acc[oy][ox] = make_float2(0.f, 0.f);
#pragma unroll
        for (int rr = 0; rr < G::ROWS; ++rr) {
          float2 in[G::COLS];
#pragma unroll
          for (int j = 0; j < G::COLS; ++j) in[j] = *reinterpret_cast<const float2*>(xw + (rr * G::IW + j) * CW);
#pragma unroll
          for (int oy = 0; oy < G::BY; ++oy) {
            const int ky = rr - oy * S;
            if (ky < 0 || ky >= K) continue;
#pragma unroll
            for (int kx = 0; kx < K; ++kx)
#pragma unroll
              for (int ox = 0; ox < G::BX; ++ox)
                acc[oy][ox] = __ffma2_rn(wr[ky * K + kx], in[ox * S + kx], acc[oy][ox]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&x_empty[sx]);  // window read: the producer may refill it
        float v[2 * G::BY * G::BX];
#pragma unroll
        for (int oy = 0; oy < G::BY; ++oy)
#pragma unroll
          for (int ox = 0; ox < G::BX; ++ox) {
            v[2 * (oy * G::BX + ox)] = __fadd_rn(acc[oy][ox].x, b1.x);
            v[2 * (oy * G::BX + ox) + 1] = __fadd_rn(acc[oy][ox].y, b1.y);
          }
        apply_act_n(v, a.dw_act);
        const int sa = it % a.as;
        if (!mbar_wait(&a_empty[sa], ((it / a.as) & 1u) ^ 1u, args.err)) { ok = false; break; }
        uint8_t* as_ = a_ring + sa * A_TILE_BYTES;
        const int chunk = cp >> 1, word = (cp & 1) * 8;
#pragma unroll
        for (int oy = 0; oy < G::BY; ++oy)
#pragma unroll
          for (int ox = 0; ox < G::BX; ++ox) {
            const int p = (py0 + oy) * DW_TW + px0 + ox;   // MMA row
            const int j = 2 * (oy * G::BX + ox);
            *reinterpret_cast<float2*>(as_ + p * 128 + ((chunk ^ (p & 7)) << 4) + word) =
                make_float2(tf32_rna(v[j]), tf32_rna(v[j + 1]));
          }
        fence_proxy_async_smem();  // this thread's A writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, TMEM_COLS);
}

struct DwpwPlan {
  int xs = 0, as = 0, bs = 0, smem = 0;
  int b_off = 0, x_off = 0, stg_off = 0, w_off = -1;
};

// Shared-memory layout for one geometry.  The pointwise filter is resident
// when it is small (bs = 0), else streamed through a ring; then the deepest
// depthwise filter when it fits next to the minimal rings, then the deepest
// window ring (whose loads have the longest latency to hide) and A ring
// (2..4 stages each) that fit next to the output staging (two 16 KB buffers
// per epilogue group).  xs == 0: does not fit.
DwpwPlan dwpw_plan(int k, int s, int bn, int c, int ngrp) {
  DwpwPlan p;
  const int cw = 32;
  const int ih = (DW_TH - 1) * s + k, iw = (DW_TW - 1) * s + k;
  const int xb = ((ih * iw * cw * 4 + 1023) / 1024) * 1024;
  const int bb = bn * 128;
  const int nkb = c / cw;
  const bool resident = nkb * bb <= DW_B_RESIDENT_MAX;
  const int wb = (((k * k + 1) * c * 4 + 1023) / 1024) * 1024;  // filter + bias
  const int fixed = ngrp * 2 * OUT_STAGE_BYTES + 1024;  // output staging, alignment slack
  auto size = [&](int xs, int as, int bs, int w) {
    return fixed + as * A_TILE_BYTES + (resident ? nkb : bs) * bb + xs * xb + w;
  };
  int xs = 2, as = 2, bs = 2;
  if (size(xs, as, bs, 0) > DW_SMEM_BUDGET) return p;
  // a resident depthwise filter first (read from L1 it stalls every step)
  const bool w_res = size(xs, as, bs, wb) <= DW_SMEM_BUDGET;
  const int w = w_res ? wb : 0;
  while (xs < 4 && size(xs + 1, as, bs, w) <= DW_SMEM_BUDGET) ++xs;
  while (as < 4 && size(xs, as + 1, bs, w) <= DW_SMEM_BUDGET) ++as;
  while (!resident && bs < 4 && size(xs, as, bs + 1, w) <= DW_SMEM_BUDGET) ++bs;
  p.xs = xs;
  p.as = as;
  p.bs = resident ? 0 : bs;
  p.b_off = as * A_TILE_BYTES;
  p.x_off = p.b_off + (resident ? nkb : bs) * bb;
  p.stg_off = p.x_off + xs * xb;
  p.w_off = w_res ? p.stg_off + ngrp * 2 * OUT_STAGE_BYTES : -1;
  p.smem = size(xs, as, bs, w);
  return p;
}

// Epilogue groups: two for stride-1 layers up to 128 output channels, whose
// tiles carry little depthwise work (one group's serial store chain would
// pace them); one otherwise (the stride-2 windows need the shared memory).
int dwpw_ngrp(int s, int bn) { return (s == 1 && bn <= 128) ? 2 : 1; }

int dwpw_bn(int n_out) {
  return n_out <= 32 ? 32 : n_out <= 64 ? 64 : n_out <= 128 ? 128 : 256;
}

template <int K, int S, int BN, int NGRP>
cudaError_t run_dwpw(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mo, const DwpwArgs& a,
                     int smem, cudaStream_t st) {
  auto kern = dwpw_kernel<K, S, BN, NGRP>;
  if (cudaError_t e = ensure_dyn_smem((const void*)kern, smem); e != cudaSuccess) return e;
  const int grid = a.g.m_tiles < current_sm_count() ? a.g.m_tiles : current_sm_count();
  kern<<<grid, DwRoles<NGRP>::THREADS, smem, st>>>(mx, mw, mo, a);
  return cudaGetLastError();
}

template <int K, int S>
cudaError_t dispatch_bn(int bn, const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mo,
                        const DwpwArgs& a, int smem, cudaStream_t st) {
  switch (bn) {
    case 32: return run_dwpw<K, S, 32, S == 1 ? 2 : 1>(mx, mw, mo, a, smem, st);
    case 64: return run_dwpw<K, S, 64, S == 1 ? 2 : 1>(mx, mw, mo, a, smem, st);
    case 128: return run_dwpw<K, S, 128, S == 1 ? 2 : 1>(mx, mw, mo, a, smem, st);
    default: return run_dwpw<K, S, 256, 1>(mx, mw, mo, a, smem, st);
  }
}

}  // namespace

bool dwpw_ok(const ConvGeom& g, int n_out) {
  if (g.kh != g.kw || (g.kh != 3 && g.kh != 5) || g.sh != g.sw || (g.sh != 1 && g.sh != 2)) return false;
  // 16-channel inputs (one half-empty channel block per tile) measured slower
  // fused than as the two separate kernels: only whole 32-channel blocks
  if ((g.c % 32) != 0 || g.m != g.c) return false;
  if (n_out <= 0 || n_out > 256 || (n_out % 4) != 0) return false;
  if (g.ph >= g.kh || g.pw >= g.kw) return false;
  // rows of the NHWC tensors stay addressable with 32-bit tile coordinates
  if ((int64_t)g.n * g.oh * g.ow >= (int64_t)1 << 31) return false;
  // maps the 8 x 16 tiles cover poorly (the rec lines' 3-row maps: 31% of a
  // tile's rows carry outputs) do more work fused than as two kernels
  const double cover = (double)g.oh * g.ow /
                       ((double)((g.oh + DW_TH - 1) / DW_TH) * DW_TH * ((g.ow + DW_TW - 1) / DW_TW) * DW_TW);
  if (cover < 0.7) return false;
  return dwpw_plan(g.kh, g.sh, dwpw_bn(n_out), g.c, dwpw_ngrp(g.sh, dwpw_bn(n_out))).xs > 0;
}

cudaError_t launch_dwpw(const float* x, const ConvGeom& g, const float* dw_w, const float* dw_bias,
                        const ActParams& dw_act, const float* pw_w, int n_out, const GemmEpilogue& epi,
                        unsigned int* err, cudaStream_t st) {
  if (!dwpw_ok(g, n_out)) return cudaErrorNotSupported;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(pw_w) |
        reinterpret_cast<uintptr_t>(epi.out)) & 15) || (epi.ldo % 4) || epi.residual || epi.col_off)
    return cudaErrorInvalidValue;
  const int cw = 32;
  const int bn = dwpw_bn(n_out);
  const DwpwPlan p = dwpw_plan(g.kh, g.sh, bn, g.c, dwpw_ngrp(g.sh, bn));
  const int ih = (DW_TH - 1) * g.sh + g.kh, iw = (DW_TW - 1) * g.sw + g.kw;
  CUtensorMap mx, mw, mo;
  {
    const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4, (uint64_t)g.c * g.w * g.h * 4};
    const uint32_t box[4] = {(uint32_t)cw, (uint32_t)iw, (uint32_t)ih, 1};
    if (!make_tensor_map(&mx, x, 4, dims, strides, box, false)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.c, (uint64_t)n_out};
    const uint64_t strides[1] = {(uint64_t)g.c * 4};
    // 32-wide k boxes (a 16-channel filter's second half reads as zeros, which
    // no MMA uses): every filter block has the standard 128-byte swizzled rows
    const uint32_t box[2] = {32u, (uint32_t)bn};
    if (!make_tensor_map(&mw, pw_w, 2, dims, strides, box, true)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[4] = {(uint64_t)n_out, (uint64_t)g.ow, (uint64_t)g.oh, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)epi.ldo * 4, (uint64_t)epi.ldo * g.ow * 4,
                                 (uint64_t)epi.ldo * g.ow * g.oh * 4};
    const uint32_t box[4] = {32, (uint32_t)DW_TW, (uint32_t)DW_TH, 1};
    if (!make_tensor_map(&mo, epi.out, 4, dims, strides, box, true)) return cudaErrorInvalidValue;
  }
  DwpwArgs a{};
  GemmArgs& ga = a.g;
  ga.M = g.n * g.oh * g.ow;
  ga.N = n_out;
  ga.K = g.c;
  ga.err = err;
  ga.nkb = g.c / cw;
  ga.bkw = cw;
  ga.tma_store = 1;
  ga.epi = epi;
  ga.ph = g.ph;
  ga.pw = g.pw;
  ga.kw = g.kw;
  ga.oh = g.oh;
  ga.ow = g.ow;
  ga.tw = DW_TW;
  ga.th = DW_TH;
  ga.tiles_x = (g.ow + DW_TW - 1) / DW_TW;
  ga.tiles_y = (g.oh + DW_TH - 1) / DW_TH;
  ga.m_tiles = g.n * ga.tiles_x * ga.tiles_y;
  a.dw_w = dw_w;
  a.dw_bias = dw_bias;
  a.dw_act = dw_act;
  a.dw_act.round_tf32 = 0;
  a.C = g.c;
  a.xs = p.xs;
  a.as = p.as;
  a.bs = p.bs;
  a.b_off = p.b_off;
  a.x_off = p.x_off;
  a.stg_off = p.stg_off;
  a.w_off = p.w_off;
  const int k = g.kh, s = g.sh;
  if (k == 3 && s == 1) return dispatch_bn<3, 1>(bn, mx, mw, mo, a, p.smem, st);
  if (k == 3 && s == 2) return dispatch_bn<3, 2>(bn, mx, mw, mo, a, p.smem, st);
  if (k == 5 && s == 1) return dispatch_bn<5, 1>(bn, mx, mw, mo, a, p.smem, st);
  return dispatch_bn<5, 2>(bn, mx, mw, mo, a, p.smem, st);
}

}  // namespace qpc
