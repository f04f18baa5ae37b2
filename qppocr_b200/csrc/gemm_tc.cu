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
// * Epilogue: warps 2-5 read their 32 TMEM lanes (tcgen05.ld 32x32b), add bias,
//   apply the fused activation, add the residual (optionally through a
//   nearest-upsample index map) and store fp32 rows.
// * A_MODE 1 (k x k, stride 1 conv): the A tile is a 4-D TMA box
//   [1][TH][TW][32ch] of the NHWC input shifted by the tap offset; rows and
//   columns outside the image are zero-filled by TMA, which is exactly the
//   conv's zero padding.  k order is tap-major then channel.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.h"

namespace qpc {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;                  // fp32 elements per 128-byte swizzle row
constexpr int A_TILE_BYTES = BM * BK * 4;

struct GemmArgs {
  int M, N, K;          // M = output rows (pixels/tokens), N = output channels
  unsigned int* err;    // device error word for bounded-wait timeouts
  int nkb;              // number of 32-wide k-blocks
  GemmEpilogue epi;
  // A_MODE 1 geometry
  int taps, kw, ph, pw, cblocks;
  int oh, ow, tw, th, tiles_x, tiles_y;
};

template <int BN, bool SPLIT>
struct Smem {
  static constexpr int B_TILE = BN * BK * 4;
  static constexpr int STAGE = A_TILE_BYTES + B_TILE + (SPLIT ? (A_TILE_BYTES + B_TILE) : 0);
};

template <int BN>
__device__ __forceinline__ void epilogue_store(const GemmArgs& args, const float (&v)[16],
                                               int64_t orow, int64_t rrow, int col0) {
  const GemmEpilogue& e = args.epi;
  float o[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = col0 + j;
    float t = v[j];
    if (col < args.N) {
      if (e.bias) t = __fadd_rn(t, __ldg(e.bias + col));
      t = apply_act(t, e.act);
      if (e.residual) t = __fadd_rn(t, __ldg(e.residual + rrow * e.ldr + col));
    }
    o[j] = t;
  }
  float* dst = e.out + orow * e.ldo + e.col_off + col0;
  const bool vec_ok = ((e.ldo | e.col_off) & 3) == 0 && col0 + 16 <= args.N;
  if (vec_ok) {
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      *reinterpret_cast<float4*>(dst + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (col0 + j < args.N) dst[j] = o[j];
  }
}

constexpr int NUM_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 convert + epilogue
constexpr int CH = 1;             // k-blocks per promotion chunk (3xTF32)
constexpr int LAG = 1;            // converter runs this many k-blocks ahead of a drain

template <int BN, int STAGES, bool SPLIT, int A_MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmBlo, const GemmArgs args) {
  using SM = Smem<BN, SPLIT>;
  // 3xTF32 ping-pongs two accumulators so the MMA runs on while a chunk drains.
  constexpr uint32_t TMEM_COLS = SPLIT ? 2 * BN : (BN < 32 ? 32 : BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t conv_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ __align__(8) uint64_t chunk_full[2];
  __shared__ __align__(8) uint64_t chunk_free[2];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Tile coordinates.  Consecutive CTAs walk the N tiles of one M block so
  // the A rows they share are still in L2.
  const int n_tiles = (args.N + BN - 1) / BN;
  const int m_blk = blockIdx.x / n_tiles;
  const int n_blk = blockIdx.x % n_tiles;
  const int n0 = n_blk * BN;
  int img = 0, oy0 = 0, ox0 = 0;
  if (A_MODE == 1) {
    const int per_img = args.tiles_x * args.tiles_y;
    img = m_blk / per_img;
    const int rem = m_blk % per_img;
    oy0 = (rem / args.tiles_x) * args.th;
    ox0 = (rem % args.tiles_x) * args.tw;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], 128);
    }
    mbar_init(&acc_bar, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&chunk_full[b], 1);
      mbar_init(&chunk_free[b], 128);
    }
    abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    if (SPLIT) prefetch_tensormap(&tmBlo);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base_slot;
  const int nkb = args.nkb;
  const int nchunks = (nkb + CH - 1) / CH;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      const uint32_t bytes = SPLIT ? (A_TILE_BYTES + 2 * SM::B_TILE) : (A_TILE_BYTES + SM::B_TILE);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        if (!mbar_wait(&empty_bar[s], ph ^ 1u, args.err)) { abort_flag = 1; break; }
        uint8_t* st = smem + s * SM::STAGE;
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        if (A_MODE == 0) {
          tma_load_2d(st, &tmA, &full_bar[s], kb * BK, m_blk * BM);
          tma_load_2d(st + A_TILE_BYTES, &tmB, &full_bar[s], kb * BK, n0);
          if (SPLIT) tma_load_2d(st + 2 * A_TILE_BYTES + SM::B_TILE, &tmBlo, &full_bar[s], kb * BK, n0);
        } else {
          const int tap = kb / args.cblocks, cb = kb % args.cblocks;
          const int ky = tap / args.kw, kx = tap % args.kw;
          tma_load_4d(st, &tmA, &full_bar[s], cb * BK, ox0 + kx - args.pw, oy0 + ky - args.ph, img);
          tma_load_4d(st + A_TILE_BYTES, &tmB, &full_bar[s], cb * BK, n0, tap, 0);
          if (SPLIT)
            tma_load_4d(st + 2 * A_TILE_BYTES + SM::B_TILE, &tmBlo, &full_bar[s], cb * BK, n0, tap, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        const bool first = SPLIT ? (kb % CH) == 0 : kb == 0;
        const int chunk = kb / CH, buf = chunk & 1;
        // accumulator `buf` is reused by chunk c once chunk c - 2 has drained
        if (SPLIT && first && chunk >= 2 &&
            !mbar_wait(&chunk_free[buf], (uint32_t)((chunk >> 1) - 1) & 1u, args.err)) {
          ok = false;
          break;
        }
        const uint32_t d_tmem = tmem_d + (SPLIT ? (uint32_t)(buf * BN) : 0u);
        if (!mbar_wait(&conv_bar[s], ph, args.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * SM::STAGE);
        const uint32_t b_addr = a_addr + A_TILE_BYTES;
#pragma unroll
        for (int ks = 0; ks < BK / 8; ++ks) {
          const uint32_t acc = (!first || ks > 0) ? 1u : 0u;
          const uint64_t ad = sw128_kmajor_desc(a_addr + ks * 32);
          const uint64_t bd = sw128_kmajor_desc(b_addr + ks * 32);
          if (SPLIT) {
            const uint64_t alo = sw128_kmajor_desc(b_addr + SM::B_TILE + ks * 32);
            const uint64_t blo = sw128_kmajor_desc(b_addr + SM::B_TILE + A_TILE_BYTES + ks * 32);
            mma_tf32(d_tmem, alo, bd, idesc, acc);
            mma_tf32(d_tmem, ad, blo, idesc, 1u);
            mma_tf32(d_tmem, ad, bd, idesc, 1u);
          } else {
            mma_tf32(d_tmem, ad, bd, idesc, acc);
          }
        }
        mma_commit(&empty_bar[s]);   // frees the stage once these MMAs have read it
        if (SPLIT && ((kb % CH) == CH - 1 || kb == nkb - 1)) mma_commit(&chunk_full[buf]);
      }
      if (!ok) abort_flag = 1;
      if (!SPLIT) mma_commit(&acc_bar);   // accumulator complete (or abandoned)
    }
  } else {
    // ---------------- warps 2-5: convert A on chip, then the epilogue.
    // TMEM lane quarter of this warp = warp % 4; its rows are 32 * (warp % 4) + lane.
    const int t = threadIdx.x - 64;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem_d + ((uint32_t)(q * 32) << 16);
    float accr[SPLIT ? BN : 1];
#pragma unroll
    for (int j = 0; j < (SPLIT ? BN : 1); ++j) accr[j] = 0.f;
    bool ok = true;
    int drained = 0;
    // Promotion of a finished chunk: TMEM partial sum -> fp32 registers (RN adds).
    auto drain = [&](int c) {
      const int b = c & 1;
      if (!ok || !mbar_wait(&chunk_full[b], (uint32_t)(c >> 1) & 1u, args.err)) { ok = false; return; }
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < (SPLIT ? BN : 16); c0 += 16) {
        uint32_t v[16];
        tmem_ld16_nowait(lane_base + (uint32_t)(b * BN) + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          accr[(c0 + j) % (SPLIT ? BN : 1)] =
              __fadd_rn(accr[(c0 + j) % (SPLIT ? BN : 1)], __uint_as_float(v[j]));
      }
      tc_fence_before();
      mbar_arrive(&chunk_free[b]);
    };
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!mbar_wait(&full_bar[s], ph, args.err)) { ok = false; break; }
      float4* a = reinterpret_cast<float4*>(smem + s * SM::STAGE);
      float4* lo = reinterpret_cast<float4*>(smem + s * SM::STAGE + A_TILE_BYTES + SM::B_TILE);
#pragma unroll
      for (int i = t; i < A_TILE_BYTES / 16; i += 128) {
        const float4 v = a[i];
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
      fence_proxy_async_smem();
      mbar_arrive(&conv_bar[s]);
      if (SPLIT)
        while (ok && drained < nchunks && min((drained + 1) * CH, nkb) - 1 <= kb - LAG) drain(drained++);
    }
    if (SPLIT)
      while (ok && drained < nchunks) drain(drained++);
    if (!SPLIT) ok = ok && mbar_wait(&acc_bar, 0, args.err);
    tc_fence_after();
    if (ok && !abort_flag) {
      int64_t orow = -1, rrow = -1;
      if (A_MODE == 0) {
        const int64_t m = (int64_t)m_blk * BM + r;
        if (m < args.M) orow = m;
      } else {
        const int oy = oy0 + r / args.tw, ox = ox0 + r % args.tw;
        if (oy < args.oh && ox < args.ow) orow = ((int64_t)img * args.oh + oy) * args.ow + ox;
      }
      if (orow >= 0) {
        rrow = orow;
        const GemmEpilogue& e = args.epi;
        if (e.residual && e.rh > 0) {
          // nearest resize source row, resize.rs:43-50: (int)((float)o * in / out)
          const int64_t pix = orow;
          const int x = (int)(pix % e.ow);
          const int y = (int)((pix / e.ow) % e.oh);
          const int64_t nn = pix / ((int64_t)e.ow * e.oh);
          int iy = (int)__fdiv_rn(__fmul_rn((float)y, (float)e.rh), (float)e.oh);
          int ix = (int)__fdiv_rn(__fmul_rn((float)x, (float)e.rw), (float)e.ow);
          iy = iy < e.rh - 1 ? iy : e.rh - 1;
          ix = ix < e.rw - 1 ? ix : e.rw - 1;
          rrow = (nn * e.rh + iy) * e.rw + ix;
        }
      }
      if (SPLIT) {
#pragma unroll
        for (int c = 0; c < BN; c += 16) {
          if (n0 + c < args.N && orow >= 0) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = accr[(c + j) % (SPLIT ? BN : 1)];
            epilogue_store<BN>(args, v, orow, rrow, n0 + c);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          if (n0 + c >= args.N) break;
          float v[16];
          tmem_ld16(lane_base + c, v);   // warp-collective; every lane participates
          if (orow >= 0) epilogue_store<BN>(args, v, orow, rrow, n0 + c);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, TMEM_COLS);
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

// fp32 tensor map, 128-byte swizzle, zero fill out of bounds.
// dims / box innermost first; strides in bytes for dims 1..rank-1.
bool make_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box) {
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
                  gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int STAGES, bool SPLIT, int A_MODE>
cudaError_t run_kernel(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& blo,
                       const GemmArgs& args, int grid, cudaStream_t st) {
  auto kern = gemm_tc_kernel<BN, STAGES, SPLIT, A_MODE>;
  const int smem = STAGES * Smem<BN, SPLIT>::STAGE + 1024;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  kern<<<grid, NUM_THREADS, smem, st>>>(a, b, blo, args);
  return cudaGetLastError();
}

template <int A_MODE>
cudaError_t dispatch(int bn, bool split, const CUtensorMap& a, const CUtensorMap& b,
                     const CUtensorMap& blo, const GemmArgs& args, int grid_m, cudaStream_t st) {
  const int grid = grid_m * ((args.N + bn - 1) / bn);
  if (!split) {
    switch (bn) {
      case 32: return run_kernel<32, 4, false, A_MODE>(a, b, blo, args, grid, st);
      case 64: return run_kernel<64, 4, false, A_MODE>(a, b, blo, args, grid, st);
      case 128: return run_kernel<128, 3, false, A_MODE>(a, b, blo, args, grid, st);
      default: return run_kernel<256, 3, false, A_MODE>(a, b, blo, args, grid, st);
    }
  }
  switch (bn) {
    case 32: return run_kernel<32, 4, true, A_MODE>(a, b, blo, args, grid, st);
    case 64: return run_kernel<64, 4, true, A_MODE>(a, b, blo, args, grid, st);
    default: return run_kernel<128, 3, true, A_MODE>(a, b, blo, args, grid, st);
  }
}

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

}  // namespace

cudaError_t launch_gemm_tc(const float* a, int64_t M, int K, int lda, const float* b,
                           const float* b_lo, int N, const GemmEpilogue& epi, int math,
                           unsigned int* err, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  if ((K & 3) || (lda & 3) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (reinterpret_cast<uintptr_t>(b) & 15))
    return cudaErrorInvalidValue;
  const bool split = math == MATH_3XTF32;
  if (split && !b_lo) return cudaErrorInvalidValue;
  const int bn = pick_bn(N, split);
  CUtensorMap ma, mb, mblo;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lda * 4};
    const uint32_t box[2] = {BK, BM};
    if (!make_map(&ma, a, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K * 4};
    const uint32_t box[2] = {BK, (uint32_t)bn};
    if (!make_map(&mb, b, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (split && !make_map(&mblo, b_lo, 2, dims, strides, box)) return cudaErrorInvalidValue;
    if (!split) mblo = mb;
  }
  GemmArgs args{};
  args.M = (int)M;
  args.N = N;
  args.K = K;
  args.nkb = (K + BK - 1) / BK;
  args.epi = epi;
  args.err = err;
  const int grid_m = (int)((M + BM - 1) / BM);
  return dispatch<0>(bn, split, ma, mb, mblo, args, grid_m, st);
}

cudaError_t launch_conv_tc(const float* x, const ConvGeom& g, const float* wk, const float* wk_lo,
                           const GemmEpilogue& epi, int math, unsigned int* err,
                           cudaStream_t st) {
  if (g.sh != 1 || g.sw != 1 || (g.c & 3)) return cudaErrorInvalidValue;
  const bool split = math == MATH_3XTF32;
  if (split && !wk_lo) return cudaErrorInvalidValue;
  // Tile shape TH x TW = 128 output pixels; choose TW to waste the fewest.
  int best_tw = 16;
  int64_t best_cost = INT64_MAX;
  for (int tw = 8; tw <= 128; tw *= 2) {
    const int th = 128 / tw;
    const int64_t cost = (int64_t)((g.ow + tw - 1) / tw) * tw * ((g.oh + th - 1) / th) * th;
    if (cost < best_cost) { best_cost = cost; best_tw = tw; }
  }
  const int tw = best_tw, th = 128 / tw;
  const int bn = pick_bn(g.m, split);
  CUtensorMap ma, mb, mblo;
  {
    const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4,
                                 (uint64_t)g.c * g.w * g.h * 4};
    const uint32_t box[4] = {BK, (uint32_t)tw, (uint32_t)th, 1};
    if (!make_map(&ma, x, 4, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const int taps = g.kh * g.kw;
    const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.m, (uint64_t)taps, 1};
    const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.m * 4,
                                 (uint64_t)g.c * g.m * taps * 4};
    const uint32_t box[4] = {BK, (uint32_t)bn, 1, 1};
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
  args.nkb = args.taps * args.cblocks;
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
  const int grid_m = g.n * args.tiles_x * args.tiles_y;
  return dispatch<1>(bn, split, ma, mb, mblo, args, grid_m, st);
}

}  // namespace qpc
