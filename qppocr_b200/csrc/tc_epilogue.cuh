// Shared pieces of the tcgen05 kernels (gemm_tc.cu, dwpw.cu): tile
// constants, the launch arguments, output-row maps and the tile epilogues
// (direct stores, and the shared-memory staged TMA store).
#pragma once
#include "kernels.h"

namespace qpc {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;                  // fp32 elements per 128-byte swizzle row
constexpr int A_TILE_BYTES = BM * BK * 4;
constexpr int OUT_STAGE_BYTES = BM * 32 * 4;  // one 128 x 32 fp32 output chunk (16 KB)

struct GemmArgs {
  int M, N, K;          // M = output rows (pixels/tokens), N = output channels
  unsigned int* err;    // device error word for bounded-wait timeouts
  int nkb;              // number of k-blocks
  int bkw;              // k-block width in floats: 32, or 24 (rows modes, K % 24 == 0 but K % 32 != 0:
                        // the boxes end at the tensor's edge instead of overrunning it; the
                        // 128-byte stage rows keep their layout, and 3 of 4 k-steps are issued)
  int m_tiles;          // output row tiles (128 rows each)
  int tma_store;        // 1: output tiles leave through smem staging + TMA store
  GemmEpilogue epi;
  // A_MODE 1 geometry
  int taps, kw, ph, pw, cblocks;
  int oh, ow, tw, th, tiles_x, tiles_y;
};

template <int BN>
__device__ __forceinline__ void epilogue_store(const GemmArgs& args, const float (&v)[16],
                                               int64_t orow, int64_t rrow, int col0) {
  const GemmEpilogue& e = args.epi;
  float o[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int col = col0 + j;
    o[j] = (e.bias && col < args.N) ? __fadd_rn(v[j], __ldg(e.bias + col)) : v[j];
  }
  apply_act_n(o, e.act);
  if (e.residual)
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (col0 + j < args.N) o[j] = __fadd_rn(o[j], __ldg(e.residual + rrow * e.ldr + col0 + j));
  if (e.round_out)
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = tf32_rna(o[j]);
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


// Output row (pixel / token) and residual row of tile row `r`; -1 if the row
// lies outside the output.
struct RowMap {
  int64_t orow, rrow;
};

template <int A_MODE>
__device__ __forceinline__ RowMap row_map(const GemmArgs& args, int m_blk, int img, int oy0, int ox0,
                                          int r) {
  // Row counts are below 2^31 (GemmArgs::M is an int): 32-bit index math.
  RowMap m{-1, -1};
  if (A_MODE == 0) {
    const int row = m_blk * BM + r;
    if (row < args.M) m.orow = row;
  } else {
    const int oy = oy0 + r / args.tw, ox = ox0 + r % args.tw;
    if (oy < args.oh && ox < args.ow) m.orow = ((int64_t)img * args.oh + oy) * args.ow + ox;
  }
  m.rrow = m.orow;
  const GemmEpilogue& e = args.epi;
  if (m.orow >= 0 && e.residual && e.rh > 0) {
    // nearest resize source row, resize.rs:43-50: (int)((float)o * in / out)
    const unsigned o = (unsigned)m.orow;
    const unsigned yx = o / (unsigned)e.ow;
    const int x = (int)(o - yx * (unsigned)e.ow);
    const unsigned nn = yx / (unsigned)e.oh;
    const int y = (int)(yx - nn * (unsigned)e.oh);
    int iy = (int)__fdiv_rn(__fmul_rn((float)y, (float)e.rh), (float)e.oh);
    int ix = (int)__fdiv_rn(__fmul_rn((float)x, (float)e.rw), (float)e.ow);
    iy = iy < e.rh - 1 ? iy : e.rh - 1;
    ix = ix < e.rw - 1 ? ix : e.rw - 1;
    m.rrow = ((int64_t)nn * e.rh + iy) * e.rw + ix;
  }
  return m;
}

// Epilogue of one tile through shared memory: for each 32-column chunk every
// thread finishes its own row (bias, activation, residual: its row's 128-byte
// residual segment, loaded before the TMEM fetch so the two overlap) into a
// 128B-swizzled staging buffer, and one thread writes the chunk with a TMA
// store.  Two staging buffers alternate; a buffer is rewritten only after the
// store issued from it two chunks earlier has finished reading it.
// Residual row of tile row r (-1 outside the output).
template <int A_MODE>
__device__ __forceinline__ int64_t residual_row(const GemmArgs& args, int m_blk, int img, int oy0, int ox0, int r) {
  const RowMap mine = row_map<A_MODE>(args, m_blk, img, oy0, ox0, r);
  return mine.orow >= 0 ? mine.rrow : -1;
}

// The 32 residual values of row `rrow`, columns col0..col0+31 (zeros past N).
__device__ __forceinline__ void load_residual(const GemmArgs& args, int64_t rrow, int col0, float4 (&rv)[8]) {
  const float* rp = args.epi.residual + rrow * args.epi.ldr + col0;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    rv[k] = (rrow >= 0 && col0 + 4 * k < args.N) ? __ldg(reinterpret_cast<const float4*>(rp) + k)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
}

// RES = false: the caller never passes a residual (saves its registers).
// BIAS = false: `fetch` has already added the bias.
template <int BN, int A_MODE, bool RES = true, bool BIAS = true, class Fetch>
__device__ __forceinline__ void store_tile(const GemmArgs& args, const CUtensorMap* tm_out,
                                           uint8_t* stage, int64_t* s_rrow, int bar_id,
                                           uint32_t& chunk_ctr, int m_blk, int n0, int img, int oy0,
                                           int ox0, int r, int t, Fetch&& fetch) {
  (void)s_rrow;
  const GemmEpilogue& e = args.epi;
  const int64_t rrow = (RES && e.residual) ? residual_row<A_MODE>(args, m_blk, img, oy0, ox0, r) : -1;
#pragma unroll 1
  for (int cc = 0; cc < BN; cc += 32) {
    if (n0 + cc >= args.N) break;
    float* sb = reinterpret_cast<float*>(stage + (chunk_ctr & 1u) * OUT_STAGE_BYTES);
    // Everything that does not touch the staging buffer first (residual
    // loads, TMEM fetch, bias, activation, residual add), so it overlaps the
    // wait for the store issued from this buffer two chunks ago.
    float4 rv[8];
    if constexpr (RES) {
      if (e.residual) load_residual(args, rrow, n0 + cc, rv);
    }
    float v[32];
    fetch(cc, v);
    if (BIAS && e.bias) {
      // columns past N are clipped by the TMA store; keep their reads in bounds
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const int col = n0 + cc + j;
        if (col < args.N) {
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(e.bias + col));
          v[j] = __fadd_rn(v[j], b4.x);
          v[j + 1] = __fadd_rn(v[j + 1], b4.y);
          v[j + 2] = __fadd_rn(v[j + 2], b4.z);
          v[j + 3] = __fadd_rn(v[j + 3], b4.w);
        }
      }
    }
    apply_act_n(v, e.act);
    if (RES && e.residual) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 q = rv[k];
        v[4 * k] = __fadd_rn(v[4 * k], q.x);
        v[4 * k + 1] = __fadd_rn(v[4 * k + 1], q.y);
        v[4 * k + 2] = __fadd_rn(v[4 * k + 2], q.z);
        v[4 * k + 3] = __fadd_rn(v[4 * k + 3], q.w);
      }
    }
    if (t == 0) bulk_wait_group_read<1>();
    named_bar_sync(bar_id, 128);  // staging buffer free
    float* myrow = sb + r * 32;
    if (e.round_out)
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tf32_rna(v[j]);
#pragma unroll
    for (int c4 = 0; c4 < 8; ++c4)
      *reinterpret_cast<float4*>(myrow + ((c4 ^ (r & 7)) << 2)) =
          make_float4(v[c4 * 4], v[c4 * 4 + 1], v[c4 * 4 + 2], v[c4 * 4 + 3]);
    fence_proxy_async_smem();
    named_bar_sync(bar_id, 128);
    if (t == 0) {
      if (A_MODE == 0) tma_store_2d(tm_out, sb, n0 + cc, m_blk * BM);
      else tma_store_4d(tm_out, sb, n0 + cc, ox0, oy0, img);
      bulk_commit_group();
    }
    ++chunk_ctr;
  }
}


// Output tile of a flat tile index: row block, first column, and for the 4-D
// (image, row, column) tilings the tile's image and top-left output pixel.
struct TileCoord {
  int m_blk, n0, img, oy0, ox0;
};

__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& a, int tile, int n_tiles, int bn) {
  TileCoord c;
  c.m_blk = tile / n_tiles;
  c.n0 = (tile % n_tiles) * bn;
  c.img = c.oy0 = c.ox0 = 0;
  if (a.tiles_x > 0) {
    const int per_img = a.tiles_x * a.tiles_y;
    c.img = c.m_blk / per_img;
    const int rem = c.m_blk % per_img;
    c.oy0 = (rem / a.tiles_x) * a.th;
    c.ox0 = (rem % a.tiles_x) * a.tw;
  }
  return c;
}

}  // namespace
}  // namespace qpc
