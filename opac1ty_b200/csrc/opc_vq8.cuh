// opc_vq8.cuh -- sub_vector_size 8 (true vector quantization): every 2-bit index selects one of
// a row's four 8-element fp16 codebook vectors (dequant_gemv.metal:31-37, 81-87 with svs = 8;
// dequantize_layer, opacc1ty/export/converter.py:26-67: W[r, 8g:8g+8] = cb[r][idx[r][g]]).
// The weights are ~0.27 bits each, so the GEMV reads little and is bound by the selection and
// multiply work; it runs on the fp16 tensor path:
//
//  * layout: a 16-row tile x 256-column block is one 128-byte index unit.  Lane l = 4g+q of a
//    warp reads the 16 bytes of row pair g (all four q-lanes the same bytes); byte s of word w
//    describes k16 step 4w+s of the block: bits 0-1 / 2-3 the indices of row g for the step's
//    first / second 8 columns, bits 4-5 / 6-7 the same for row g+8.
//  * codebooks: per tile, lane l holds 8 words: word c (0..3) = row g's vector c at halves
//    (2q, 2q+1), word 4+c the same for row g+8.  An m16n8k16 A-fragment register is one of four
//    such words, chosen by a 2-bit index: a 4-way select, no memory lookup.
//  * x is staged once per CTA in shared memory (nc batch columns, the B fragments' columns).
//  * one CTA per row tile (8 warps splitting the k blocks, the next block's index unit loaded
//    ahead) and per nc batch columns; warps reduce in a fixed order through shared memory
//    (deterministic); outlier rows (zero codebooks, masked out) are computed by extra CTAs on the
//    same tensor path, their A fragments loaded block by block from the row-major fp16 copies.
#pragma once

#include "opc_device.cuh"

namespace opc {

constexpr int kVq8BlockCols = 256;     // k columns per index unit
constexpr int kVq8UnitBytes = 128;     // 16 rows x 32 groups x 2 bits
constexpr int kVq8CbTileBytes = 1024;  // 16 rows x 4 vectors x 8 fp16
constexpr int kVq8Warps = 8;

constexpr int kVq8XsMaxBytes = 96 * 1024;  // staged x per CTA

struct Vq8Args {
  const uint4* units;      // [MT][KB] index units (16 bytes per row pair g)
  const uint4* cb;         // [MT][32 lanes][2] codebook words
  const uint16_t* tile_mask;
  const __half* orows;     // [slots][K_pad] fp16 outlier rows (zero past K)
  const int32_t* orow;     // [slots] output row, -1 = padding
  const __half* x;
  __half* y;
  int64_t ldx, ldy;
  int32_t M, K, K_pad, MT, KB, OT, batch;
  int32_t nc;              // batch columns per CTA (1, 2, 4 or 8): x[nc][K_pad] staged in smem
  int32_t x_vec16;         // x rows 16-byte loadable
};

// 4-way select of a codebook word by a 2-bit index
__device__ __forceinline__ uint32_t vq8_sel(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t i) {
  const uint32_t lo = (i & 1u) ? c1 : c0;
  const uint32_t hi = (i & 1u) ? c3 : c2;
  return (i & 2u) ? hi : lo;
}

// Grid: x = MT packed tiles + OT outlier tiles, y = batch chunks of nc columns.  Dynamic shared
// memory: x[nc][K_pad + 8] fp16 (the +8 halves make the B-fragment reads conflict-free).
__global__ void __launch_bounds__(kVq8Warps * 32) vq8_gemv_kernel(const Vq8Args a) {
  extern __shared__ __align__(16) unsigned char vq8_smem[];
  __shared__ float red[kVq8Warps][32][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.y * a.nc;
  const int ncols = min(a.nc, a.batch - n0);
  const int xstride = a.K_pad + 8;
  __half* xs = reinterpret_cast<__half*>(vq8_smem);
  const bool packed = blockIdx.x < a.MT;
  const int t = packed ? blockIdx.x : blockIdx.x - a.MT;
  // the tile's codebook words and this warp's first index unit: issued before staging x, so the
  // three memory round trips overlap
  uint4 c01 = make_uint4(0, 0, 0, 0), c23 = make_uint4(0, 0, 0, 0), iw = make_uint4(0, 0, 0, 0);
  const uint4* ub = a.units + static_cast<int64_t>(t) * a.KB * 8 + g;
  if (packed) {
    c01 = ld_nc_v4(a.cb + (static_cast<int64_t>(t) * 32 + lane) * 2);
    c23 = ld_nc_v4(a.cb + (static_cast<int64_t>(t) * 32 + lane) * 2 + 1);
    if (warp < a.KB) iw = ld_nc_v4(ub + warp * 8);
  }
  // stage this CTA's batch columns of x (zero past K)
  const int chunks = a.K_pad / 8;
  for (int i = threadIdx.x; i < ncols * chunks; i += blockDim.x) {
    const int n = i / chunks, k = (i - n * chunks) * 8;
    const __half* src = a.x + static_cast<int64_t>(n0 + n) * a.ldx + k;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (k + 8 <= a.K && a.x_vec16) {
      v = ld_nc_v4(src);
    } else if (k < a.K) {
      uint32_t h[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = (k + e < a.K) ? ld_nc_u16(src + e) : 0u;
      v = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    }
    *reinterpret_cast<uint4*>(xs + n * xstride + k) = v;
  }
  __syncthreads();
  const bool live_col = g < ncols;  // this lane's B-fragment column
  const uint32_t xrow = smem_u32(xs + (live_col ? g : 0) * xstride) + 4 * q;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (packed) {
    // c01/c23: this lane's 8 codebook words (rows g, g+8; pair q of every vector)
    for (int kb = warp; kb < a.KB; kb += kVq8Warps) {
      const uint4 nxt = kb + kVq8Warps < a.KB ? ld_nc_v4(ub + (kb + kVq8Warps) * 8) : iw;  // next block's unit
      const uint32_t words[4] = {iw.x, iw.y, iw.z, iw.w};
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        const uint32_t byte = (words[s >> 2] >> (8 * (s & 3))) & 0xffu;
        const uint32_t xa = xrow + 2 * (kb * kVq8BlockCols + 16 * s);
        uint32_t A[4];
        A[0] = vq8_sel(c01.x, c01.y, c01.z, c01.w, byte & 3u);          // row g,   k, k+1
        A[1] = vq8_sel(c23.x, c23.y, c23.z, c23.w, (byte >> 4) & 3u);   // row g+8, k, k+1
        A[2] = vq8_sel(c01.x, c01.y, c01.z, c01.w, (byte >> 2) & 3u);   // row g,   k+8, k+9
        A[3] = vq8_sel(c23.x, c23.y, c23.z, c23.w, byte >> 6);          // row g+8, k+8, k+9
        const uint32_t b0 = live_col ? lds32(xa) : 0u, b1 = live_col ? lds32(xa + 16) : 0u;
        mma16816(acc, A, b0, b1);
      }
      iw = nxt;
    }
  } else {
    // outlier tile t: A fragments straight from the row-major fp16 rows, a block at a time
    const __half* w0 = a.orows + static_cast<int64_t>(16 * t + g) * a.K_pad + 2 * q;
    const __half* w1 = w0 + static_cast<int64_t>(8) * a.K_pad;
    for (int kb = warp; kb < a.KB; kb += kVq8Warps) {
      uint32_t Ab[16][4];
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        const int k = kb * kVq8BlockCols + 16 * s;
        Ab[s][0] = ld_nc_u32(w0 + k);
        Ab[s][1] = ld_nc_u32(w1 + k);
        Ab[s][2] = ld_nc_u32(w0 + k + 8);
        Ab[s][3] = ld_nc_u32(w1 + k + 8);
      }
#pragma unroll
      for (int s = 0; s < 16; ++s) {
        const uint32_t xa = xrow + 2 * (kb * kVq8BlockCols + 16 * s);
        const uint32_t b0 = live_col ? lds32(xa) : 0u, b1 = live_col ? lds32(xa + 16) : 0u;
        mma16816(acc, Ab[s], b0, b1);
      }
    }
  }
  // fixed-order reduction over the warps (deterministic)
#pragma unroll
  for (int r = 0; r < 4; ++r) red[warp][lane][r] = acc[r];
  __syncthreads();
  if (warp != 0) return;
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < kVq8Warps; ++w)
#pragma unroll
    for (int r = 0; r < 4; ++r) sum[r] += red[w][lane][r];
  // C fragment: sum[0], sum[1] = row g, columns 2q, 2q+1; sum[2], sum[3] = row g+8
  const uint32_t mask = packed ? a.tile_mask[t] : 0u;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int ri = g + 8 * (r >> 1);
    const int n = n0 + 2 * q + (r & 1);
    if (n >= n0 + ncols) continue;
    int row;
    if (packed) {
      row = 16 * t + ri;
      if (row >= a.M || ((mask >> ri) & 1u)) continue;
    } else {
      row = a.orow[16 * t + ri];
      if (row < 0) continue;
    }
    a.y[static_cast<int64_t>(n) * a.ldy + row] = __float2half_rn(sum[r]);
  }
}

// ------------------------------------------------------------------ load-time repack
struct Vq8Geom {
  int32_t M, K, K_pad, MT, KB, n_slots;
};

// indices [M][K/8] uint8 (0..3) -> index units; one thread per 32-bit word of a unit
__global__ void vq8_repack_indices_kernel(Vq8Geom G, const uint8_t* idx, uint32_t* units, int* bad) {
  const int64_t n_words = static_cast<int64_t>(G.MT) * G.KB * 32;
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (wi >= n_words) return;
  const int w = static_cast<int>(wi & 3), g = static_cast<int>((wi >> 2) & 7);
  const int64_t tk = wi >> 5;
  const int kb = static_cast<int>(tk % G.KB), t = static_cast<int>(tk / G.KB);
  const int groups = G.K / 8;
  uint32_t v = 0;
#pragma unroll
  for (int s4 = 0; s4 < 4; ++s4) {
    const int step = 4 * w + s4;
    const int gr0 = kb * (kVq8BlockCols / 8) + 2 * step;  // group of the step's first 8 columns
#pragma unroll
    for (int f = 0; f < 4; ++f) {  // (row g, gr0), (row g, gr0+1), (row g+8, gr0), (row g+8, gr0+1)
      const int row = 16 * t + g + 8 * (f >> 1);
      const int gr = gr0 + (f & 1);
      uint32_t code = 0;
      if (row < G.M && gr < groups) {
        const uint32_t v8 = idx[static_cast<int64_t>(row) * groups + gr];
        if (v8 > 3u) atomicExch(bad, 1);
        code = v8 & 3u;
      }
      v |= code << (8 * s4 + 2 * f);
    }
  }
  units[wi] = v;
}

// codebooks [M][4][8] fp16 -> per-tile lane words; outlier rows (tile_mask) get zeros
__global__ void vq8_repack_codebooks_kernel(Vq8Geom G, const uint16_t* cb, const uint16_t* tile_mask, uint32_t* out) {
  const int64_t n_words = static_cast<int64_t>(G.MT) * 32 * 8;
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (wi >= n_words) return;
  const int word = static_cast<int>(wi & 7), lane = static_cast<int>((wi >> 3) & 31);
  const int t = static_cast<int>(wi >> 8);
  const int g = lane >> 2, q = lane & 3;
  const int c = word & 3, row = 16 * t + g + 8 * (word >> 2);
  uint32_t v = 0;
  if (row < G.M && !((tile_mask[t] >> (row & 15)) & 1u)) {
    const uint16_t* vec = cb + (static_cast<int64_t>(row) * 4 + c) * 8;
    v = static_cast<uint32_t>(vec[2 * q]) | (static_cast<uint32_t>(vec[2 * q + 1]) << 16);
  }
  out[wi] = v;
}

// outlier rows: slot s <- source row src[s] of the outlier values (fp16 [n][K]), K padded
__global__ void vq8_repack_outliers_kernel(Vq8Geom G, const uint16_t* ov, const int32_t* src, uint16_t* orows) {
  const int64_t n = static_cast<int64_t>(G.n_slots) * G.K_pad;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int s = static_cast<int>(i / G.K_pad), k = static_cast<int>(i % G.K_pad);
  const int r = src[s];
  orows[i] = (r >= 0 && k < G.K) ? ov[static_cast<int64_t>(r) * G.K + k] : static_cast<uint16_t>(0);
}

// W_hat [M][K] fp16 from the repacked form (bit-exact: every weight is a stored fp16 value)
__global__ void vq8_dequant_kernel(Vq8Geom G, const uint32_t* units, const uint32_t* cbw, const uint16_t* tile_mask,
                                   const uint16_t* orows, const int32_t* orow, __half* w, int64_t ldw) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(G.M) * G.K) return;
  const int row = static_cast<int>(i / G.K), k = static_cast<int>(i % G.K);
  const int t = row >> 4, ri = row & 15, g = ri & 7, hi = ri >> 3;
  uint16_t v;
  if ((tile_mask[t] >> ri) & 1u) {
    int s = 0;
    while (s < G.n_slots && orow[s] != row) ++s;  // load-time check path only
    v = s < G.n_slots ? orows[static_cast<int64_t>(s) * G.K_pad + k] : static_cast<uint16_t>(0);
  } else {
    const int kb = k / kVq8BlockCols, kin = k % kVq8BlockCols;
    const int step = kin >> 4, second = (kin >> 3) & 1, q = (kin & 7) >> 1;
    const uint32_t word = units[(static_cast<int64_t>(t) * G.KB + kb) * 32 + g * 4 + (step >> 2)];
    const uint32_t code = (word >> (8 * (step & 3) + 2 * (2 * hi + second))) & 3u;
    const uint32_t cw = cbw[(static_cast<int64_t>(t) * 32 + (4 * g + q)) * 8 + 4 * hi + code];
    v = static_cast<uint16_t>((kin & 1) ? (cw >> 16) : (cw & 0xffffu));
  }
  w[static_cast<int64_t>(row) * ldw + k] = __ushort_as_half(v);
}

}  // namespace opc
