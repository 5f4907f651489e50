// opc_layer.cuh -- load-time repack of a .bf2 layer into the streamed device layout, and the
// bit-exact dequantization kernel used to prove that layout against the reference.
#pragma once

#include "opc_device.cuh"

namespace opc {

struct LayerGeom {
  int64_t Up, U;
  int32_t M, K, K_pad, M_pad, MT, KT, OT, KO;
};

// indices [M][K] uint8 (svs == 1) -> packed units.  One thread per 32-bit output word.
__global__ void repack_indices_kernel(LayerGeom G, const uint8_t* __restrict__ idx, uint32_t* __restrict__ out,
                                      int* __restrict__ bad) {
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n_words = G.Up * (kUnitBytes / 4);
  if (wi >= n_words) return;
  const int64_t unit = wi / (kUnitBytes / 4);
  const int within = static_cast<int>(wi % (kUnitBytes / 4));
  const int lane = within >> 2, j = within & 3;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t = unit / G.KT;
  const int kt = static_cast<int>(unit % G.KT);
  uint32_t word = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int o = 0; o < 2; ++o) {
        const int64_t row = t * kTileRows + g + 8 * (r & 1);
        const int col = kt * kPackedCols + (2 * j + h) * 16 + 4 * q + 2 * (r >> 1) + o;
        uint32_t v = 0;
        if (row < G.M && col < G.K) {
          v = idx[row * G.K + col];
          if (v > 3u) atomicExch(bad, 1);
        }
        word |= (v & 3u) << field_shift(r, h, o);
      }
  out[wi] = word;
}

// codebooks [M][4] fp16 (svs == 1) -> split form; outlier and padding rows are zero.
__global__ void repack_codebooks_kernel(LayerGeom G, const uint16_t* __restrict__ cb,
                                        const uint16_t* __restrict__ tile_mask, uint2* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= G.M_pad) return;
  uint2 v = make_uint2(0u, 0u);
  const bool outlier = (tile_mask[r / kTileRows] >> (r % kTileRows)) & 1u;
  if (r < G.M && !outlier) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t h = cb[r * 4 + c];
      v.x |= (h & 0xffu) << (8 * c);
      v.y |= (h >> 8) << (8 * c);
    }
  }
  out[r] = v;
}

// outlier rows [n][K] fp16 -> dense units in A-fragment order.  slot_src[s] is the source row
// (in the outlier value array) of outlier slot s, or -1 for padding slots.
__global__ void repack_outliers_kernel(LayerGeom G, const uint16_t* __restrict__ ov,
                                       const int32_t* __restrict__ slot_src, uint32_t* __restrict__ out) {
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n_words = (G.U - G.Up) * (kUnitBytes / 4);
  if (wi >= n_words) return;
  const int64_t unit = wi / (kUnitBytes / 4);
  const int within = static_cast<int>(wi % (kUnitBytes / 4));
  const int lane = within >> 2, r = within & 3;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t = unit / G.KO;
  const int ks = static_cast<int>(unit % G.KO);
  const int src = slot_src[t * kTileRows + g + 8 * (r & 1)];
  const int col = ks * kDenseCols + 4 * q + 2 * (r >> 1);
  uint32_t word = 0;
  if (src >= 0) {
    const uint16_t* rowp = ov + static_cast<int64_t>(src) * G.K;
    const uint32_t lo = (col < G.K) ? rowp[col] : 0u;
    const uint32_t hi = (col + 1 < G.K) ? rowp[col + 1] : 0u;
    word = lo | (hi << 16);
  }
  out[G.Up * (kUnitBytes / 4) + wi] = word;
}

// W_hat [M][K] fp16 from the repacked layer.  One warp per unit; the packed path decodes with
// the same decode_word routine as the GEMV.
__global__ void dequant_kernel(LayerGeom G, const uint8_t* __restrict__ units, const uint2* __restrict__ cb,
                               const uint16_t* __restrict__ tile_mask, const int32_t* __restrict__ orow,
                               uint16_t* __restrict__ w, int64_t ldw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (unit >= G.U) return;
  const int g = lane >> 2, q = lane & 3;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(units + unit * kUnitBytes) + lane);
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  auto put = [&](int64_t row, int col, uint32_t pair) {
    if (col < G.K) w[row * ldw + col] = static_cast<uint16_t>(pair & 0xffffu);
    if (col + 1 < G.K) w[row * ldw + col + 1] = static_cast<uint16_t>(pair >> 16);
  };
  if (unit < G.Up) {
    const int64_t t = unit / G.KT;
    const int kt = static_cast<int>(unit % G.KT);
    const int64_t r0 = t * kTileRows + g;
    const uint2 c0 = __ldg(cb + r0), c1 = __ldg(cb + r0 + 8);
    const uint32_t cbl[2] = {c0.x, c1.x}, cbh[2] = {c0.y, c1.y};
    const uint32_t mask = tile_mask[t];
    const bool live0 = r0 < G.M && !((mask >> g) & 1u);
    const bool live1 = r0 + 8 < G.M && !((mask >> (g + 8)) & 1u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t A0[4], A1[4];
      decode_word(wv[j], cbl, cbh, kNegZero2, A0, A1);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int col = kt * kPackedCols + (2 * j + h) * 16 + 4 * q + 2 * (r >> 1);
          const bool live = (r & 1) ? live1 : live0;
          if (live) put(r0 + 8 * (r & 1), col, h ? A1[r] : A0[r]);
        }
    }
  } else {
    const int64_t t = (unit - G.Up) / G.KO;
    const int ks = static_cast<int>((unit - G.Up) % G.KO);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = orow[t * kTileRows + g + 8 * (r & 1)];
      const int col = ks * kDenseCols + 4 * q + 2 * (r >> 1);
      if (row >= 0) put(row, col, wv[r]);
    }
  }
}

}  // namespace opc
