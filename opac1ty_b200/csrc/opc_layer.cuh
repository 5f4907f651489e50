// opc_layer.cuh -- load-time repack of a .bf2 layer into the streamed device layout, and the
// bit-exact dequantization kernel used to prove that layout against the reference.
//
// Device buffers of a repacked layer (sizes in opc_plan_layer):
//   units     [packed units | int8 outlier units | fp16 outlier units], 512 bytes each, then the
//             outlier rows row-major [slots][K_pad] fp16 (the prefill GEMM's dense pass)
//   codebooks [M_pad] x 8 B split fp16 centroids, then [M_pad] x 16 B integer codebooks
//             {4 x int8 high part, 4 x int8 low part, int32 exponent, 0}; an outlier row's entry
//             is {0, 0, exponent of its integer row, outlier slot}
//   tile_mask [MT] uint16
//   outlier_rows [slots] int32 output rows, then [slots] int32 exponents of the int8 rows
#pragma once

#include "opc_device.cuh"

namespace opc {

struct LayerGeom {
  int64_t Up, U;   // packed units, packed + one outlier format
  int32_t M, K, K_pad, M_pad, MT, KT, OT, KO;
};

// Integer form of a row of fp16 values with max magnitude `amax`: v * 2^e rounded to an integer
// n with |n| <= 2^14, split n = 256*hi + lo with lo, hi in int8 (lo in [-128, 127], hi in
// [-64, 64]).  e = 14 - (binary exponent of amax), so amax * 2^e lies in [2^13, 2^14).
__device__ __forceinline__ int int_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  return 14 - frexp_exponent(amax);  // amax comes from fp16 values: a normal float
}
__device__ __forceinline__ void int_parts(float v, int e, int* hi, int* lo) {
  const int n = __float2int_rn(ldexpf(v, e));
  const int l = ((n + 128) & 255) - 128;
  *lo = l;
  *hi = (n - l) >> 8;
}

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
  for (int hi = 0; hi < 2; ++hi)
#pragma unroll
    for (int ko = 0; ko < 8; ++ko) {
      const int64_t row = t * kTileRows + g + 8 * hi;
      const int col = kt * kPackedCols + 32 * j + 8 * q + ko;
      uint32_t v = 0;
      if (row < G.M && col < G.K) {
        v = idx[row * G.K + col];
        if (v > 3u) atomicExch(bad, 1);
      }
      word |= (v & 3u) << (2 * packed_field(hi, ko));
    }
  out[wi] = word;
}

// codebooks [M][4] fp16 (svs == 1) -> split fp16 form and integer form; outlier and padding
// rows are zero in both.
__global__ void repack_codebooks_kernel(LayerGeom G, const uint16_t* __restrict__ cb,
                                        const uint16_t* __restrict__ tile_mask, uint2* __restrict__ out,
                                        uint4* __restrict__ outq) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= G.M_pad) return;
  uint2 v = make_uint2(0u, 0u);
  uint4 vq = make_uint4(0u, 0u, 0u, 0u);
  const bool outlier = (tile_mask[r / kTileRows] >> (r % kTileRows)) & 1u;
  if (r < G.M && !outlier) {
    float f[4], amax = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t h = cb[r * 4 + c];
      v.x |= (h & 0xffu) << (8 * c);
      v.y |= (h >> 8) << (8 * c);
      f[c] = __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
      amax = fmaxf(amax, fabsf(f[c]));
    }
    const int e = int_exponent(amax);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int hi, lo;
      int_parts(f[c], e, &hi, &lo);
      vq.x |= (static_cast<uint32_t>(hi) & 0xffu) << (8 * c);
      vq.y |= (static_cast<uint32_t>(lo) & 0xffu) << (8 * c);
    }
    vq.z = static_cast<uint32_t>(e);
  }
  out[r] = v;
  outq[r] = vq;
}

// Exponent of each outlier slot's integer row (one block per slot).  The integer-codebook entry
// of an outlier row (zero centroids) also records {.z = exponent, .w = slot}, so a row can be
// mapped to its slot (used by the decode-chain kernel).
__global__ void outlier_exponent_kernel(LayerGeom G, const uint16_t* __restrict__ ov,
                                        const int32_t* __restrict__ slot_src, const int32_t* __restrict__ orow,
                                        int32_t* __restrict__ oexp, uint4* __restrict__ cbq) {
  const int slot = blockIdx.x;
  const int src = slot_src[slot];
  float m = 0.f;
  if (src >= 0) {
    const uint16_t* rowp = ov + static_cast<int64_t>(src) * G.K;
    for (int k = threadIdx.x; k < G.K; k += blockDim.x)
      m = fmaxf(m, fabsf(__half2float(__ushort_as_half(static_cast<unsigned short>(rowp[k])))));
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
    const int e = int_exponent(t);
    oexp[slot] = e;
    const int row = orow[slot];
    if (row >= 0) cbq[row] = make_uint4(0u, 0u, static_cast<uint32_t>(e), static_cast<uint32_t>(slot));
  }
}

// outlier rows [n][K] fp16 -> dense units of both kernels.  slot_src[s] is the source row (in
// the outlier value array) of outlier slot s, or -1 for padding slots.
//  * int8 unit (tile t, s in 0..KO-1): k block s>>3, staged int8 positions 16*(s&7) + 0..15;
//    lane (g,q) holds words {hi row g, hi row g+8, lo row g, lo row g+8}, each the 4 bytes of
//    positions 16*(s&7) + 4q + 0..3 (an m16n8k16 int8 A fragment per part).
//  * fp16 unit (tile t, s): k block s>>3, staged fp16 positions 32q + 4*(s&7) + 0..3 for lane q;
//    register r holds row g + 8*(r&1) at positions 32q + 4*(s&7) + 2*(r>>1) + (0, 1) (an
//    m16n8k16 fp16 A fragment whose B fragment is the 8 bytes at those positions).
__global__ void repack_outliers_kernel(LayerGeom G, const uint16_t* __restrict__ ov,
                                       const int32_t* __restrict__ slot_src, const int32_t* __restrict__ oexp,
                                       uint32_t* __restrict__ out_q, uint32_t* __restrict__ out_h) {
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n_words = (G.U - G.Up) * (kUnitBytes / 4);
  if (wi >= n_words) return;
  const int64_t unit = wi / (kUnitBytes / 4);
  const int within = static_cast<int>(wi % (kUnitBytes / 4));
  const int lane = within >> 2, r = within & 3;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t = unit / G.KO;
  const int s = static_cast<int>(unit % G.KO);
  const int kb = (s >> 3) * kPackedCols, s8 = s & 7;
  auto value = [&](int src, int k) -> uint16_t {
    return (src >= 0 && k < G.K) ? ov[static_cast<int64_t>(src) * G.K + k] : static_cast<uint16_t>(0);
  };
  // int8 word r: part (r >> 1) (0 = hi, 1 = lo) of row g + 8*(r & 1)
  {
    const int slot = static_cast<int>(t * kTileRows + g + 8 * (r & 1));
    const int src = slot_src[slot];
    const int e = src >= 0 ? oexp[slot] : 0;
    uint32_t word = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int k = kb + kin_of_pos8(16 * s8 + 4 * q + c);
      const float f = __half2float(__ushort_as_half(value(src, k)));
      int hi, lo;
      int_parts(f, e, &hi, &lo);
      word |= (static_cast<uint32_t>((r >> 1) ? lo : hi) & 0xffu) << (8 * c);
    }
    out_q[wi] = word;
  }
  // fp16 word r
  {
    const int src = slot_src[t * kTileRows + g + 8 * (r & 1)];
    const int p0 = 32 * q + 4 * s8 + 2 * (r >> 1);
    const uint32_t lo = value(src, kb + kin_of_pos16(p0));
    const uint32_t hi = value(src, kb + kin_of_pos16(p0 + 1));
    out_h[wi] = lo | (hi << 16);
  }
}

// Row-major copy of the outlier rows by slot, zero-padded to K_pad (padding slots are zero).
__global__ void repack_dense_outliers_kernel(LayerGeom G, const uint16_t* __restrict__ ov,
                                             const int32_t* __restrict__ slot_src, int32_t n_slots,
                                             uint16_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(n_slots) * G.K_pad) return;
  const int slot = static_cast<int>(i / G.K_pad), k = static_cast<int>(i % G.K_pad);
  const int src = slot_src[slot];
  out[i] = (src >= 0 && k < G.K) ? ov[static_cast<int64_t>(src) * G.K + k] : static_cast<uint16_t>(0);
}

// W_hat [M][K] fp16 from the repacked layer.  One warp per unit of the packed region and of the
// fp16 outlier region; the packed path decodes with the fp16 GEMV's decode_word.
__global__ void dequant_kernel(LayerGeom G, const uint8_t* __restrict__ units, const uint8_t* __restrict__ ounits_h,
                               const uint2* __restrict__ cb, const uint16_t* __restrict__ tile_mask,
                               const int32_t* __restrict__ orow, uint16_t* __restrict__ w, int64_t ldw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (unit >= G.U) return;
  const int g = lane >> 2, q = lane & 3;
  const uint8_t* src = unit < G.Up ? units + unit * kUnitBytes : ounits_h + (unit - G.Up) * kUnitBytes;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + lane);
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  auto put1 = [&](int64_t row, int col, uint16_t h) {
    if (col < G.K) w[row * ldw + col] = h;
  };
  if (unit < G.Up) {
    const int64_t t = unit / G.KT;
    const int kt = static_cast<int>(unit % G.KT);
    const int64_t r0 = t * kTileRows + g;
    const uint2 c0 = __ldg(cb + r0), c1 = __ldg(cb + r0 + 8);
    const uint32_t cbl[2] = {c0.x, c1.x}, cbh[2] = {c0.y, c1.y};
    const uint32_t mask = tile_mask[t];
    const bool live[2] = {r0 < G.M && !((mask >> g) & 1u), r0 + 8 < G.M && !((mask >> (g + 8)) & 1u)};
    // k offsets of decode_word's registers: step 0 (0,2 | 1,3), step 1 (4,6 | 5,7)
    constexpr int kofs[2][2][2] = {{{0, 2}, {1, 3}}, {{4, 6}, {5, 7}}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t A[2][4];
      decode_word(wv[j], cbl, cbh, kNegZero2, A[0], A[1]);
#pragma unroll
      for (int st = 0; st < 2; ++st)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int h = r & 1;
          if (!live[h]) continue;
          const int col0 = kt * kPackedCols + 32 * j + 8 * q;
          put1(r0 + 8 * h, col0 + kofs[st][r >> 1][0], static_cast<uint16_t>(A[st][r] & 0xffffu));
          put1(r0 + 8 * h, col0 + kofs[st][r >> 1][1], static_cast<uint16_t>(A[st][r] >> 16));
        }
    }
  } else {
    const int64_t t = (unit - G.Up) / G.KO;
    const int s = static_cast<int>((unit - G.Up) % G.KO);
    const int kb = (s >> 3) * kPackedCols, s8 = s & 7;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = orow[t * kTileRows + g + 8 * (r & 1)];
      const int p0 = 32 * q + 4 * s8 + 2 * (r >> 1);
      if (row >= 0) {
        put1(row, kb + kin_of_pos16(p0), static_cast<uint16_t>(wv[r] & 0xffffu));
        put1(row, kb + kin_of_pos16(p0 + 1), static_cast<uint16_t>(wv[r] >> 16));
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// sub_vector_size 8 on the decode chain.  The chain streams the layer's own 128-byte index units
// (four of them, 16 rows x 1024 columns, per 512-byte chain unit) and multiplies integer forms
// of the selected codebook vectors with its staged x digits (int8 mma.sync, exact int64 sums like
// svs 1).  Per row the four 8-element vectors become integers n = round(v * 2^e) with one
// exponent e for all 32 values (int_exponent of the largest), stored as 64 bytes: for vector c,
// 16 bytes {hi[0..7], lo[0..7]} (n = 256 hi + lo), so that one 16-byte load gives the A-fragment
// registers of both vector halves for both parts.  Outlier and padding rows are zero, and cbq
// gets {0, 0, e, 0} per row for the chain's row metadata.  One thread per row.
// ------------------------------------------------------------------------------------------------
__global__ void vq8_chain_vectors_kernel(int32_t M, int32_t M_pad, const uint4* __restrict__ cb8,
                                         const uint16_t* __restrict__ tile_mask, uint4* __restrict__ cbv,
                                         uint4* __restrict__ cbq) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M_pad) return;
  const bool outlier = (tile_mask[r / kTileRows] >> (r % kTileRows)) & 1u;
  if (r >= M || outlier) {
    for (int c = 0; c < 4; ++c) cbv[static_cast<int64_t>(r) * 4 + c] = make_uint4(0u, 0u, 0u, 0u);
    cbq[r] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  // opc_vq8.cuh layout: lane 4g+q of tile t holds, for rows g (first uint4) and g+8 (second),
  // elements 2q, 2q+1 of vectors 0..3 (one 32-bit word per vector)
  const int t = r >> 4, gr = r & 15, g = gr & 7, h = gr >> 3;
  float f[4][8];
  float amax = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = cb8[(static_cast<int64_t>(t) * 32 + 4 * g + q) * 2 + h];
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      f[c][2 * q] = __half2float(__ushort_as_half(static_cast<unsigned short>(ww[c] & 0xffffu)));
      f[c][2 * q + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(ww[c] >> 16)));
      amax = fmaxf(amax, fmaxf(fabsf(f[c][2 * q]), fabsf(f[c][2 * q + 1])));
    }
  }
  const int e = int_exponent(amax);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      int hi, lo;
      int_parts(f[c][s], e, &hi, &lo);
      hw[s >> 2] |= (static_cast<uint32_t>(hi) & 0xffu) << (8 * (s & 3));
      lw[s >> 2] |= (static_cast<uint32_t>(lo) & 0xffu) << (8 * (s & 3));
    }
    cbv[static_cast<int64_t>(r) * 4 + c] = make_uint4(hw[0], hw[1], lw[0], lw[1]);
  }
  cbq[r] = make_uint4(0u, 0u, static_cast<uint32_t>(e), 0u);
}

}  // namespace opc
