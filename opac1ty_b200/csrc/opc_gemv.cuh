// opc_gemv.cuh -- fused 2-bit codebook dequant + GEMV / small-batch GEMM for sm_100a.
//
// What it computes (reference semantics, opacc1ty/export/converter.py:26-67 followed by a
// matmul):  y[b][r] = sum_k x[b][k] * W_hat[r][k], where W_hat[r][k] = cb[r][idx[r][k]] for
// ordinary rows and the stored fp16 row for outlier rows.  The reference's Metal kernel
// (kernels/dequant_gemv.metal:57-134) runs one thread per output row with byte loads along K;
// this kernel is organised around HBM streaming instead:
//
//  * The repacked layer is one flat array of 512-byte units (packed 16x128 index tiles, then
//    fp16 outlier 16x16 blocks).  Units are split into equal contiguous ranges, one per CTA,
//    and each CTA's range into equal sub-ranges, one per warp, so every warp streams the same
//    number of bytes whatever the layer shape.
//  * Each warp streams its sub-range through a private ring of shared-memory stages filled by
//    bulk async copies (TMA engine, no multicast); no registers hold in-flight loads.  The first
//    stages are issued before griddepcontrol.wait, i.e. while the previous kernel of a decode
//    chain is still running: weights never depend on the activations.
//  * Decode is register-only: per pair of weights one IMAD builds a PRMT selector and one PRMT
//    gathers half2(cb[i], cb[j]) from the row's split codebook (opc_device.cuh); the products
//    run on the tensor cores (mma.sync m16n8k16, fp32 accumulation) with x as the B operand, so
//    batch 1..8 costs the same as batch 1.  x is staged in shared memory in the mma's k order,
//    one 16-byte load per two k-steps.
//  * A segment (one 16-row tile) cut by a warp boundary is summed in shared memory by the first
//    warp of the CTA that touches it, in warp order.  A segment cut by a CTA boundary is then
//    finished by whichever of its CTAs arrives last: CTA partials go to per-CTA slots in the
//    workspace, an atomic counter per segment elects the finisher, which adds the slots in CTA
//    order and resets the counter.  The summation order is fixed, so results are deterministic.
#pragma once

#include "opc_device.cuh"

namespace opc {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kStages = 4;        // ring depth per warp
constexpr int kChunkUnits = 4;    // units per bulk copy
constexpr int kChunkBytes = kChunkUnits * kUnitBytes;
constexpr int kRingBytesPerWarp = kStages * kChunkBytes;
constexpr int kBarBytesPerWarp = kStages * 8;

// Permuted shared-memory copy of x: for batch row b and k block kt (128 columns), k sits at
// position xs_pos16(k - 128kt), so the B fragments of lane q (4 words x 8 halves) are the 64
// contiguous bytes at position 32q.  Rows are padded by 16 bytes so different batch rows use
// different banks.
__host__ __device__ constexpr int xs_row_bytes(int KT) { return KT * 256 + 16; }

struct GemvArgs {
  const uint8_t* units;         // packed units (unit u at units + 512u)
  const uint8_t* ounits;        // fp16 outlier units (unit u >= Up at ounits + 512(u - Up))
  const uint2* cb;              // [M_pad] split codebooks
  const uint16_t* tile_mask;    // [MT]
  const int32_t* orow;          // [OT*16]
  const __half* x;
  __half* y;
  float* gslots;                // [grid][2][NT*128] CTA partials of CTA-spanning segments
  int32_t* counters;            // [MT + OT]
  int64_t ldx, ldy;
  int32_t Up, U;                // packed units, total units (< 2^31)
  int32_t M, K, K_pad, MT, KT, OT, KO, batch;
  int32_t xs_bytes;             // shared bytes reserved for x (0: read x from global)
  int32_t x_vec16;              // x rows 16-byte loadable (K%8==0, ldx%8==0, aligned)
  int32_t x_vec8;               // x rows 8-byte loadable (K%4==0, ldx%4==0, aligned)
  uint32_t negz;                // kNegZero2 (0x80008000), kept in a register by the decode
};

struct Seg {
  int32_t id, begin, end;
};

__device__ __forceinline__ Seg seg_at(const GemvArgs& a, int32_t u) {
  if (u < a.Up) {
    const int32_t t = u / a.KT;
    return {t, t * a.KT, (t + 1) * a.KT};
  }
  const int32_t t = (u - a.Up) / a.KO;
  return {a.MT + t, a.Up + t * a.KO, a.Up + (t + 1) * a.KO};
}

// Everything a lane needs about a segment besides the streamed units.
struct Meta {
  uint32_t cbl[2], cbh[2];  // split codebooks of rows g, g+8 (packed segments)
  int32_t row[2];           // output row of rows g, g+8, or -1 (padding / written elsewhere)
};

__device__ __forceinline__ Meta load_meta(const GemvArgs& a, int32_t seg, int g) {
  Meta m;
  if (seg < a.MT) {
    const int r0 = seg * kTileRows + g;
    const uint2 c0 = __ldg(a.cb + r0);
    const uint2 c1 = __ldg(a.cb + r0 + 8);
    const uint32_t mask = __ldg(a.tile_mask + seg);
    m.cbl[0] = c0.x; m.cbh[0] = c0.y;
    m.cbl[1] = c1.x; m.cbh[1] = c1.y;
    m.row[0] = (r0 < a.M && !((mask >> g) & 1u)) ? r0 : -1;
    m.row[1] = (r0 + 8 < a.M && !((mask >> (g + 8)) & 1u)) ? r0 + 8 : -1;
  } else {
    const int t = seg - a.MT;
    m.cbl[0] = m.cbh[0] = m.cbl[1] = m.cbh[1] = 0u;
    m.row[0] = __ldg(a.orow + t * kTileRows + g);
    m.row[1] = __ldg(a.orow + t * kTileRows + g + 8);
  }
  return m;
}

// x[bcol][k..k+3] from global memory (natural layout), zero outside [0, K).
__device__ __forceinline__ uint2 load_x4_global(const GemvArgs& a, int bcol, int k) {
  const __half* p = a.x + bcol * a.ldx + k;
  if (a.x_vec8 && k + 4 <= a.K) return __ldcg(reinterpret_cast<const uint2*>(p));
  uint16_t h[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = (k + e < a.K) ? __ldcg(reinterpret_cast<const unsigned short*>(p) + e) : 0;
  return make_uint2(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16));
}
// (x0,x1 | x2,x3) -> (x0,x2 | x1,x3): the staged order of 4 consecutive halves.
__device__ __forceinline__ uint2 swap_mid(uint2 v) { return make_uint2(prmt(v.x, v.y, 0x5410u), prmt(v.x, v.y, 0x7632u)); }

template <int NT>
__device__ __forceinline__ void zero_acc(float acc[2][NT][4]) {
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[c][n][e] = 0.f;
}

// Per-lane constants of the hot loop, hoisted out of the kernel-parameter bank.
template <int NT>
struct LaneCtx {
  uint32_t negz;
  // Shared-memory address of this lane's 64-byte column group in x row 8nt+g, advancing kts
  // bytes per k block.  Lanes whose batch column does not exist point at a 64-byte zero block
  // with kts = 0.  (32-bit shared-window addresses keep the address arithmetic 32-bit.)
  uint32_t xq[NT];
  uint32_t kts[NT];
};

// One packed unit: 8 k-steps of 16 columns for a 16-row tile.  Even k-steps accumulate into
// chain 0, odd ones into chain 1 (two independent mma dependency chains).
template <int NT, bool XS>
__device__ __forceinline__ void packed_unit(const GemvArgs& a, const LaneCtx<NT>& lc, uint32_t unit,
                                            int kt, int g, int q, const Meta& m, float acc[2][NT][4]) {
  const uint4 wv = lds128(unit);
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t A0[4], A1[4];
    decode_word(w[j], m.cbl, m.cbh, lc.negz, A0, A1);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint4 b;
      if (XS) {
        b = lds128(lc.xq[nt] + kt * lc.kts[nt] + j * 16);
      } else {
        b = make_uint4(0, 0, 0, 0);
        const int bcol = 8 * nt + g;
        if (bcol < a.batch) {
          const int k = kt * kPackedCols + 32 * j + 8 * q;
          const uint2 b0 = swap_mid(load_x4_global(a, bcol, k)), b1 = swap_mid(load_x4_global(a, bcol, k + 4));
          b = make_uint4(b0.x, b0.y, b1.x, b1.y);
        }
      }
      mma16816(acc[0][nt], A0, b.x, b.y);
      mma16816(acc[1][nt], A1, b.z, b.w);
    }
  }
}

// One outlier unit: a 16x16 fp16 block already in A-fragment order; unit ks of the segment
// covers the staged positions 32q + 4(ks&7) + 0..3 of k block ks>>3.
template <int NT, bool XS>
__device__ __forceinline__ void dense_unit(const GemvArgs& a, const LaneCtx<NT>& lc, uint32_t unit, int ks,
                                           int g, int q, float acc[2][NT][4]) {
  const uint4 av = lds128(unit);
  const uint32_t A[4] = {av.x, av.y, av.z, av.w};
  const int kt = ks >> 3, s = ks & 7;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    uint2 b;
    if (XS) {
      b = lds64(lc.xq[nt] + kt * lc.kts[nt] + s * 8);
    } else {
      b = make_uint2(0, 0);
      const int bcol = 8 * nt + g;
      // staged positions 32q + 4s + 0..3 = k offsets (0,2,1,3) from 32(s>>1) + 8q + 4(s&1)
      if (bcol < a.batch) b = swap_mid(load_x4_global(a, bcol, kt * kPackedCols + 32 * (s >> 1) + 8 * q + 4 * (s & 1)));
    }
    mma16816(acc[0][nt], A, b.x, b.y);
  }
}

template <int NT>
__device__ __forceinline__ void fold_chains(const float acc[2][NT][4], float out[NT][4]) {
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) out[n][e] = acc[0][n][e] + acc[1][n][e];
}

// C fragment: element e of n-tile nt is (row g + 8*(e>>1), batch column 8nt + 2q + (e&1)).
template <int NT>
__device__ __forceinline__ void write_out(const GemvArgs& a, const Meta& m, const float v[NT][4], int q) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int b = 8 * nt + 2 * q + (e & 1);
      const int row = m.row[e >> 1];
      if (b < a.batch && row >= 0) a.y[b * a.ldy + row] = __float2half_rn(v[nt][e]);
    }
}

// Contiguous equal split of [0, n) into p parts: part i starts at i*n/p.
__device__ __forceinline__ int32_t part_start(int32_t i, int32_t n, int32_t p) {
  return static_cast<int32_t>(static_cast<int64_t>(i) * n / p);
}
// The part containing element e (the last part starting at or before e).
__device__ __forceinline__ int32_t part_of(int32_t e, int32_t n, int32_t p) {
  return static_cast<int32_t>((static_cast<int64_t>(e + 1) * p + n - 1) / n - 1);
}

// Walk of a warp's unit range segment by segment (no divisions after the start).
struct Cursor {
  int32_t u, seg, begin, end;
};

__device__ __forceinline__ Cursor cursor_at(const GemvArgs& a, int32_t u) {
  const Seg s = seg_at(a, u);
  return {u, s.id, s.begin, s.end};
}
__device__ __forceinline__ int32_t chunk_units(const Cursor& c, int32_t u1) {
  int32_t n = c.end - c.u;
  if (u1 - c.u < n) n = u1 - c.u;
  return n < kChunkUnits ? n : kChunkUnits;
}
__device__ __forceinline__ void advance_in_segment(Cursor& c, int32_t n) { c.u += n; }
__device__ __forceinline__ void next_segment(const GemvArgs& a, Cursor& c) {
  c.seg += 1;
  c.begin = c.end;
  c.end = c.begin + (c.seg < a.MT ? a.KT : a.KO);
}
__device__ __forceinline__ void advance(const GemvArgs& a, Cursor& c, int32_t n) {
  c.u += n;
  if (c.u == c.end) next_segment(a, c);
}

template <int NT>
struct SmemSlots {
  // Per warp: two partial-sum slots (its first and last segment) and their segment ids.
  float v[kGemvWarps][2][NT * 128];
  int32_t seg[kGemvWarps][2];
};

template <int NT>
__device__ __forceinline__ void put_slot(SmemSlots<NT>* ss, int warp, int sl, int lane, int32_t seg,
                                         const float v[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    *reinterpret_cast<float4*>(&ss->v[warp][sl][nt * 128 + lane * 4]) = make_float4(v[nt][0], v[nt][1], v[nt][2], v[nt][3]);
  if (lane == 0) ss->seg[warp][sl] = seg;
}

// Sum segment S over the CTA's warps in warp order (the caller is the first warp touching S),
// then either write y (S lies inside the CTA's range) or take part in the cross-CTA fixup.
template <int NT>
__device__ void reduce_segment(const GemvArgs& a, SmemSlots<NT>* ss, Seg S, int32_t c0, int32_t c1, int lane,
                               int g, int q) {
  const int32_t n = c1 - c0;
  const int32_t lo = S.begin > c0 ? S.begin : c0;
  const int32_t hi = (S.end < c1 ? S.end : c1) - 1;
  const int wa = part_of(lo - c0, n, kGemvWarps), wb = part_of(hi - c0, n, kGemvWarps);
  float tot[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) tot[nt][e] = 0.f;
  for (int w = wa; w <= wb; ++w) {
    const int32_t ws = c0 + part_start(w, n, kGemvWarps), we = c0 + part_start(w + 1, n, kGemvWarps);
    if (we <= ws) continue;                 // empty warp range (only when n < 8)
    const int sl = (ws >= S.begin) ? 0 : 1;  // S is w's first segment iff it contains ws
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float4 p = *reinterpret_cast<const float4*>(&ss->v[w][sl][nt * 128 + lane * 4]);
      tot[nt][0] += p.x; tot[nt][1] += p.y; tot[nt][2] += p.z; tot[nt][3] += p.w;
    }
  }
  if (S.begin >= c0 && S.end <= c1) {
    write_out<NT>(a, load_meta(a, S.id, g), tot, q);
    return;
  }
  // Cross-CTA fixup.
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int which = (S.begin <= c0) ? 0 : 1;  // 0: S contains c0 (this CTA's first segment)
  float* mine = a.gslots + (static_cast<int64_t>(cta) * 2 + which) * (NT * 128);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    __stcg(reinterpret_cast<float4*>(mine + nt * 128 + lane * 4), make_float4(tot[nt][0], tot[nt][1], tot[nt][2], tot[nt][3]));
  __threadfence();
  __syncwarp();
  const int ca = part_of(S.begin, a.U, G), cb = part_of(S.end - 1, a.U, G);
  int old = 0;
  if (lane == 0) old = atomicAdd(a.counters + S.id, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != cb - ca) return;  // not the last CTA to arrive
  __threadfence();
  float fin[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) fin[nt][e] = 0.f;
  for (int c = ca; c <= cb; ++c) {
    const int cw = (part_start(c, a.U, G) >= S.begin) ? 0 : 1;
    const float* src = a.gslots + (static_cast<int64_t>(c) * 2 + cw) * (NT * 128);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float4 p = (c == cta) ? make_float4(tot[nt][0], tot[nt][1], tot[nt][2], tot[nt][3])
                                  : __ldcg(reinterpret_cast<const float4*>(src + nt * 128 + lane * 4));
      fin[nt][0] += p.x; fin[nt][1] += p.y; fin[nt][2] += p.z; fin[nt][3] += p.w;
    }
  }
  write_out<NT>(a, load_meta(a, S.id, g), fin, q);
  if (lane == 0) atomicExch(a.counters + S.id, 0);
}

template <int NT, bool XS>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  // The warp index comes from a shuffle so the compiler knows every value derived from it
  // (the warp's unit range, chunk counts, segment bounds) is warp-uniform.
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int32_t c0 = part_start(cta, a.U, G), c1 = part_start(cta + 1, a.U, G);
  const int32_t n_cta = c1 - c0;
  const int32_t u0 = c0 + part_start(warp, n_cta, kGemvWarps), u1 = c0 + part_start(warp + 1, n_cta, kGemvWarps);
  const int32_t n_units = u1 - u0;

  const uint32_t xs_base = smem_u32(smem);
  const uint32_t ring_base = xs_base + a.xs_bytes + warp * kRingBytesPerWarp;
  const uint32_t bar_base = xs_base + a.xs_bytes + kGemvWarps * kRingBytesPerWarp + warp * kBarBytesPerWarp;
  SmemSlots<NT>* ss = reinterpret_cast<SmemSlots<NT>*>(smem + a.xs_bytes + kGemvWarps * (kRingBytesPerWarp + kBarBytesPerWarp));

  // Chunks never straddle a segment: chunk size = min(kChunkUnits, units left in the segment,
  // units left in the range).  Lane 0 walks the same chunk sequence kStages chunks ahead of
  // the consumer (cursor `pc`), so both agree on every chunk's size and stage slot.
  auto issue_chunk = [&](const Cursor& pcur, int32_t c) {
    const int32_t cnt = chunk_units(pcur, u1);
    const int slot = c % kStages;
    const uint32_t bar = bar_base + slot * 8;
    mbar_expect_tx(bar, static_cast<uint32_t>(cnt * kUnitBytes));
    const uint8_t* src = pcur.u < a.Up ? a.units + static_cast<int64_t>(pcur.u) * kUnitBytes
                                       : a.ounits + static_cast<int64_t>(pcur.u - a.Up) * kUnitBytes;
    bulk_g2s(ring_base + slot * kChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar);
  };
  Cursor pc = cursor_at(a, u0);
  int32_t pchunk = 0;

  // Prologue: start streaming weights (they do not depend on the previous kernel).
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(bar_base + s * 8, 1);
    fence_mbar_init();
    for (; pchunk < kStages && pc.u < u1; ++pchunk) {
      issue_chunk(pc, pchunk);
      advance(a, pc, chunk_units(pc, u1));
    }
    ss->seg[warp][0] = -1;
    ss->seg[warp][1] = -1;
  }
  __syncwarp();
  griddep_launch_dependents();
  griddep_wait();  // x and the workspace may be written by the previous kernel

  if (XS) {
    // Stage x[batch][K] into the permuted layout, zero-padded to K_pad.  Every thread first
    // issues all its 16-byte loads (L2-coherent), then stores them.
    const int per_row = a.K_pad / 8;
    const int total = a.batch * per_row;
    if (threadIdx.x < 4)  // the 64-byte zero block after the last row (B of absent batch columns)
      *reinterpret_cast<uint4*>(smem + a.batch * xs_row_bytes(a.KT) + threadIdx.x * 16) = make_uint4(0, 0, 0, 0);
    for (int base = 0; base < total; base += 8 * kGemvThreads) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = base + i * kGemvThreads + threadIdx.x;
        v[i] = make_uint4(0, 0, 0, 0);
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          if (a.x_vec16) {
            if (k < a.K) v[i] = __ldcg(reinterpret_cast<const uint4*>(a.x + b * a.ldx + k));
          } else {
            uint16_t h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              h[e] = (k + e < a.K) ? __ldcg(reinterpret_cast<const unsigned short*>(a.x + b * a.ldx + k + e)) : 0;
            v[i] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                              h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = base + i * kGemvThreads + threadIdx.x;
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          // 8 consecutive k (offsets 0..7 of one lane column group and word) -> 16 bytes at
          // position xs_pos16(k & 127), halves in the order (0,2,1,3,4,6,5,7)
          const uint32_t dst = xs_base + static_cast<uint32_t>(b * xs_row_bytes(a.KT) + (k >> 7) * 256 +
                                                               xs_pos16(k & 127) * 2);
          const uint2 lo = swap_mid(make_uint2(v[i].x, v[i].y)), hi = swap_mid(make_uint2(v[i].z, v[i].w));
          sts128(dst, make_uint4(lo.x, lo.y, hi.x, hi.y));
        }
      }
    }
  }
  __syncthreads();  // x staged; every warp's slot ids initialised

  LaneCtx<NT> lc;
  lc.negz = a.negz;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int bcol = 8 * nt + g;
    const bool live = bcol < a.batch;
    lc.xq[nt] = xs_base + static_cast<uint32_t>(live ? bcol * xs_row_bytes(a.KT) + q * 64 : a.batch * xs_row_bytes(a.KT));
    lc.kts[nt] = live ? 256u : 0u;
  }
  const uint32_t ring_lane = ring_base + lane * 16;
  const int32_t MT = a.MT;

  bool ok = true;
  if (n_units > 0) {
    const int32_t n_seg = a.MT + a.OT;
    Cursor cc = cursor_at(a, u0);
    Meta cur = load_meta(a, cc.seg, g);
    Meta nxt = cur;
    if (cc.seg + 1 < n_seg) nxt = load_meta(a, cc.seg + 1, g);
    float acc[2][NT][4];
    zero_acc<NT>(acc);
    for (int32_t c = 0; cc.u < u1; ++c) {
      const int slot = c % kStages;
      if (!mbar_wait_bounded(bar_base + slot * 8, static_cast<uint32_t>((c / kStages) & 1))) {
        ok = false;
        break;
      }
      const int32_t cnt = chunk_units(cc, u1);
      const uint32_t stage = ring_lane + slot * kChunkBytes;
      const int32_t k0 = cc.u - cc.begin;
      if (cc.seg < MT) {
        if (cnt == kChunkUnits) {
#pragma unroll
          for (int i = 0; i < kChunkUnits; ++i) packed_unit<NT, XS>(a, lc, stage + i * kUnitBytes, k0 + i, g, q, cur, acc);
        } else {
          for (int i = 0; i < cnt; ++i) packed_unit<NT, XS>(a, lc, stage + i * kUnitBytes, k0 + i, g, q, cur, acc);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kChunkUnits; ++i)
          if (i < cnt) dense_unit<NT, XS>(a, lc, stage + i * kUnitBytes, k0 + i, g, q, acc);
      }
      advance_in_segment(cc, cnt);
      if (cc.u == cc.end && cc.u < u1) {  // segment complete inside the range
        float v[NT][4];
        fold_chains<NT>(acc, v);
        if (cc.begin < u0)
          put_slot<NT>(ss, warp, 0, lane, cc.seg, v);  // began in an earlier warp's range
        else
          write_out<NT>(a, cur, v, q);
        zero_acc<NT>(acc);
        next_segment(a, cc);
        cur = nxt;
        if (cc.seg + 1 < n_seg) nxt = load_meta(a, cc.seg + 1, g);
      }
      __syncwarp();
      if (lane == 0 && pc.u < u1) {
        issue_chunk(pc, pchunk++);
        advance(a, pc, chunk_units(pc, u1));
      }
    }
    if (ok) {
      float v[NT][4];
      fold_chains<NT>(acc, v);
      if (cc.begin >= u0 && cc.end <= u1)
        write_out<NT>(a, cur, v, q);
      else
        put_slot<NT>(ss, warp, cc.begin <= u0 ? 0 : 1, lane, cc.seg, v);
    } else {
      if (lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
      // Give copies still in flight a bounded chance to land before the CTA exits.
      for (int st = 0; st < kStages; ++st) (void)mbar_wait_bounded(bar_base + st * 8, 0);
    }
  }
  __syncthreads();  // every warp's partials are in shared memory
  if (!ok || n_units <= 0) return;

  // Segments this warp reduces: its first segment when that began before the CTA's range
  // (the warp is then the CTA's first warp), and its last segment when the last segment began
  // inside this warp's range or before the CTA's range.
  const int32_t s0 = ss->seg[warp][0], s1 = ss->seg[warp][1];
  if (s0 >= 0) {
    const Seg S = seg_at(a, s0 < a.MT ? s0 * a.KT : a.Up + (s0 - a.MT) * a.KO);
    const bool first_is_last = (S.end >= u1);  // stored as slot 0 because it was also the last
    if ((S.begin < u0 && u0 == c0) || (first_is_last && S.begin >= u0))
      reduce_segment<NT>(a, ss, S, c0, c1, lane, g, q);
  }
  if (s1 >= 0) {
    const Seg S = seg_at(a, s1 < a.MT ? s1 * a.KT : a.Up + (s1 - a.MT) * a.KO);
    if (S.begin >= u0 || u0 == c0) reduce_segment<NT>(a, ss, S, c0, c1, lane, g, q);
  }
}

}  // namespace opc
