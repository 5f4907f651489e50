// opc_gemvd.cuh -- single-launch integer GEMV for batch 1..2, built for launch latency.
//
// Same arithmetic as gemvq_kernel (opc_gemvq.cuh): centroids as row-scaled integers split into
// int8 parts, x staged as offset 22-bit integers in three unsigned digit columns, two int8
// mma.sync per 16 weights, exact int64 dot products and one fp16 rounding per output -- so the
// results equal gemvq_kernel's and the decode chain's bit for bit.  What differs is everything
// around the arithmetic, which is what a single launch of a Llama-shaped layer is made of
// (a 128 x 1024 layer took 8.3 us back to back in a graph with gemvq_kernel, an empty kernel of
// the same shape 0.7 us):
//
//  * No producer warp and no mbarriers.  Every warp streams its own contiguous unit range through
//    a ring of kDRing 512-byte slots in shared memory with per-lane 16-byte cp.async copies.  A
//    lane copies exactly the 16 bytes of a unit it later reads itself, so cp.async.wait_group
//    alone orders copy and use (no warp or CTA synchronisation in the units loop).  The first
//    kDRing - 1 units of every warp are requested before griddepcontrol.wait, i.e. while the
//    previous kernel of the stream finishes.
//  * Unit ranges come from one 32-bit division per bound (warp w of NW active warps takes units
//    [w U / NW, (w+1) U / NW); the host checks NW * U < 2^32), no 64-bit division anywhere.
//  * Row tiles shared by several warps are reduced in the workspace's int64 accumulators with
//    count-carrying atomics: every contributor adds 2^52 + t (t its exact partial dot product,
//    |partial sums| < 2^51) with one returning atomic per row; the contributor that completes the
//    count (the number of warps whose ranges meet the tile, computed from the same division) holds
//    the exact total, writes the row and clears the accumulator for the next launch.  No counters,
//    no fences, no second pass.
//  * The code is small: the units loop is not unrolled, and the staging and finishing paths have
//    one copy each.
#pragma once

#include "opc_chain.cuh"

namespace opc {

constexpr int kDWarps = 16;
constexpr int kDThreads = kDWarps * 32;
constexpr int kDRing = 8;                                    // units in flight per warp (power of two)
constexpr int kDRingBytes = kDWarps * kDRing * kUnitBytes;   // 64 KB per CTA

struct GemvDArgs {
  const uint8_t* units;        // packed units (unit u at units + 512u)
  const uint8_t* ounits;       // int8 outlier units (unit u >= Up at ounits + 512(u - Up))
  const uint4* cbq;            // [M_pad] {hi x4, lo x4, e_r, 0}
  const uint16_t* tile_mask;   // [MT]
  const int32_t* orow;         // [OT*16] output row of each outlier slot, -1 = padding
  const int32_t* oexp;         // [OT*16] exponent of each outlier slot's integer row
  const __half* x;
  __half* y;
  unsigned long long* acc;     // [M_pad][2] count-carrying accumulators, zero between launches
  int64_t ldx, ldy;
  int32_t Up, U, NW;           // packed units, all units, active warps (min(grid * kDWarps, U))
  int32_t M, K, K_pad, MT, KT, OT, KO, batch;
  int32_t xs_bytes;            // staged x incl. ones and zero blocks, multiple of 128
  int32_t x_vec16;             // x rows 16-byte loadable
  uint32_t negz;
};

__device__ __forceinline__ void cp_async_wait_ring() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kDRing - 1) : "memory");
}

// x chunk (columns k..k+7 of batch row b), zero past K.
__device__ __forceinline__ uint4 gemvd_x_chunk(const GemvDArgs& a, int b, int k) {
  const __half* src = a.x + b * a.ldx + k;
  if (a.x_vec16) return k < a.K ? ld_cg_v4(src) : make_uint4(0, 0, 0, 0);
  uint16_t h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) h[e] = (k + e < a.K) ? __ldcg(reinterpret_cast<const unsigned short*>(src) + e) : 0;
  return make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16), h[4] | (uint32_t(h[5]) << 16),
                    h[6] | (uint32_t(h[7]) << 16));
}

// The active warp whose range holds unit u (the ranges are [w U / NW, (w+1) U / NW)).
__device__ __forceinline__ uint32_t gemvd_warp_of(uint32_t u, uint32_t U, uint32_t NW) {
  return ((u + 1u) * NW - 1u) / U;
}

__global__ void __launch_bounds__(kDThreads, 1) gemvd_kernel(const GemvDArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint32_t amax_bits[kQMaxBatch];
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const uint32_t xs_base = smem_u32(smem);
  const uint32_t ring = xs_base + static_cast<uint32_t>(a.xs_bytes) + warp * (kDRing * kUnitBytes) + lane * 16;
  const uint32_t U = static_cast<uint32_t>(a.U), NW = static_cast<uint32_t>(a.NW);
  const uint32_t gw = blockIdx.x * kDWarps + warp;
  int32_t u0 = 0, u1 = 0;
  if (gw < NW) {
    u0 = static_cast<int32_t>((gw * U) / NW);
    u1 = static_cast<int32_t>(((gw + 1u) * U) / NW);
  }
  // weights do not depend on the previous kernel: request the first units before waiting for it
#pragma unroll
  for (int i = 0; i < kDRing - 1; ++i) {
    const int32_t u = u0 + i;
    if (u < u1) {
      const uint8_t* src = u < a.Up ? a.units + static_cast<int64_t>(u) * kUnitBytes
                                    : a.ounits + static_cast<int64_t>(u - a.Up) * kUnitBytes;
      cp_async16(ring + i * kUnitBytes, src + lane * 16);
    }
    cp_async_commit();
  }
  if (tid < kQMaxBatch) amax_bits[tid] = 0u;
  __syncthreads();
  griddep_launch_dependents();
  griddep_wait();  // x (and the workspace) may be written by the previous kernel

  // ---- stage x: max |x| per batch row, then the offset digits at their staged positions
  const int per_row = a.K_pad / 8;
  float mx0 = 0.f, mx1 = 0.f;
  for (int b = 0; b < a.batch; ++b)
    for (int c = tid; c < per_row; c += kDThreads) {
      const float m = chain_chunk_amax(gemvd_x_chunk(a, b, c * 8));
      if (b == 0) mx0 = fmaxf(mx0, m);
      else mx1 = fmaxf(mx1, m);
    }
  {
    // non-negative floats order like their bit patterns (a NaN maximum counts as 0)
    const uint32_t m0 = __reduce_max_sync(0xffffffffu, mx0 == mx0 ? __float_as_uint(mx0) : 0u);
    const uint32_t m1 = __reduce_max_sync(0xffffffffu, mx1 == mx1 ? __float_as_uint(mx1) : 0u);
    if (lane == 0) {
      atomicMax(&amax_bits[0], m0);
      atomicMax(&amax_bits[1], m1);
    }
  }
  if (tid < 16)  // ones block, zero block (B operands of the ones and absent columns)
    sts128(xs_base + a.xs_bytes - kQZeroBytes - kQOnesBytes + tid * 16,
           tid < 8 ? make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u) : make_uint4(0, 0, 0, 0));
  __syncthreads();
  const float fm0 = __uint_as_float(amax_bits[0]), fm1 = __uint_as_float(amax_bits[1]);
  const int ex0 = fm0 > 0.f ? 22 - frexp_exponent(fm0) : 0;
  const int ex1 = fm1 > 0.f ? 22 - frexp_exponent(fm1) : 0;
  const uint32_t colb = static_cast<uint32_t>(xsq_col_bytes(a.KT));
  for (int b = 0; b < a.batch; ++b)
    for (int c = tid; c < per_row; c += kDThreads) {
      const int k = c * 8;
      chain_store_digits(gemvd_x_chunk(a, b, k), pow2f(b == 0 ? ex0 : ex1), xs_base + 3 * b * colb, colb,
                         static_cast<uint32_t>((k >> 7) * 128 + xs_pos8(k & 127)));
    }
  __syncthreads();
  if (u0 >= u1) return;

  // ---- this warp's units
  const int g = lane >> 2, q = lane & 3;
  const int bcol = g >> 2, dig = g & 3;
  const bool live_col = dig < 3 && bcol < a.batch;
  const uint32_t colbase = live_col ? xs_base + (3 * bcol + dig) * colb
                                    : xs_base + a.xs_bytes - (bcol < a.batch ? kQZeroBytes + kQOnesBytes : kQZeroBytes);
  const uint32_t kts = live_col ? 128u : 0u;
  const uint32_t xq = colbase + 32 * q, xo = colbase + 4 * q;
  GemvQArgs qa;  // the view load_metaq takes
  qa.cbq = a.cbq; qa.tile_mask = a.tile_mask; qa.orow = a.orow; qa.oexp = a.oexp; qa.M = a.M; qa.MT = a.MT;
  int32_t seg, sb, se;  // current segment: index, first unit, end unit
  if (u0 < a.Up) {
    seg = u0 / a.KT;
    sb = seg * a.KT;
    se = sb + a.KT;
  } else {
    const int32_t t = (u0 - a.Up) / a.KO;
    seg = a.MT + t;
    sb = a.Up + t * a.KO;
    se = sb + a.KO;
  }
  MetaQ cur = load_metaq(qa, seg, g);
  MetaQ nxt = cur;  // the next segment's, in flight while this one streams
  if (se < u1) nxt = load_metaq(qa, seg + 1, g);
  AccQ A;
  zero_accq(A);
  const int b = q >> 1;
  const bool live_out = !(q & 1) && b < a.batch;
  const int ex = b ? ex1 : ex0;
#pragma unroll 1
  for (int32_t u = u0; u < u1; ++u) {
    {  // refill the slot of unit u - 1 with unit u + kDRing - 1
      const int32_t un = u + kDRing - 1;
      if (un < u1) {
        const uint8_t* src = un < a.Up ? a.units + static_cast<int64_t>(un) * kUnitBytes
                                       : a.ounits + static_cast<int64_t>(un - a.Up) * kUnitBytes;
        cp_async16(ring + ((un - u0) & (kDRing - 1)) * kUnitBytes, src + lane * 16);
      }
      cp_async_commit();
    }
    cp_async_wait_ring();  // unit u has landed (this lane's 16 bytes of it)
    const uint4 wv = lds128(ring + ((u - u0) & (kDRing - 1)) * kUnitBytes);
    const int32_t kb = u - sb;
    if (seg < a.MT) {
      const uint32_t xa = xq + static_cast<uint32_t>(kb) * kts;
      const uint4 b01 = lds128(xa), b23 = lds128(xa + 16);
      const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t Ah[4], Al[4];
        decode_word_q(w[j], cur.qh, cur.ql, a.negz, Ah, Al);
        imma16832(A.h[j & 1], Ah, bb[2 * j], bb[2 * j + 1]);
        imma16832(A.l[j & 1], Al, bb[2 * j], bb[2 * j + 1]);
      }
    } else {
      const uint32_t bv = lds32(xo + static_cast<uint32_t>(kb >> 3) * kts + (kb & 7) * 16);
      if (kb & 1) {  // two accumulator chains, indexed statically (a runtime index would put A in local memory)
        imma16816(A.h[1], wv.x, wv.y, bv);
        imma16816(A.l[1], wv.z, wv.w, bv);
      } else {
        imma16816(A.h[0], wv.x, wv.y, bv);
        imma16816(A.l[0], wv.z, wv.w, bv);
      }
    }
    if (u + 1 == se || u + 1 == u1) {  // a segment of the range is complete
      long long t[2];
      finish_dot(A, q, t);
      if (sb >= u0 && se <= u1) {  // the whole tile is this warp's
        if (live_out) {
          if (cur.row[0] >= 0) a.y[b * a.ldy + cur.row[0]] = scale_to_half(t[0], cur.e[0] + ex);
          if (cur.row[1] >= 0) a.y[b * a.ldy + cur.row[1]] = scale_to_half(t[1], cur.e[1] + ex);
        }
      } else {
        const int need = static_cast<int>(gemvd_warp_of(static_cast<uint32_t>(se - 1), U, NW) -
                                          gemvd_warp_of(static_cast<uint32_t>(sb), U, NW)) + 1;
        if (live_out) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (cur.row[r] < 0) continue;
            unsigned long long* p = a.acc + static_cast<int64_t>(cur.row[r]) * 2 + b;
            const unsigned long long d = kCountOne + static_cast<unsigned long long>(t[r]);
            long long tot;
            if (count_add_complete(atomicAdd(p, d), d, need, &tot)) {
              *p = 0ull;
              a.y[b * a.ldy + cur.row[r]] = scale_to_half(tot, cur.e[r] + ex);
            }
          }
        }
      }
      if (u + 1 == u1) break;
      zero_accq(A);
      ++seg;
      sb = se;
      se = sb + (seg < a.MT ? a.KT : a.KO);
      cur = nxt;
      if (se < u1) nxt = load_metaq(qa, seg + 1, g);
    }
  }
}

}  // namespace opc
