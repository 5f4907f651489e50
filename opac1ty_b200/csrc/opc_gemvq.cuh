// opc_gemvq.cuh -- fused 2-bit codebook GEMV for batch 1..2 with exact integer accumulation.
//
// Same computation as opc_gemv.cuh (y = x . W_hat^T, W_hat from the per-row 4-entry codebooks
// plus outlier rows; reference semantics opacc1ty/export/converter.py:26-67), organised so that
// each 16 weights cost 8 PRMT + 3 other ALU operations and 2 int8 mma.sync:
//
//  * Every row's fp16 centroids are stored as integers n = cb * 2^e_r (|n| <= 2^14, exact for
//    centroids within 2^4 of the row's largest, else rounded to 2^-14 of it), split into two
//    int8 parts n = 256*hi + lo.  One PRMT per part gathers four int8 weights, its selector
//    being the masked index word itself (decode_word_q).
//  * x is staged per CTA as integers m = round(x * 2^e_x), |m| < 2^22 (e_x from the CTA's max
//    |x|), stored offset as m' = m + 2^22 in [0, 2^23): one FFMA per value yields a float whose
//    low three bytes are m' itself (x_digits_q), and those bytes are the unsigned digits
//    m' = 65536*d0 + 256*d1 + d2, placed in three B-operand columns (int8 x uint8 mma.sync).  A
//    fourth column of ones gives each row's weight sum W, and T = T' - 2^22 W removes the offset:
//    one m16n8k32 per codebook part yields all eight column products, in int32 and exactly.
//  * At the end of a row tile the products combine into the exact int64 dot product
//    T = sum_k n_k m_k, and y = fp16(T * 2^-(e_r + e_x)) is rounded once.  Partial sums of a tile
//    split between warps or CTAs are int64 and add exactly (atomics included), so the result
//    does not depend on the partition or on arrival order.
//  * A dedicated producer warp streams each consumer warp's contiguous unit range through that
//    warp's ring of shared-memory stages with bulk async copies (no multicast); consumers wait
//    on "full" mbarriers and release stages through "empty" mbarriers.  The producer starts
//    before griddepcontrol.wait, so weights stream while the previous kernel finishes.
#pragma once

#include "opc_device.cuh"

namespace opc {

constexpr int kQConsumers = 15;                    // consumer warps per CTA (+1 producer: 4 warps per SM sub-partition)
constexpr int kQProducerWarp = kQConsumers;        // warp index of the producer
constexpr int kQThreads = (kQConsumers + 1) * 32;
constexpr int kQConsumerThreads = kQConsumers * 32;
constexpr int kQChunkUnits = 8;   // 4 KB per bulk copy: measured 6.9 TB/s streaming (2 KB copies: 5.3)
constexpr int kQChunkBytes = kQChunkUnits * kUnitBytes;
constexpr int kQMaxStages = 4;
constexpr int kQMaxBatch = 2;
constexpr int kQZeroBytes = 128;                   // B operand of absent columns (zeros) ...
constexpr int kQOnesBytes = 128;                   // ... and of the ones columns; both end the staged x

// Staged x: column c = 3*b + d (batch row b, digit d) is a row of KT*128 + 16 bytes; k of block kt
// sits at byte 128*kt + xs_pos8(k & 127).  The last 256 bytes of the staged area are a block of
// ones and a block of zeros, read with stride 0 by the ones and absent columns.
__host__ __device__ constexpr int xsq_col_bytes(int KT) { return KT * 128 + 16; }

struct GemvQArgs {
  const uint8_t* units;        // packed units (unit u at units + 512u)
  const uint8_t* ounits;       // int8 outlier units (unit u >= Up at ounits + 512(u - Up))
  const uint4* cbq;            // [M_pad] {hi x4, lo x4, e_r, 0}
  const uint16_t* tile_mask;   // [MT]
  const int32_t* orow;         // [OT*16] output row of each outlier slot, -1 = padding
  const int32_t* oexp;         // [OT*16] exponent of each outlier slot's integer row
  const __half* x;
  __half* y;
  unsigned long long* acc;     // [M_pad][2] int64 partial dot products of CTA-spanning tiles (zero)
  int32_t* counters;           // [MT + OT] arrivals per tile (zero)
  int64_t ldx, ldy;
  int32_t Up, U;
  int32_t M, K, K_pad, MT, KT, OT, KO, batch;
  int32_t stages;              // ring stages per consumer warp (2..kQMaxStages)
  int32_t xs_bytes;            // staged x incl. zero block, multiple of 128
  int32_t x_vec16;             // x rows 16-byte loadable
  uint32_t negz;
};

struct SegQ {
  int32_t id, begin, end;
};
__device__ __forceinline__ SegQ segq_at(const GemvQArgs& a, int32_t u) {
  if (u < a.Up) {
    const int32_t t = u / a.KT;
    return {t, t * a.KT, (t + 1) * a.KT};
  }
  const int32_t t = (u - a.Up) / a.KO;
  return {a.MT + t, a.Up + t * a.KO, a.Up + (t + 1) * a.KO};
}

struct CursorQ {
  int32_t u, seg, begin, end;
};
__device__ __forceinline__ CursorQ cursorq_at(const GemvQArgs& a, int32_t u) {
  const SegQ s = segq_at(a, u);
  return {u, s.id, s.begin, s.end};
}
__device__ __forceinline__ int32_t chunkq_units(const CursorQ& c, int32_t u1) {
  int32_t n = c.end - c.u;
  if (u1 - c.u < n) n = u1 - c.u;
  return n < kQChunkUnits ? n : kQChunkUnits;
}
__device__ __forceinline__ void nextq_segment(const GemvQArgs& a, CursorQ& c) {
  c.seg += 1;
  c.begin = c.end;
  c.end = c.begin + (c.seg < a.MT ? a.KT : a.KO);
}

__host__ __device__ __forceinline__ int32_t partq_start(int32_t i, int32_t n, int32_t p) {
  return static_cast<int32_t>(static_cast<int64_t>(i) * n / p);
}
__host__ __device__ __forceinline__ int32_t partq_of(int32_t e, int32_t n, int32_t p) {
  return static_cast<int32_t>((static_cast<int64_t>(e + 1) * p + n - 1) / n - 1);
}

// Per-segment data of a lane: integer codebooks and exponents of rows g, g+8, output rows.
struct MetaQ {
  uint32_t qh[2], ql[2];
  int32_t e[2];
  int32_t row[2];
};
__device__ __forceinline__ MetaQ load_metaq(const GemvQArgs& a, int32_t seg, int g) {
  MetaQ m;
  if (seg < a.MT) {
    const int r0 = seg * kTileRows + g;
    const uint4 c0 = ld_nc_v4(a.cbq + r0), c1 = ld_nc_v4(a.cbq + r0 + 8);
    const uint32_t mask = ld_nc_u16(a.tile_mask + seg);
    m.qh[0] = c0.x; m.ql[0] = c0.y; m.e[0] = static_cast<int32_t>(c0.z);
    m.qh[1] = c1.x; m.ql[1] = c1.y; m.e[1] = static_cast<int32_t>(c1.z);
    m.row[0] = (r0 < a.M && !((mask >> g) & 1u)) ? r0 : -1;
    m.row[1] = (r0 + 8 < a.M && !((mask >> (g + 8)) & 1u)) ? r0 + 8 : -1;
  } else {
    const int s = (seg - a.MT) * kTileRows + g;
    m.qh[0] = m.qh[1] = m.ql[0] = m.ql[1] = 0u;
    m.row[0] = static_cast<int32_t>(ld_nc_u32(a.orow + s));
    m.row[1] = static_cast<int32_t>(ld_nc_u32(a.orow + s + 8));
    m.e[0] = static_cast<int32_t>(ld_nc_u32(a.oexp + s));
    m.e[1] = static_cast<int32_t>(ld_nc_u32(a.oexp + s + 8));
  }
  return m;
}

// Accumulators: [codebook part hi/lo][4 C-fragment values], two chains each.
struct AccQ {
  int32_t h[2][4], l[2][4];
};
__device__ __forceinline__ void zero_accq(AccQ& A) {
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) A.h[c][e] = A.l[c][e] = 0;
}

// Exact int64 dot products of rows g (t[0]) and g+8 (t[1]) for batch row q>>1, valid in lanes
// with even q.  C fragment: element e is (row g + 8*(e>>1), column 2q + (e&1)); columns 0,1,2 are
// the digits d0,d1,d2 of batch row 0 and 4,5,6 those of batch row 1; 3 and 7 are the ones
// columns (zero for an absent batch row).
// T = 2^24 H0 + 2^16 (H1 + L0) + 2^8 (H2 + L1) + L2 - 2^22 (2^8 H3 + L3), with H/L the hi/lo
// codebook-part products: the digits hold m + 2^22, and the ones column's products sum the row's
// weights over the same k (a partial range's offset cancels within that range).
__device__ __forceinline__ void finish_dot(const AccQ& A, int q, long long t[2]) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const long long h0 = static_cast<long long>(A.h[0][2 * r]) + A.h[1][2 * r];
    const long long h1 = static_cast<long long>(A.h[0][2 * r + 1]) + A.h[1][2 * r + 1];
    const long long l0 = static_cast<long long>(A.l[0][2 * r]) + A.l[1][2 * r];
    const long long l1 = static_cast<long long>(A.l[0][2 * r + 1]) + A.l[1][2 * r + 1];
    long long v;
    if ((q & 1) == 0)
      v = (h0 << 24) + ((h1 + l0) << 16) + (l1 << 8);  // columns d0, d1
    else
      v = (h0 << 8) + l0 - (((h1 << 8) + l1) << 22);   // columns d2, ones
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    t[r] = v;
  }
}

// Eight fp16 values of x (packed pairs) as offset integers m' = round(x * 2^ex) + 2^22, for
// |x| * 2^ex < 2^22.  x * 2^ex is exact, and adding 1.5 * 2^23 in the same FFMA rounds it to an
// integer (to nearest, ties to even) with a float whose low 23 bits are then m' itself.  Byte
// permutes gather the three bytes of m' of four values into one word per digit column: d2 (low
// byte), d1, d0 (high byte, < 128).  A zero (padding past K included) encodes as 2^22 like any
// other zero, so the ones column may cover the whole padded row.
struct XDigitsQ {
  uint32_t d[3][2];  // [column d0, d1, d2][values 0-3, 4-7]
};
__device__ __forceinline__ XDigitsQ x_digits_q(const uint4& v, float sc) {
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  uint32_t f[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
    f[2 * e] = __float_as_uint(fmaf(p.x, sc, 12582912.0f));
    f[2 * e + 1] = __float_as_uint(fmaf(p.y, sc, 12582912.0f));
  }
  XDigitsQ r;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t* g4 = f + 4 * h;
    const uint32_t lo01 = prmt(g4[0], g4[1], 0x5140u), lo23 = prmt(g4[2], g4[3], 0x5140u);  // bytes 0, 1
    const uint32_t hi01 = prmt(g4[0], g4[1], 0x0062u), hi23 = prmt(g4[2], g4[3], 0x0062u);  // byte 2
    r.d[2][h] = prmt(lo01, lo23, 0x5410u);
    r.d[1][h] = prmt(lo01, lo23, 0x7632u);
    r.d[0][h] = prmt(hi01, hi23, 0x5410u);
  }
  return r;
}

__device__ __forceinline__ __half scale_to_half(long long t, int e) {
  // t * 2^-e, rounded once: |t| < 2^53 converts exactly, the power of two is exact.
  const double s = __longlong_as_double(static_cast<long long>(1023 - e) << 52);
  return __double2half(static_cast<double>(t) * s);
}

struct SmemSlotsQ {
  long long v[kQConsumers][2][32][2];  // per warp: first/last segment, per lane rows g/g+8
  int32_t seg[kQConsumers][2];
  int32_t ex[kQMaxBatch];              // x exponents
  uint32_t amax_bits[kQMaxBatch];      // staging: max |x| (float bits) per batch row
};

// x exponents of batch rows 0 and 1 are passed as scalars (no array, so no local memory).
__device__ __forceinline__ void write_outq(const GemvQArgs& a, const MetaQ& m, const long long t[2], int q, int ex0,
                                           int ex1) {
  const int b = q >> 1;
  if ((q & 1) || b >= a.batch) return;
  const int ex = b ? ex1 : ex0;
#pragma unroll
  for (int r = 0; r < 2; ++r)
    if (m.row[r] >= 0) a.y[b * a.ldy + m.row[r]] = scale_to_half(t[r], m.e[r] + ex);
}

__device__ __forceinline__ void put_slotq(SmemSlotsQ* ss, int warp, int sl, int lane, int32_t seg, const long long t[2]) {
  ss->v[warp][sl][lane][0] = t[0];
  ss->v[warp][sl][lane][1] = t[1];
  if (lane == 0) ss->seg[warp][sl] = seg;
}

// Sum segment S over the CTA's warps, then write y (S inside the CTA's range) or add into the
// global accumulators, the last CTA to arrive writing y and clearing them.
__device__ void reduce_segmentq(const GemvQArgs& a, SmemSlotsQ* ss, SegQ S, int32_t c0, int32_t c1, int lane,
                                int g, int q) {
  const int32_t n = c1 - c0;
  const int32_t lo = S.begin > c0 ? S.begin : c0;
  const int32_t hi = (S.end < c1 ? S.end : c1) - 1;
  const int wa = partq_of(lo - c0, n, kQConsumers), wb = partq_of(hi - c0, n, kQConsumers);
  long long tot[2] = {0, 0};
  for (int w = wa; w <= wb; ++w) {
    const int32_t ws = c0 + partq_start(w, n, kQConsumers), we = c0 + partq_start(w + 1, n, kQConsumers);
    if (we <= ws) continue;
    const int sl = (ws >= S.begin) ? 0 : 1;
    tot[0] += ss->v[w][sl][lane][0];
    tot[1] += ss->v[w][sl][lane][1];
  }
  const MetaQ m = load_metaq(a, S.id, g);
  if (S.begin >= c0 && S.end <= c1) {
    write_outq(a, m, tot, q, ss->ex[0], ss->ex[1]);
    return;
  }
  const int b = q >> 1;
  const bool live = !(q & 1) && b < a.batch;
  if (live) {
#pragma unroll
    for (int r = 0; r < 2; ++r)
      if (m.row[r] >= 0) atomicAdd(a.acc + static_cast<int64_t>(m.row[r]) * 2 + b, static_cast<unsigned long long>(tot[r]));
  }
  __syncwarp();  // the lanes' adds are ordered before lane 0's arrival
  const int G = static_cast<int>(gridDim.x);
  const int ca = partq_of(S.begin, a.U, G), cb = partq_of(S.end - 1, a.U, G);
  int old = 0;
  if (lane == 0) old = atom_add_acq_rel_gpu(a.counters + S.id, 1);  // release ours, acquire earlier ones
  old = __shfl_sync(0xffffffffu, old, 0);
  __syncwarp();
  if (old != cb - ca) return;
  if (live) {
    long long fin[2] = {0, 0};
#pragma unroll
    for (int r = 0; r < 2; ++r)
      if (m.row[r] >= 0)
        fin[r] = static_cast<long long>(atomicExch(a.acc + static_cast<int64_t>(m.row[r]) * 2 + b, 0ull));
    write_outq(a, m, fin, q, ss->ex[0], ss->ex[1]);
  }
  if (lane == 0) atomicExch(a.counters + S.id, 0);
}

__global__ void __launch_bounds__(kQThreads, 1) gemvq_kernel(const GemvQArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int32_t c0 = partq_start(cta, a.U, G), c1 = partq_start(cta + 1, a.U, G);
  const int32_t n_cta = c1 - c0;
  const int S = a.stages;

  const uint32_t xs_base = smem_u32(smem);
  const uint32_t ring_base = xs_base + a.xs_bytes;
  const uint32_t full_base = ring_base + kQConsumers * S * kQChunkBytes;
  const uint32_t empty_base = full_base + kQConsumers * S * 8;
  SmemSlotsQ* ss = reinterpret_cast<SmemSlotsQ*>(smem + a.xs_bytes + kQConsumers * S * (kQChunkBytes + 16));

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQConsumers * S; ++i) {
      mbar_init(full_base + i * 8, 1);
      mbar_init(empty_base + i * 8, 1);
    }
    fence_mbar_init();
  }
  if (threadIdx.x < kQConsumers * 2) ss->seg[threadIdx.x >> 1][threadIdx.x & 1] = -1;
  if (threadIdx.x < kQMaxBatch) ss->amax_bits[threadIdx.x] = 0u;
  __syncthreads();
  griddep_launch_dependents();

  // ------------------------------------------------------------------ producer warp
  if (warp == kQProducerWarp) {
    const int i = lane;  // consumer warp served by this lane
    int32_t u1 = 0;
    CursorQ pc = {0, 0, 0, 0};
    bool active = false;
    if (i < kQConsumers) {
      const int32_t u0 = c0 + partq_start(i, n_cta, kQConsumers);
      u1 = c0 + partq_start(i + 1, n_cta, kQConsumers);
      active = u0 < u1;
      if (active) pc = cursorq_at(a, u0);
    }
    const uint32_t ring = ring_base + i * S * kQChunkBytes;
    int32_t c = 0;
    uint64_t t_idle = 0;
    bool failed = false;
    while (__any_sync(0xffffffffu, active)) {
      bool issued = false;
      if (active) {
        const int slot = c % S;
        const int round = c / S;
        if (round == 0 || mbar_test(empty_base + (i * S + slot) * 8, static_cast<uint32_t>((round - 1) & 1))) {
          const int32_t cnt = chunkq_units(pc, u1);
          const uint32_t bar = full_base + (i * S + slot) * 8;
          mbar_expect_tx(bar, static_cast<uint32_t>(cnt * kUnitBytes));
          const uint8_t* src = pc.u < a.Up ? a.units + static_cast<int64_t>(pc.u) * kUnitBytes
                                           : a.ounits + static_cast<int64_t>(pc.u - a.Up) * kUnitBytes;
          bulk_g2s(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar);
          pc.u += cnt;
          if (pc.u == pc.end) nextq_segment(a, pc);
          ++c;
          issued = true;
          if (pc.u >= u1) active = false;
        }
      }
      if (__any_sync(0xffffffffu, issued)) {
        t_idle = 0;
      } else {
        const uint64_t now = globaltimer_ns();
        if (t_idle == 0) t_idle = now;
        else if (now - t_idle > kWaitLimitNs) {
          failed = true;
          break;
        }
        nanosleep_ns(64);
      }
    }
    if (failed && lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  const int g = lane >> 2, q = lane & 3;
  const int32_t u0 = c0 + partq_start(warp, n_cta, kQConsumers), u1 = c0 + partq_start(warp + 1, n_cta, kQConsumers);
  const int32_t n_units = u1 - u0;
  const int tid = threadIdx.x;  // 0 .. kQConsumerThreads-1

  griddep_wait();  // x and the workspace may be written by the previous kernel

  // Stage x: pass 1, max |x| per batch row; pass 2, integer digits at their staged positions.
  // Each pass loads 8 chunks of 8 halves per thread at once (all loads in flight together).
  {
    const int per_row = a.K_pad / 8;
    const int total = a.batch * per_row;
    auto load8 = [&](int base, uint4 v[8]) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = base + i * kQConsumerThreads;
        v[i] = make_uint4(0, 0, 0, 0);
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          if (a.x_vec16) {
            if (k < a.K) v[i] = ld_cg_v4(a.x + b * a.ldx + k);
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
    };
    float mx[kQMaxBatch] = {0.f, 0.f};
    for (int base = tid; base < total; base += 8 * kQConsumerThreads) {
      uint4 v[8];
      load8(base, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = base + i * kQConsumerThreads;
        if (c < total) {
          const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          float m = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
            m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
          }
          if (c / per_row == 0) mx[0] = fmaxf(mx[0], m);
          else mx[1] = fmaxf(mx[1], m);
        }
      }
    }
    // non-negative floats order like their bit patterns: one warp max and one shared-memory
    // atomic per warp and batch row (a NaN maximum counts as 0, as fmaxf would skip it)
#pragma unroll
    for (int b = 0; b < kQMaxBatch; ++b) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, mx[b] == mx[b] ? __float_as_uint(mx[b]) : 0u);
      if (lane == 0) atomicMax(&ss->amax_bits[b], m);
    }
    if (tid < 16)  // ones block, zero block (B operands of the ones and absent columns)
      sts128(xs_base + a.xs_bytes - kQZeroBytes - kQOnesBytes + tid * 16,
             tid < 8 ? make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u) : make_uint4(0, 0, 0, 0));
    named_barrier(1, kQConsumerThreads);
    // max |x| * 2^e in [2^21, 2^22): offset digits d0 in [0, 128], d1, d2 in [0, 255]
    const float m0 = __uint_as_float(ss->amax_bits[0]), m1 = __uint_as_float(ss->amax_bits[1]);
    const int ex0 = m0 > 0.f ? 22 - frexp_exponent(m0) : 0;
    const int ex1 = m1 > 0.f ? 22 - frexp_exponent(m1) : 0;
    if (tid == 0) {
      ss->ex[0] = ex0;
      ss->ex[1] = ex1;
    }
    const uint32_t colb = static_cast<uint32_t>(xsq_col_bytes(a.KT));
    for (int base = tid; base < total; base += 8 * kQConsumerThreads) {
      uint4 v[8];
      load8(base, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = base + i * kQConsumerThreads;
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          const float sc = __int_as_float((127 + (b == 0 ? ex0 : ex1)) << 23);  // exact 2^e
          const XDigitsQ d = x_digits_q(v[i], sc);
          const uint32_t pos = static_cast<uint32_t>((k >> 7) * 128 + xs_pos8(k & 127));
#pragma unroll
          for (int dd = 0; dd < 3; ++dd) sts64(xs_base + (3 * b + dd) * colb + pos, d.d[dd][0], d.d[dd][1]);
        }
      }
    }
  }
  named_barrier(1, kQConsumerThreads);  // x staged, exponents published

  // B-operand column of this lane: batch row g>>2, digit g&3 (digit 3: the ones block; absent
  // batch rows: the zero block).
  const int bcol = g >> 2, dig = g & 3;
  const bool live_col = dig < 3 && bcol < a.batch;
  const uint32_t colbase = live_col ? xs_base + (3 * bcol + dig) * xsq_col_bytes(a.KT)
                                    : xs_base + a.xs_bytes - (bcol < a.batch ? kQZeroBytes + kQOnesBytes : kQZeroBytes);
  const uint32_t kts = live_col ? 128u : 0u;
  const uint32_t xq = colbase + 32 * q;  // packed units: 32 bytes per k block
  const uint32_t xo = colbase + 4 * q;   // outlier units: 4 bytes at 16*(s&7) per k block
  const uint32_t negz = a.negz;
  const uint32_t ring = ring_base + warp * S * kQChunkBytes + lane * 16;
  const uint32_t fullw = full_base + warp * S * 8, emptyw = empty_base + warp * S * 8;

  bool ok = true;
  if (n_units > 0) {
    const int32_t n_seg = a.MT + a.OT;
    CursorQ cc = cursorq_at(a, u0);
    MetaQ cur = load_metaq(a, cc.seg, g);
    MetaQ nxt = cur;
    if (cc.seg + 1 < n_seg) nxt = load_metaq(a, cc.seg + 1, g);
    AccQ A;
    zero_accq(A);
    int slot = 0;
    uint32_t phase = 0;
    while (cc.u < u1) {
      if (!mbar_wait_bounded(fullw + slot * 8, phase)) {
        ok = false;
        break;
      }
      const int32_t cnt = chunkq_units(cc, u1);
      const uint32_t stage = ring + slot * kQChunkBytes;
      const int32_t k0 = cc.u - cc.begin;
      if (cc.seg < a.MT) {
#pragma unroll 1
        for (int i = 0; i < cnt; ++i) {  // not unrolled: measured as fast, and far less code
          const uint4 wv = lds128(stage + i * kUnitBytes);
          const uint32_t xa = xq + static_cast<uint32_t>(k0 + i) * kts;
          const uint4 b01 = lds128(xa), b23 = lds128(xa + 16);
          const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
          const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t Ah[4], Al[4];
            decode_word_q(w[j], cur.qh, cur.ql, negz, Ah, Al);
            imma16832(A.h[j & 1], Ah, bb[2 * j], bb[2 * j + 1]);
            imma16832(A.l[j & 1], Al, bb[2 * j], bb[2 * j + 1]);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kQChunkUnits; ++i) {
          if (i < cnt) {
            const uint4 av = lds128(stage + i * kUnitBytes);
            const int32_t s = k0 + i;
            const uint32_t bv = lds32(xo + static_cast<uint32_t>(s >> 3) * kts + (s & 7) * 16);
            imma16816(A.h[i & 1], av.x, av.y, bv);
            imma16816(A.l[i & 1], av.z, av.w, bv);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(emptyw + slot * 8);
      if (++slot == S) {
        slot = 0;
        phase ^= 1u;
      }
      cc.u += cnt;
      if (cc.u == cc.end && cc.u < u1) {  // segment complete inside the range
        long long t[2];
        finish_dot(A, q, t);
        if (cc.begin < u0)
          put_slotq(ss, warp, 0, lane, cc.seg, t);
        else
          write_outq(a, cur, t, q, ss->ex[0], ss->ex[1]);
        zero_accq(A);
        nextq_segment(a, cc);
        cur = nxt;
        if (cc.seg + 1 < n_seg) nxt = load_metaq(a, cc.seg + 1, g);
      }
    }
    if (ok) {
      long long t[2];
      finish_dot(A, q, t);
      if (cc.begin >= u0 && cc.end <= u1)
        write_outq(a, cur, t, q, ss->ex[0], ss->ex[1]);
      else
        put_slotq(ss, warp, cc.begin <= u0 ? 0 : 1, lane, cc.seg, t);
    } else {
      if (lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
      for (int st = 0; st < S; ++st) (void)mbar_wait_bounded(fullw + st * 8, 0);
    }
  }
  named_barrier(1, kQConsumerThreads);  // every warp's partials are in shared memory
  if (!ok || n_units <= 0) return;

  const int32_t s0 = ss->seg[warp][0], s1 = ss->seg[warp][1];
  if (s0 >= 0) {
    const SegQ Sg = segq_at(a, s0 < a.MT ? s0 * a.KT : a.Up + (s0 - a.MT) * a.KO);
    const bool first_is_last = (Sg.end >= u1);
    if ((Sg.begin < u0 && u0 == c0) || (first_is_last && Sg.begin >= u0))
      reduce_segmentq(a, ss, Sg, c0, c1, lane, g, q);
  }
  if (s1 >= 0) {
    const SegQ Sg = segq_at(a, s1 < a.MT ? s1 * a.KT : a.Up + (s1 - a.MT) * a.KO);
    if (Sg.begin >= u0 || u0 == c0) reduce_segmentq(a, ss, Sg, c0, c1, lane, g, q);
  }
}

}  // namespace opc
