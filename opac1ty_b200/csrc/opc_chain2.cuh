// opc_chain2.cuh -- the decode step as a dataflow over 128-column blocks (batch 1, one GPU).
//
// Same per-layer arithmetic as opc_gemvq.cuh (8 PRMT + 3 other ALU operations and two int8
// mma.sync per 16 weights, exact integer dot products, one fp16 rounding per output), with the
// activations exchanged between layers in their integer digit form instead of fp16:
//
//  * The fixed-point scale of a layer's input is chosen BEFORE that input is computed, from a
//    bound: |y_r| <= ||W row r||_2 * ||x||_2 (Cauchy-Schwarz).  For layer j+1 the exponent e_{j+1}
//    satisfies  wbound_j * ||x_j||_2 * 2^e_{j+1} < 2^29,  where wbound_j >= every row norm of
//    layer j (host-computed) and ||x_j||_2 comes from an exact integer sum over x_j's digits.  So
//    every CTA computes the same e_{j+1} as soon as it holds x_j, and no maximum over the finished
//    outputs is needed: no grid-wide reduction, no barrier between layers.
//  * The warp that finishes output row r of layer j rounds it to fp16 h (what callers read),
//    forms m = round(h * 2^e_{j+1}) (|m| < 2^29) and stores the four offset digits of
//    m + 2^30 straight into x_{j+1}'s digit buffer, in the exact byte layout the shared-memory
//    B operands use; per 128-row block it then adds the rows' sum of a^2 (a = (|m| >> 14) + 1,
//    for the next bound) and releases the block's row counter.
//  * One staging warp per CTA polls the counters of x_{j+1}'s blocks (acquire) and copies each
//    complete block (512 bytes) into shared memory with one bulk async copy completing on that
//    block's mbarrier.  Consumer warps wait only on the blocks their units use, so a warp starts a
//    layer as soon as its own blocks are in: no CTA-wide barrier per layer, no per-CTA x
//    conversion, no max|x| barrier.  x is double-buffered by layer parity, so the next layer is
//    staged while slow warps still finish this one.
//  * Layer 0 reads the caller's fp16 input and derives its scale from max|x| as the per-launch
//    GEMV does; the chain's output is fp16 like every layer's.
//
// Digit layout of a 128-column block (512 bytes, in global memory and in shared memory alike):
// plane d (0..3, d = 0 the most significant digit) at byte 128d; within a plane the byte of k
// (0..127) is xs_pos8(k) with its 16-byte chunk index XOR-ed with d.  A lane reading digit column
// g (its B-operand column) at logical chunks (2q, 2q+1) then hits the physical chunks
// (2q ^ g, (2q+1) ^ g): the eight lanes of each quarter warp touch eight distinct chunks (all 32
// banks), and the outlier units' 4-byte reads (chunk s & 7) are conflict-free as well.
// B-operand columns: 0..3 the digit planes, 4 ones (removes the 2^30 offset exactly), 5..7 zero.
//
// Every wait is bounded (kWaitLimitNs); a role that gives up records device error 3 and sets the
// CTA's abort flag, which every other wait loop of the CTA polls.  A layer whose output is not
// finite records device error 5 (its digits are those of the clamped value).
#pragma once

#include "opc_chain.cuh"

namespace opc {

constexpr int kC2Digits = 4;                       // digit planes of x (batch 1)
constexpr int kC2BlockBytes = kC2Digits * 128;     // one 128-column block of x
constexpr int kC2Offset = 1 << 30;                 // digits hold m + 2^30, |m| < 2^29
constexpr int kC2ScaleBits = 29;                   // |m| < 2^29
// 14 consumer warps, the producer warp and the staging warp: 16 warps, four per SM sub-partition
// (a fifth warp on one sub-partition would cap every thread at 96 registers)
constexpr int kC2Consumers = 14;
constexpr int kC2ConsumerThreads = kC2Consumers * 32;
constexpr int kC2ProducerWarp = kC2Consumers;
constexpr int kC2XWarp = kC2Consumers + 1;
constexpr int kC2Threads = (kC2Consumers + 2) * 32;
constexpr int kC2MaxBlocks = 256;                  // blocks per parity buffer (K_pad <= 32768)
constexpr int kDevErrNonFinite = 5;

struct Chain2Layer {
  const uint8_t* units;          // packed units
  const uint8_t* ounits;         // int8 outlier units
  const uint4* cbq;              // [M_pad] integer codebooks; outlier rows {0, 0, e, slot}
  const uint16_t* tile_mask;     // [MT]
  const int32_t* orow;           // [OT*16] row of each outlier slot (-1: padding)
  const int32_t* oexp;           // [OT*16]
  unsigned long long* acc;       // [OT*16] outlier-slot dot products (zero between launches)
  int32_t* ocnt;                 // [OT] contributions received per outlier tile (zero between launches)
  const int32_t* onc;            // [OT] warps contributing to each outlier tile
  const __half* x;               // layer 0: the chain input (fp16)
  const uint8_t* xd;             // layer >= 1: digits of x_j, [KT][512]
  const uint32_t* xcnt;          // layer >= 1: [KT] rows of x_j landed (counts launches)
  const unsigned long long* xS;  // layer >= 1: [KT] sums of a^2 per block; the other launch parity's
                                 // sums follow s_total entries later
  __half* y;                     // fp16 output
  uint8_t* yd;                   // digits of x_{j+1} (the next layer's xd; null for the last layer)
  uint32_t* ycnt;                // the next layer's xcnt
  unsigned long long* yS;        // the next layer's xS
  int64_t ldx, ldy;
  int32_t Up, U, M, K, K_pad, MT, KT, OT, KO;
  int32_t y_rows;                // rows of y that form x_{j+1} (its K); 0 for the last layer
  int32_t KT_next;               // k blocks of x_{j+1}
  int32_t x_vec16;               // layer 0: x 16-byte loadable
  int32_t write_y;               // 0: a later layer overwrites the fp16 output (not written)
  int32_t y_alias_x0;            // the fp16 output overlaps layer 0's input
  float wbound;                  // >= ||row r of W_hat||_2 for every row r
  int32_t pad[3];
};
static_assert(sizeof(Chain2Layer) % 16 == 0, "Chain2Layer is copied in 16-byte pieces");
static_assert(sizeof(Chain2Layer) / 16 + kChainSharePieces <= 32, "one warp copies a descriptor and a share");

struct Chain2Args {
  const Chain2Layer* layers;
  const int4* parts;             // [n_layers][grid][kChainSharePieces] warp shares (as chain_kernel)
  unsigned int* sync;            // [grid] "layer 0 staged" flags
  unsigned int* epoch;           // [0] launches completed (bit 31: poisoned), [1] CTAs finished
  unsigned long long* s_all;     // [2][s_total] every layer's per-block sums (zeroed by parity)
  unsigned long long* trace;     // optional [n_layers][grid][8] globaltimer stamps
  int32_t n_layers, stages, s_total;
  int32_t nb0, nb1;              // blocks of the parity-0 / parity-1 x buffers
  uint32_t negz;
};

struct Chain2Shared {
  Chain2Layer layer[2];                                   // descriptors of layers j (slot j & 1)
  int4 part[2][kChainSharePieces];                        // this CTA's warp shares
  unsigned long long tile_acc[kChainSplitSlots][kTileRows];
  int32_t tile_cnt[kChainSplitSlots];
  unsigned long long s0;                                  // layer-0 staging: sum of a^2
  uint32_t amax0;                                         // layer-0 staging: max |x| (float bits)
  int32_t ex[4];                                          // exponent of x_j in slot j & 3
  int32_t abort;
  uint32_t epoch;
};

// Byte offset of digit plane d of column k (0..127) inside a block.
__host__ __device__ __forceinline__ uint32_t c2_digit_offset(int d, int k) {
  const int p = xs_pos8(k);
  return static_cast<uint32_t>(d * 128 + (((p >> 4) ^ d) << 4) + (p & 15));
}

// Exponent e such that a row of any layer whose input has digit sum S at exponent ex (and whose
// rows have norm <= wbound) satisfies |round(h * 2^e)| < 2^29 for its fp16 outputs h.  The same
// arithmetic on the same inputs in every CTA, so every CTA derives the same exponent.
//   ||x||_2 <= 2^(14 - ex) * sqrt(S)   (|m| + 1/2 <= a * 2^14 for a = (|m| >> 14) + 1)
//   |h| <= wbound * ||x||_2 * (1 + 2^-10), with 2^-8 of margin for the rounding here.
__device__ __forceinline__ int c2_next_exponent(unsigned long long S, float wbound, int ex) {
  const double xn = ldexp(sqrt(static_cast<double>(S)), 14 - ex);
  const double b = static_cast<double>(wbound) * xn * (1.0 + 1.0 / 256.0);
  if (!(b > 0.0) || !(b < 1e300)) return 0;
  int eb = 0;
  (void)frexp(b, &eb);                  // b < 2^eb
  int e = kC2ScaleBits - eb;            // b * 2^e < 2^29
  if (e > 200) e = 200;
  if (e < -200) e = -200;
  return e;
}

// t * 2^-e rounded once to fp16, for any int64 t: values beyond 2^53 are first narrowed to 53
// bits with a sticky bit (round-to-odd), which keeps the single rounding to fp16 correct.
__device__ __forceinline__ __half c2_scale_to_half(long long t, int e) {
  const unsigned long long u = t < 0 ? 0ull - static_cast<unsigned long long>(t) : static_cast<unsigned long long>(t);
  double v;
  if (u < (1ull << 53)) {
    v = static_cast<double>(u);
  } else {
    const int s = 11 - __clzll(static_cast<long long>(u));  // bits above 53
    const unsigned long long lost = u & ((1ull << s) - 1ull);
    const unsigned long long n = (u >> s) | (lost ? 1ull : 0ull);
    v = ldexp(static_cast<double>(n), s);                   // exact: n < 2^53, times a power of two
  }
  v = ldexp(v, -e);
  return __double2half(t < 0 ? -v : v);
}

// The offset digits of row value h at exponent e (|round(h * 2^e)| < 2^29 by the bound) as one
// word m + 2^30 (byte 3 = digit 0, the most significant); a = (|m| >> 14) + 1 for the next bound.
// A non-finite h (only possible past the fp16 range) is clamped and reported.
__device__ __forceinline__ uint32_t c2_row_digits(__half h, int e, uint32_t* a) {
  float f = __half2float(h);
  if (!(fabsf(f) <= 65504.f)) {
    atomicCAS(&g_opc_device_error, 0, kDevErrNonFinite);
    f = f != f ? 0.f : copysignf(65504.f, f);
  }
  long long m = __double2ll_rn(ldexp(static_cast<double>(f), e));
  const long long lim = (1ll << kC2ScaleBits) - 1;
  m = m > lim ? lim : (m < -lim ? -lim : m);
  const unsigned long long am = static_cast<unsigned long long>(m < 0 ? -m : m);
  *a = static_cast<uint32_t>(am >> 14) + 1u;
  return static_cast<uint32_t>(m + kC2Offset);
}

// Store the digits of word w (m + 2^30) of column k into a block at `blk` (global memory).
__device__ __forceinline__ void c2_store_digits(uint8_t* blk, int k, uint32_t w) {
#pragma unroll
  for (int d = 0; d < kC2Digits; ++d) blk[c2_digit_offset(d, k)] = static_cast<uint8_t>(w >> (8 * (3 - d)));
}

// Exact int64 dot products of rows g (t[0]) and g+8 (t[1]) from the accumulators, all lanes of a
// row group holding the sum.  Columns: 0..3 digits (weights 2^24, 2^16, 2^8, 1), 4 ones (-2^30).
__device__ __forceinline__ void c2_finish_dot(const AccQ& A, int q, long long t[2]) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const long long p0 = 256ll * (static_cast<long long>(A.h[0][2 * r]) + A.h[1][2 * r]) +
                         (static_cast<long long>(A.l[0][2 * r]) + A.l[1][2 * r]);
    const long long p1 = 256ll * (static_cast<long long>(A.h[0][2 * r + 1]) + A.h[1][2 * r + 1]) +
                         (static_cast<long long>(A.l[0][2 * r + 1]) + A.l[1][2 * r + 1]);
    long long v;
    if (q == 0) v = (p0 << 24) + (p1 << 16);
    else if (q == 1) v = (p0 << 8) + p1;
    else if (q == 2) v = -(p0 << 30);
    else v = 0;
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    t[r] = v;
  }
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Make generic-proxy data that this thread has acquired visible to its later bulk copies.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bounded wait on an mbarrier phase that also gives up when the CTA aborts.
__device__ __noinline__ bool c2_wait(uint32_t bar, uint32_t parity, const volatile int32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Rows r0, r1 (local; -1 = none) with exponents e0, e1 and dot products t0, t1 of a segment whose
// rows all lie in one 128-row block (a packed tile): fp16 outputs, digits of the next layer's
// input, then the block's sum of a^2 and its row count (released after the digit stores).
__device__ __noinline__ void c2_write_tile(const Chain2Layer& L, int r0, int r1, int e0, int e1, long long t0,
                                           long long t1, int lane, int q, int ex, int ex_next, int64_t s_off) {
  uint32_t a2 = 0, n = 0;
  int blk = -1;
  if (q == 0) {
    const int rows[2] = {r0, r1};
    const long long ts[2] = {t0, t1};
    const int es[2] = {e0, e1};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = rows[i];
      if (r < 0) continue;
      const __half h = c2_scale_to_half(ts[i], es[i] + ex);
      if (L.write_y) L.y[r] = h;
      if (r < L.y_rows) {
        uint32_t a;
        const uint32_t w = c2_row_digits(h, ex_next, &a);
        c2_store_digits(L.yd + static_cast<int64_t>(r >> 7) * kC2BlockBytes, r & 127, w);
        a2 += a * a;  // a <= 2^15 + 1: a^2 < 2^31, two rows per lane fit
        n += 1;
        blk = r >> 7;
      }
    }
  }
  // one block per tile: sum the lanes' contributions and count the rows
  unsigned long long s = a2;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  uint32_t nn = __reduce_add_sync(0xffffffffu, n);
  const int b = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(blk + 1)) - 1;
  __syncwarp();  // every lane's digit stores are ordered before lane 0's release below
  if (lane == 0 && b >= 0 && nn > 0) {
    atomicAdd(L.yS + s_off + b, s);
    red_release_add_u32(L.ycnt + b, nn);
  }
}

// Rows of an outlier tile (any blocks): each lane publishes its own rows.
__device__ __noinline__ void c2_write_rows(const Chain2Layer& L, int r0, int r1, int e0, int e1, long long t0,
                                           long long t1, int q, int ex, int ex_next, int64_t s_off) {
  if (q != 0) return;
  const int rows[2] = {r0, r1};
  const long long ts[2] = {t0, t1};
  const int es[2] = {e0, e1};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = rows[i];
    if (r < 0) continue;
    const __half h = c2_scale_to_half(ts[i], es[i] + ex);
    if (L.write_y) L.y[r] = h;
    if (r < L.y_rows) {
      uint32_t a;
      const uint32_t w = c2_row_digits(h, ex_next, &a);
      c2_store_digits(L.yd + static_cast<int64_t>(r >> 7) * kC2BlockBytes, r & 127, w);
      atomicAdd(L.yS + s_off + (r >> 7), static_cast<unsigned long long>(a) * a);
      red_release_add_u32(L.ycnt + (r >> 7), 1u);
    }
  }
}

__global__ void __launch_bounds__(kC2Threads, 1) chain2_kernel(const Chain2Args args) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int S = args.stages;
  const int nbmax = args.nb0 > args.nb1 ? args.nb0 : args.nb1;

  const uint32_t xs_base[2] = {smem_u32(smem), smem_u32(smem) + static_cast<uint32_t>(args.nb0) * kC2BlockBytes};
  const uint32_t ones_base = xs_base[1] + static_cast<uint32_t>(args.nb1) * kC2BlockBytes;
  const uint32_t zero_base = ones_base + 128;
  const uint32_t ring_base = zero_base + 128;
  const uint32_t full_base = ring_base + kC2Consumers * S * kQChunkBytes;
  const uint32_t empty_base = full_base + kC2Consumers * S * 8;
  const uint32_t xbar_base = empty_base + kC2Consumers * S * 8;      // [2][nbmax]
  const uint32_t xfree_base = xbar_base + 2 * nbmax * 8;            // [2]: consumers done with a layer
  const uint32_t xall_base = xfree_base + 16;                       // [2]: a layer's x staged, next exponent set
  const uint32_t xdesc_base = xall_base + 16;                       // [2]: a layer's descriptor in place
  const uint32_t sh_off = xdesc_base + 16 - xs_base[0];
  Chain2Shared* sh = reinterpret_cast<Chain2Shared*>(smem + ((sh_off + 15u) & ~15u));

  if (threadIdx.x == 0) {
    for (int i = 0; i < kC2Consumers * S; ++i) {
      mbar_init(full_base + i * 8, 1);
      mbar_init(empty_base + i * 8, 1);
    }
    for (int i = 0; i < 2 * nbmax; ++i) mbar_init(xbar_base + i * 8, 1);
    for (int p = 0; p < 2; ++p) {
      mbar_init(xfree_base + p * 8, kC2Consumers);
      mbar_init(xall_base + p * 8, 1);
      mbar_init(xdesc_base + p * 8, 32);
    }
    fence_mbar_init();
    const uint32_t ep = ld_relaxed_u32(args.epoch);
    sh->epoch = ep & ~kChainPoisoned;
    sh->abort = (ep & kChainPoisoned) ? 1 : 0;
    if (ep & kChainPoisoned) atomicCAS(&g_opc_device_error, 0, kDevErrChainPoisoned);
    sh->s0 = 0ull;
    sh->amax0 = 0u;
  }
  for (int i = threadIdx.x; i < kChainSplitSlots * kTileRows; i += blockDim.x) (&sh->tile_acc[0][0])[i] = 0ull;
  for (int i = threadIdx.x; i < kChainSplitSlots; i += blockDim.x) sh->tile_cnt[i] = 0;
  if (threadIdx.x < 16)  // ones block, zero block (B operands of the ones and absent columns)
    sts128(ones_base + threadIdx.x * 16,
           threadIdx.x < 8 ? make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u) : make_uint4(0, 0, 0, 0));
  {
    constexpr int kDesc = static_cast<int>(sizeof(Chain2Layer) / 16);
    const int t = static_cast<int>(threadIdx.x);
    for (int slot = 0; slot < 2 && slot < args.n_layers; ++slot) {
      if (t < kDesc)
        reinterpret_cast<uint4*>(&sh->layer[slot])[t] = ld_nc_v4(reinterpret_cast<const uint4*>(args.layers + slot) + t);
      else if (t < kDesc + kChainSharePieces)
        reinterpret_cast<uint4*>(sh->part[slot])[t - kDesc] = ld_nc_v4(
            reinterpret_cast<const uint4*>(args.parts + kChainSharePieces * (static_cast<int64_t>(slot) * G + cta)) +
            (t - kDesc));
    }
  }
  __syncthreads();
  if (sh->abort) return;  // poisoned: no work, no flags
  const uint32_t epoch = sh->epoch;
  const uint32_t par = epoch & 1u;  // launch parity: which half of the block sums this launch uses
  const int64_t s_off = static_cast<int64_t>(par) * args.s_total;
  // the other half of every layer's block sums starts the next launch at zero
  for (int i = cta + G * static_cast<int>(threadIdx.x); i < args.s_total; i += G * static_cast<int>(blockDim.x))
    args.s_all[static_cast<int64_t>(par ^ 1u) * args.s_total + i] = 0ull;
  const volatile int32_t* abort_flag = &sh->abort;
  auto give_up = [&]() {
    sh->abort = 1;
    atomicCAS(&g_opc_device_error, 0, kDevErrBarrierTimeout);
  };

  // ------------------------------------------------------------------ producer warp
  if (warp == kC2ProducerWarp) {
    const int i = lane;
    const uint32_t ring = ring_base + i * S * kQChunkBytes;
    struct Raw {
      uint64_t units, ounits;
      uint32_t Up, MT, KT, KO, u0, u1, seg0;
    };
    auto fetch = [&](int jn, Raw& r) {
      if (jn >= args.n_layers || i >= kC2Consumers) return;
      const Chain2Layer* Ln = args.layers + jn;
      r.units = ld_nc_u64(&Ln->units);
      r.ounits = ld_nc_u64(&Ln->ounits);
      r.Up = ld_nc_u32(&Ln->Up);
      r.MT = ld_nc_u32(&Ln->MT);
      r.KT = ld_nc_u32(&Ln->KT);
      r.KO = ld_nc_u32(&Ln->KO);
      const int32_t* sr = reinterpret_cast<const int32_t*>(args.parts + kChainSharePieces * (static_cast<int64_t>(jn) * G + cta));
      r.u0 = ld_nc_u32(sr + kShU0 + i);
      r.u1 = ld_nc_u32(sr + kShU1 + i);
      r.seg0 = ld_nc_u32(sr + kShSeg0 + i);
    };
    int j = 0;
    const uint8_t* units = nullptr;
    const uint8_t* ounits = nullptr;
    int32_t Up = 0, MT = 0, KT = 1, KO = 1, u1 = 0;
    int32_t pu = 0, seg = 0, send = 0;
    Raw nx;
    fetch(0, nx);
    auto next_range = [&]() {
      while (j < args.n_layers) {
        units = reinterpret_cast<const uint8_t*>(nx.units);
        ounits = reinterpret_cast<const uint8_t*>(nx.ounits);
        Up = static_cast<int32_t>(nx.Up);
        MT = static_cast<int32_t>(nx.MT);
        KT = static_cast<int32_t>(nx.KT);
        KO = static_cast<int32_t>(nx.KO);
        const int32_t u0 = static_cast<int32_t>(nx.u0);
        u1 = static_cast<int32_t>(nx.u1);
        seg = static_cast<int32_t>(nx.seg0);
        fetch(j + 1, nx);
        if (u0 < u1) {
          pu = u0;
          send = seg < MT ? (seg + 1) * KT : Up + (seg - MT + 1) * KO;
          return true;
        }
        ++j;
      }
      return false;
    };
    bool active = i < kC2Consumers;
    if (active) active = next_range();
    int slot = 0, round = 0;
    uint64_t t_idle = 0;
    bool failed = false;
    while (__any_sync(0xffffffffu, active)) {
      bool issued = false;
      if (active) {
        if (round == 0 || mbar_test(empty_base + (i * S + slot) * 8, static_cast<uint32_t>((round - 1) & 1))) {
          int32_t cnt = send - pu;
          if (u1 - pu < cnt) cnt = u1 - pu;
          if (cnt > kQChunkUnits) cnt = kQChunkUnits;
          const uint32_t bar = full_base + (i * S + slot) * 8;
          mbar_expect_tx(bar, static_cast<uint32_t>(cnt * kUnitBytes));
          const uint8_t* src = pu < Up ? units + static_cast<int64_t>(pu) * kUnitBytes
                                       : ounits + static_cast<int64_t>(pu - Up) * kUnitBytes;
          bulk_g2s(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar);
          pu += cnt;
          if (pu == send && pu < u1) {
            ++seg;
            send += seg < MT ? KT : KO;
          }
          if (++slot == S) {
            slot = 0;
            ++round;
          }
          issued = true;
          if (pu >= u1) {
            ++j;
            active = next_range();
          }
        }
      }
      if (__any_sync(0xffffffffu, issued)) {
        t_idle = 0;
      } else {
        if (*abort_flag) break;
        const uint64_t now = globaltimer_ns();
        if (t_idle == 0) t_idle = now;
        else if (now - t_idle > 2 * kWaitLimitNs) {
          failed = true;
          break;
        }
        nanosleep_ns(64);
      }
    }
    if (failed && lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
    if (i < kC2Consumers) {
      for (int s = 0; s < S; ++s) {
        const int n_in_slot = round + (s < slot ? 1 : 0);
        if (n_in_slot > 0) mbar_wait_bounded(full_base + (i * S + s) * 8, static_cast<uint32_t>((n_in_slot - 1) & 1));
      }
    }
    return;
  }

  // ------------------------------------------------------------------ staging warp
  if (warp == kC2XWarp) {
    // Per block of x_j (j >= 1): wait for its rows (counter, acquire), add its sum of a^2, copy it
    // into shared memory (bulk copy completing on the block's mbarrier).  Lane l takes blocks
    // l, l+32, ...  Blocks past this layer's KT (up to the buffer's) complete their phase with a
    // plain arrival, so every block barrier of a parity completes once per layer of that parity.
    bool ok = true;
    int ex_cur = 0;
    if (args.n_layers > 1) {
      ok = c2_wait(xall_base, 0u, abort_flag);  // layer 0 staged by the consumers: e_1 is set
      if (ok) ex_cur = sh->ex[1];
    }
    bool staged0_seen = false;
    // uses of each parity's block barriers so far (for the phase to wait on before reusing one),
    // and which of this lane's blocks completed or will complete their latest use (copy issued
    // or plain arrival): those are waited for before the CTA exits, even after an abort
    int uses[2] = {0, 0};
    uint32_t posted[2] = {0u, 0u};
    for (int j = 1; j < args.n_layers && ok; ++j) {
      const int p = j & 1;
      const int nbp = p ? args.nb1 : args.nb0;
      unsigned long long* tr = args.trace ? args.trace + (static_cast<int64_t>(j) * G + cta) * kChainTracePhases : nullptr;
      if (j >= 2) {
        // consumers are done with layer j-2 (same buffer and descriptor slot)
        if (!c2_wait(xfree_base + p * 8, static_cast<uint32_t>(((j - 2) >> 1) & 1), abort_flag)) { ok = false; break; }
        constexpr int kDesc = static_cast<int>(sizeof(Chain2Layer) / 16);
        if (lane < kDesc)
          reinterpret_cast<uint4*>(&sh->layer[p])[lane] = ld_nc_v4(reinterpret_cast<const uint4*>(args.layers + j) + lane);
        else if (lane < kDesc + kChainSharePieces)
          reinterpret_cast<uint4*>(sh->part[p])[lane - kDesc] = ld_nc_v4(
              reinterpret_cast<const uint4*>(args.parts + kChainSharePieces * (static_cast<int64_t>(j) * G + cta)) +
              (lane - kDesc));
        mbar_arrive(xdesc_base + p * 8);  // every lane: its piece is in place
      }
      if (tr && lane == 0) tr[0] = globaltimer_ns();
      const Chain2Layer* Lg = args.layers + j;
      const int KT = static_cast<int>(ld_nc_u32(&Lg->KT));
      const int K = static_cast<int>(ld_nc_u32(&Lg->K));
      const uint8_t* xd = reinterpret_cast<const uint8_t*>(ld_nc_u64(&Lg->xd));
      const uint32_t* xcnt = reinterpret_cast<const uint32_t*>(ld_nc_u64(&Lg->xcnt));
      const unsigned long long* xS = reinterpret_cast<const unsigned long long*>(ld_nc_u64(&Lg->xS)) + s_off;
      const int y_alias = static_cast<int>(ld_nc_u32(&Lg->y_alias_x0));
      const float wbound = __uint_as_float(ld_nc_u32(&Lg->wbound));
      const uint32_t ph = static_cast<uint32_t>(uses[p] & 1);
      // make sure this parity's previous copies into the blocks have landed (their phase done)
      if (uses[p] > 0) {
        for (int b = lane; b < nbp; b += 32)
          if (!c2_wait(xbar_base + (p * nbmax + b) * 8, ph ^ 1u, abort_flag)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      }
      // pending blocks of this lane as a bit mask (at most 8 per lane: KT <= 256)
      uint32_t pending = 0;
      posted[p] = 0u;
      for (int i = 0, b = lane; b < nbp; ++i, b += 32) {
        if (b < KT) {
          pending |= 1u << i;
        } else {
          mbar_arrive(xbar_base + (p * nbmax + b) * 8);
          posted[p] |= 1u << i;
        }
      }
      unsigned long long s_lane = 0;
      uint64_t t0 = 0, first_ready = 0, last_ready = 0;  // trace: this lane's first and last arrivals
      while (pending) {
        // poll every pending counter of this lane with relaxed loads (all in flight together);
        // one acquire fence then orders whatever landed before its sums are read and copied
        uint32_t ready = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (!(pending & (1u << i))) continue;
          const int b = lane + 32 * i;
          const uint32_t rows = static_cast<uint32_t>(min(128, K - 128 * b));
          const uint32_t v = ld_relaxed_u32(xcnt + b);
          if (static_cast<int32_t>(v - (epoch + 1u) * rows) >= 0) ready |= 1u << i;
        }
        if (ready) {
          if (tr) {
            const uint64_t now = globaltimer_ns();
            if (first_ready == 0) first_ready = now;
            last_ready = now;
          }
          fence_acq_rel_gpu();
          fence_proxy_async_global();  // the acquired digits are visible to the bulk copies below
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (!(ready & (1u << i))) continue;
            const int b = lane + 32 * i;
            s_lane += ld_relaxed_u64(xS + b);
            const uint32_t bar = xbar_base + (p * nbmax + b) * 8;
            mbar_expect_tx(bar, kC2BlockBytes);
            bulk_g2s(xs_base[p] + b * kC2BlockBytes, xd + static_cast<int64_t>(b) * kC2BlockBytes, kC2BlockBytes, bar);
          }
          pending &= ~ready;
          posted[p] |= ready;
        }
        if (!pending) break;
        if (*abort_flag) { ok = false; break; }
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > kWaitLimitNs) { give_up(); ok = false; break; }
      }
      uses[p] += 1;
      if (tr) {  // the warp's first and last block arrivals
        unsigned long long fr = first_ready ? first_ready : ~0ull, lr = last_ready;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          fr = min(fr, __shfl_xor_sync(0xffffffffu, fr, o));
          lr = max(lr, __shfl_xor_sync(0xffffffffu, lr, o));
        }
        if (lane == 0) {
          tr[4] = fr == ~0ull ? 0ull : fr;
          tr[5] = lr;
        }
      }
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      // the next layer's exponent from the exact sum over every block of x_j
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s_lane += __shfl_xor_sync(0xffffffffu, s_lane, o);
      const int ex_next = c2_next_exponent(s_lane, wbound, ex_cur);
      // a layer writing over the chain input starts once every CTA has read that input
      if (y_alias && !staged0_seen) {
        if (!poll_flags_warp(args.sync, G, lane, 2u * epoch + 1u, false)) {
          if (lane == 0) give_up();
          ok = false;
          break;
        }
        staged0_seen = true;
      }
      if (lane == 0) {
        if (j + 1 < args.n_layers) sh->ex[(j + 1) & 3] = ex_next;
        if (tr) tr[1] = globaltimer_ns();
        mbar_arrive(xall_base + p * 8);
      }
      ex_cur = ex_next;
      (void)K;
    }
    if (!ok && lane == 0) sh->abort = 1;
    // copies issued into the buffers land before the CTA exits (earlier uses completed before
    // their barriers were reused; a copy always completes, so this wait ends)
    for (int p = 0; p < 2; ++p) {
      if (uses[p] == 0) continue;
      for (int i = 0; i < 8; ++i)
        if (posted[p] & (1u << i))
          (void)mbar_wait_bounded(xbar_base + (p * nbmax + lane + 32 * i) * 8, static_cast<uint32_t>((uses[p] - 1) & 1));
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  const int g = lane >> 2, q = lane & 3;
  const int tid = threadIdx.x;
  const uint32_t negz = args.negz;
  const uint32_t ring = ring_base + warp * S * kQChunkBytes + lane * 16;
  const uint32_t fullw = full_base + warp * S * 8, emptyw = empty_base + warp * S * 8;
  int slot = 0;
  uint32_t phase = 0;
  bool ok = true;

  // ---- layer 0: the caller's fp16 x into digits (parity-0 buffer), exponent from max |x|
  {
    const Chain2Layer& L = sh->layer[0];
    const int n_chunks = L.K_pad / 8;
    float mx = 0.f;
    for (int c = tid; c < n_chunks; c += kC2ConsumerThreads) {
      const int k = c * 8;
      const uint4 v = k < L.K ? chain_load_x0(L.x, L.ldx, 0, k, L.K, L.x_vec16) : make_uint4(0, 0, 0, 0);
      mx = fmaxf(mx, chain_chunk_amax(v));
    }
    const uint32_t m = __reduce_max_sync(0xffffffffu, mx == mx ? __float_as_uint(mx) : 0u);
    if (lane == 0) atomicMax(&sh->amax0, m);
    named_barrier(1, kC2ConsumerThreads);
    const float m0 = __uint_as_float(sh->amax0);
    const int e0 = m0 > 0.f ? kC2ScaleBits - 1 - frexp_exponent(m0) : 0;  // max |x| * 2^e0 < 2^28
    unsigned long long s = 0;
    for (int c = tid; c < n_chunks; c += kC2ConsumerThreads) {
      const int k = c * 8;
      const uint4 v = k < L.K ? chain_load_x0(L.x, L.ldx, 0, k, L.K, L.x_vec16) : make_uint4(0, 0, 0, 0);
      const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
      uint32_t w[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hv[e]));
        const int ma = __float2int_rn(ldexpf(f.x, e0)), mb = __float2int_rn(ldexpf(f.y, e0));
        const uint32_t aa = (static_cast<uint32_t>(ma < 0 ? -ma : ma) >> 14) + 1u;
        const uint32_t ab = (static_cast<uint32_t>(mb < 0 ? -mb : mb) >> 14) + 1u;
        s += static_cast<unsigned long long>(aa) * aa + static_cast<unsigned long long>(ab) * ab;
        w[2 * e] = static_cast<uint32_t>(ma + kC2Offset);
        w[2 * e + 1] = static_cast<uint32_t>(mb + kC2Offset);
      }
      // 8 consecutive columns share one 16-byte chunk per plane: one 8-byte store per plane
      const uint32_t blk = xs_base[0] + static_cast<uint32_t>(k >> 7) * kC2BlockBytes;
#pragma unroll
      for (int d = 0; d < kC2Digits; ++d) {
        const uint32_t bs = 3 - d;  // byte of the word holding digit d
        const uint32_t sel = bs | ((bs + 4) << 4);
        const uint32_t lo = prmt(prmt(w[0], w[1], sel), prmt(w[2], w[3], sel), 0x5410u);
        const uint32_t hi = prmt(prmt(w[4], w[5], sel), prmt(w[6], w[7], sel), 0x5410u);
        sts64(blk + c2_digit_offset(d, k & 127), lo, hi);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) atomicAdd(&sh->s0, s);
    fence_proxy_async_shared();  // these generic writes precede later bulk copies into the buffer
    named_barrier(1, kC2ConsumerThreads);
    if (tid == 0) {
      sh->ex[0] = e0;
      sh->ex[1] = c2_next_exponent(sh->s0, L.wbound, e0);
      fence_acq_rel_gpu();
      st_relaxed_u32(args.sync + cta, 2u * epoch + 1u);  // layer-0 input read by this CTA
      mbar_arrive(xall_base);
    }
  }

  for (int j = 0; j < args.n_layers && ok; ++j) {
    const int p = j & 1;
    unsigned long long* tr = args.trace ? args.trace + (static_cast<int64_t>(j) * G + cta) * kChainTracePhases : nullptr;
    if (j >= 2 && !c2_wait(xdesc_base + p * 8, static_cast<uint32_t>(((j >> 1) - 1) & 1), abort_flag)) {
      ok = false;
      break;
    }
    const Chain2Layer& L = sh->layer[p];
    const int32_t* sr = reinterpret_cast<const int32_t*>(sh->part[p]);
    const int32_t u0 = sr[kShU0 + warp], u1 = sr[kShU1 + warp];
    GemvQArgs qa;
    qa.cbq = L.cbq; qa.tile_mask = L.tile_mask; qa.orow = L.orow; qa.oexp = L.oexp; qa.M = L.M; qa.MT = L.MT;
    ChainCursor cc;
    cc.u = u0;
    cc.seg = sr[kShSeg0 + warp];
    cc.begin = cc.seg < L.MT ? cc.seg * L.KT : L.Up + (cc.seg - L.MT) * L.KO;
    cc.end = cc.begin + (cc.seg < L.MT ? L.KT : L.KO);
    MetaQ cur, nxt;
    if (u0 < u1) {
      cur = chain_load_meta(qa, cc.seg, g);
      nxt = chain_load_meta(qa, min(cc.seg + 1, L.MT + L.OT - 1), g);
    }
    if (tr && tid == 0) tr[2] = globaltimer_ns();
    bool first_wait = false;  // trace: warp 0's first chunk of this layer had its x blocks
    const uint32_t xsb = xs_base[p];
    const uint32_t xph = static_cast<uint32_t>(((j >> 1) - ((j & 1) ^ 1)) & 1);  // block barrier phase (j >= 1)
    const uint32_t xbar_p = xbar_base + p * nbmax * 8;
    // B-operand column of this lane: digit plane g (0..3), the ones block (4) or zeros (5..7)
    const bool digit_col = g < kC2Digits;
    const uint32_t col_base = digit_col ? xsb + g * 128 : (g == kC2Digits ? ones_base : zero_base);
    const uint32_t blk_stride = digit_col ? static_cast<uint32_t>(kC2BlockBytes) : 0u;
    const uint32_t c_lo = static_cast<uint32_t>(((2 * q) ^ g) << 4), c_hi = static_cast<uint32_t>(((2 * q + 1) ^ g) << 4);
    int ex = 0, ex_next = 0;
    bool ex_known = false;
    auto need_ex = [&]() -> bool {
      if (ex_known) return true;
      if (!c2_wait(xall_base + p * 8, static_cast<uint32_t>((j >> 1) & 1), abort_flag)) return false;
      ex = sh->ex[j & 3];
      ex_next = sh->ex[(j + 1) & 3];
      ex_known = true;
      return true;
    };

    if (u0 < u1) {
      AccQ A;
      zero_accq(A);
      while (cc.u < u1) {
        if (!c2_wait(fullw + slot * 8, phase, abort_flag)) {
          ok = false;
          break;
        }
        const int32_t cnt = chain_chunk(cc, u1);
        const uint32_t stage = ring + slot * kQChunkBytes;
        const int32_t k0 = cc.u - cc.begin;
        if (cc.seg < L.MT) {
          if (j > 0) {  // the chunk's x blocks k0 .. k0+cnt-1 are in shared memory
            // one inline test per block; the bounded wait only for a block still in flight
            uint32_t missing = 0;
#pragma unroll
            for (int i = 0; i < kQChunkUnits; ++i)
              if (i < cnt && !mbar_test(xbar_p + (k0 + i) * 8, xph)) missing |= 1u << i;
            if (missing) {
              if (tr && tid == 0 && !first_wait) tr[6] = globaltimer_ns();
              bool in = true;
              for (int i = 0; i < cnt && in; ++i)
                if (missing & (1u << i)) in = c2_wait(xbar_p + (k0 + i) * 8, xph, abort_flag);
              if (!in) { ok = false; break; }
            }
            if (tr && tid == 0 && !first_wait) {
              tr[7] = globaltimer_ns();
              first_wait = true;
            }
          }
#pragma unroll 1
          for (int i = 0; i < cnt; ++i) {
            const uint4 wv = lds128(stage + i * kUnitBytes);
            const uint32_t xa = col_base + static_cast<uint32_t>(k0 + i) * blk_stride;
            const uint4 b01 = lds128(xa + c_lo), b23 = lds128(xa + c_hi);
            const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
            const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
              uint32_t Ah[4], Al[4];
              decode_word_q(w[jw], cur.qh, cur.ql, negz, Ah, Al);
              imma16832(A.h[jw & 1], Ah, bb[2 * jw], bb[2 * jw + 1]);
              imma16832(A.l[jw & 1], Al, bb[2 * jw], bb[2 * jw + 1]);
            }
          }
        } else {
          if (j > 0) {
            bool in = c2_wait(xbar_p + (k0 >> 3) * 8, xph, abort_flag);
            if (in && ((k0 + cnt - 1) >> 3) != (k0 >> 3)) in = c2_wait(xbar_p + ((k0 + cnt - 1) >> 3) * 8, xph, abort_flag);
            if (!in) { ok = false; break; }
          }
#pragma unroll
          for (int i = 0; i < kQChunkUnits; ++i) {
            if (i < cnt) {
              const uint4 av = lds128(stage + i * kUnitBytes);
              const int32_t s = k0 + i;
              const uint32_t bv = lds32(col_base + static_cast<uint32_t>(s >> 3) * blk_stride +
                                        ((static_cast<uint32_t>((s & 7) ^ g)) << 4) + 4 * q);
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
        if (cc.u == cc.end || cc.u == u1) {  // a segment of the range is complete
          long long t[2];
          c2_finish_dot(A, q, t);
          int r0 = cur.row[0], r1 = cur.row[1];
          const int seg = cc.seg;
          const bool whole = cc.begin >= u0 && cc.end <= u1;
          if (seg < L.MT) {  // packed tile: base row and raw mask -> output rows (-1: masked or past M)
            const uint32_t mask = static_cast<uint32_t>(r1);
            r1 = (r0 + 8 < L.M && !((mask >> (g + 8)) & 1u)) ? r0 + 8 : -1;
            r0 = (r0 < L.M && !((mask >> g) & 1u)) ? r0 : -1;
          }
          if (seg >= L.MT) {
            // outlier tile: exact int64 adds into the slot accumulators, completed by the last
            // contributing warp (acq_rel count), which publishes the tile's rows
            const int tt = seg - L.MT;
            const int s0 = tt * kTileRows + g, s1 = s0 + 8;
            const int need = static_cast<int>(ld_nc_u32(L.onc + tt));
            if (q == 0) {
              if (r0 >= 0) atomicAdd(L.acc + s0, static_cast<unsigned long long>(t[0]));
              if (r1 >= 0) atomicAdd(L.acc + s1, static_cast<unsigned long long>(t[1]));
            }
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atom_add_acq_rel_gpu(L.ocnt + tt, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            __syncwarp();
            if (old == need - 1) {
              long long f0 = 0, f1 = 0;
              if (q == 0) {
                if (r0 >= 0) f0 = static_cast<long long>(atomicExch(L.acc + s0, 0ull));
                if (r1 >= 0) f1 = static_cast<long long>(atomicExch(L.acc + s1, 0ull));
              }
              if (lane == 0) st_relaxed_u32(reinterpret_cast<unsigned int*>(L.ocnt + tt), 0u);
              if (!need_ex()) { ok = false; break; }
              c2_write_rows(L, r0, r1, cur.e[0], cur.e[1], f0, f1, q, ex, ex_next, s_off);
            }
          } else if (whole) {
            if (!need_ex()) { ok = false; break; }
            c2_write_tile(L, r0, r1, cur.e[0], cur.e[1], t[0], t[1], lane, q, ex, ex_next, s_off);
          } else {
            // packed tile shared with other warps of this CTA: exact adds in shared memory, the
            // warp completing the count of contributors writes the tile
            const int32_t tb = seg * L.KT, te = tb + L.KT;
            const int wp = sr[kShWp];
            int n_contrib = 0;
            for (int w = 0; w < wp; ++w) {
              const int32_t a = sr[kShU0 + w], b = sr[kShU1 + w];
              n_contrib += (a < b && a < te && b > tb) ? 1 : 0;
            }
            const int sl = (seg - sr[kShTile0]) & (kChainSplitSlots - 1);
            if (q == 0) {
              atomicAdd(&sh->tile_acc[sl][g], static_cast<unsigned long long>(t[0]));
              atomicAdd(&sh->tile_acc[sl][g + 8], static_cast<unsigned long long>(t[1]));
            }
            __threadfence_block();
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atomicAdd(&sh->tile_cnt[sl], 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == n_contrib - 1) {
              __threadfence_block();
              long long f0 = 0, f1 = 0;
              if (q == 0) {
                f0 = static_cast<long long>(atomicExch(&sh->tile_acc[sl][g], 0ull));
                f1 = static_cast<long long>(atomicExch(&sh->tile_acc[sl][g + 8], 0ull));
              }
              if (lane == 0) sh->tile_cnt[sl] = 0;
              if (!need_ex()) { ok = false; break; }
              c2_write_tile(L, r0, r1, cur.e[0], cur.e[1], f0, f1, lane, q, ex, ex_next, s_off);
            }
          }
          if (cc.u == u1) break;
          zero_accq(A);
          cc.seg += 1;
          cc.begin = cc.end;
          cc.end = cc.begin + (cc.seg < L.MT ? L.KT : L.KO);
          cur = nxt;
          if (cc.seg + 1 < L.MT + L.OT) nxt = chain_load_meta(qa, cc.seg + 1, g);
        }
      }
    }
    if (tr && tid == 0) tr[3] = globaltimer_ns();
    if (!ok) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(xfree_base + p * 8);  // this warp is done with layer j
  }
  if (!ok) {
    sh->abort = 1;
    atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
  }

  // ---- end of the launch: the last CTA to finish advances the epoch
  named_barrier(1, kC2ConsumerThreads);
  if (tid == 0) {
    if (sh->abort) atomicOr(args.epoch, kChainPoisoned);
    __threadfence();
    const unsigned int done = atomicAdd(args.epoch + 1, 1u);
    if (done == static_cast<unsigned int>(G) - 1u) {
      st_relaxed_u32(args.epoch + 1, 0u);
      atomicAdd(args.epoch, 1u);
    }
  }
}

}  // namespace opc
