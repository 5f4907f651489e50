// opc_chain.cuh -- persistent decode-chain kernel: a whole sequence of dependent fused 2-bit
// GEMVs (one decode token through every projection of every block) in one cooperative launch,
// on one GPU or row-sharded over several GPUs of a node.
//
// Each layer is the integer-split GEMV of opc_gemvq.cuh (8 PRMT + 3 ALU operations and two int8
// mma.sync per 16 weights, exact int64 dot products).  What changes is the orchestration:
//
//  * One CTA per SM stays resident for the whole chain.  A producer warp streams every layer's
//    units for the CTA's 15 consumer warps through their rings and runs ahead across layer
//    boundaries (weights do not depend on activations), so HBM keeps streaming while the
//    consumers wait for a layer's input.
//  * Dataflow instead of grid barriers: every output element of layer j is published as one
//    32-bit exchange word (fp16 value | 16-bit tag) with a single store; the tag names the launch
//    and the layer.  A CTA staging layer j+1 polls the words of its x chunks until every tag is
//    the expected one, so it starts as soon as the last row it needs has landed -- no fence, no
//    flag, no grid barrier between layers.  The fp16 value also goes to the plain output buffer
//    y (what callers read) unless a later layer of the chain overwrites that buffer.
//  * Packed row tiles are handed out whole (CTA c gets tiles round(c*MT/G) .. round((c+1)*MT/G)),
//    so a tile is split only between warps of one CTA and reduced in shared memory.  Outlier
//    tiles (16 fp16 rows, 8x heavier per row) are split evenly across all CTAs.  Partial dot
//    products of a shared tile are added exactly into int64 accumulators that also count the
//    contributions (2^52 per contributor above the sum), one returning atomic per row: the
//    contributor whose addition completes the count holds the exact total and publishes the row.
//  * Within a CTA, packed warps split its units in proportion to their speed (the warps of an SM
//    sub-partition share its issue slots; host-computed).
//
// Row sharding over `world` GPUs (one process per GPU): every rank holds a contiguous shard of
// each layer's output rows and computes it from the full x.  There is no all-gather: a rank
// stores each finished row (fp16 and exchange word) straight into every rank's buffers over
// NVLink, through peer pointers mapped by CUDA IPC, with system-scope stores; readers poll their
// own local copy.  Peer memory is touched only by plain stores and the flag stores below; nothing
// in this kernel uses TMA or bulk copies with cluster multicast.
//
// Per launch, two flag values per CTA: "layer 0 staged" (a layer whose fp16 output overlaps the
// chain input waits for it from every CTA before running) and, with several ranks, "finished"
// (a last barrier: no rank starts its next launch while a peer still reads or writes this one's
// buffers).  Flags and tags count launches (the epoch word), so nothing is cleared between
// launches; the last CTA to finish advances the epoch.  A launch that gives up on a bounded wait
// poisons the epoch word and every later launch of the chain refuses to run.
#pragma once

#include "opc_gemvq.cuh"

namespace opc {

constexpr int kMaxRanks = 8;

struct ChainLayer {
  const uint8_t* units;          // packed units (this rank's rows)
  const uint8_t* ounits;         // int8 outlier units
  const uint4* cbq;              // [M_pad] integer codebooks; outlier rows {0, 0, e, slot}
  const uint16_t* tile_mask;     // [MT]
  const int32_t* orow;           // [OT*16] local row of each outlier slot (-1: padding)
  const int32_t* oexp;           // [OT*16]
  const __half* x;               // layer 0: the chain input (fp16)
  const uint32_t* xw;            // layer >= 1: the previous layer's exchange words (this rank's copy)
  unsigned long long* acc;       // [OT*16][2] outlier-slot dot products, count-carrying (zero between launches)
  const uint4* cbv;              // sub_vector_size 8: [M_pad][4] integer vectors {hi[8], lo[8]}
  const int32_t* onc;            // [OT] warps contributing to each outlier tile
  __half* y_peer[kMaxRanks];     // this rank's first row in rank p's fp16 copy of the full output
  uint32_t* yw_peer[kMaxRanks];  // this rank's first row in rank p's exchange words of it
  int64_t ldx, ldy, ldxw, ldyw;  // row strides (elements); ldxw, ldyw multiples of 8
  int32_t Up, U, M, K, K_pad, MT, KT, OT, KO;
  int32_t x_vec16;               // layer 0: x rows 16-byte loadable
  int32_t row_off, m_full;       // this rank's first row; rows of the full output
  int32_t write_y;               // 0: a later layer overwrites the fp16 output (not written)
  int32_t y_alias_x0;            // the fp16 output overlaps layer 0's input
  // sub_vector_size 8 (opc_layer.cuh, vq8_chain_vectors_kernel): units are 512-byte groups of four
  // 128-byte index units (16 rows x 1024 columns), decoded through the vector codebooks cbv;
  // cb_stride = the 128-column blocks of the staged x (KT counts 1024-column units then)
  int32_t vq8, cb_stride, pad_[2];
};

// Per layer and CTA, the host-computed shares of its consumer warps, so the kernel does no integer
// division: int32 [0..14] first unit of warp w, [15] packed warps wp, [16..30] end unit of warp w,
// [31] the CTA's first packed tile, [32..46] first segment of warp w (0 for an empty range).
constexpr int kChainShareInts = 48;
constexpr int kChainSharePieces = kChainShareInts / 4;  // int4 pieces
constexpr int kShU0 = 0, kShWp = 15, kShU1 = 16, kShTile0 = 31, kShSeg0 = 32;

static_assert(sizeof(ChainLayer) % 16 == 0, "ChainLayer is copied in 16-byte pieces");
static_assert(sizeof(ChainLayer) / 16 + kChainSharePieces <= 32, "one warp copies a descriptor and a CTA share");
static_assert(kQConsumers == 15, "share table layout");

struct ChainArgs {
  const ChainLayer* layers;
  const int4* parts;         // [n_layers][grid][kChainSharePieces] each CTA's warp shares
  unsigned int* sync;        // [world][grid] flags of every rank's CTAs, in this rank's memory
  unsigned int* sync_peer[kMaxRanks];  // rank p's flag array (sync_peer[rank] == sync)
  unsigned int* epoch;       // [0] launches completed (bit 31: poisoned), [1] CTAs finished
  unsigned long long* trace; // optional [n_layers][grid][24] globaltimer stamps (ns) per CTA:
                             // [0..7] by its first consumer thread: layer start, setup done,
                             // first x poll done, x complete, max barrier passed, digits
                             // stored, x staged, own units done; [8 + w] consumer warp w's
                             // units (and row writes) done
  int32_t n_layers, batch, stages, xs_bytes;
  uint32_t negz;
  int32_t l2_prefetch;       // stream weights with an L2 evict-first policy
  int32_t rank, world;
};
constexpr int kChainTracePhases = 24;  // 8 phase stamps, then one per consumer warp (units done)
constexpr uint32_t kChainPoisoned = 0x80000000u;
constexpr uint32_t kChainTagPeriod = 65535u;  // tags run 1..65535
constexpr int32_t kChainMaxLayers = 65534;    // so consecutive launches never share a layer's tag

// Tag of layer j's exchange words in the launch with epoch e: ((e * n_layers + j) mod 65535) + 1,
// never 0 (the value of a cleared word).  A word of layer j is rewritten once per launch, so it
// holds this launch's tag or the previous launch's, which differs by n_layers (mod 65535).
__host__ __device__ __forceinline__ uint32_t chain_tag_base(uint32_t epoch, int32_t n_layers) {
  return static_cast<uint32_t>((static_cast<uint64_t>(epoch) * static_cast<uint64_t>(n_layers)) % kChainTagPeriod);
}
__host__ __device__ __forceinline__ uint32_t chain_tag(uint32_t base, int32_t j) {
  uint32_t t = base + static_cast<uint32_t>(j);
  if (t >= kChainTagPeriod) t -= kChainTagPeriod;
  return t + 1u;
}

// This CTA's share of a layer: packed units [pu0, pu1) (whole tiles) and outlier units
// [ou0, ou1); warps 0..wp-1 take the packed share, the other consumer warps the outlier share.
struct ChainPart {
  int32_t pu0, pu1, ou0, ou1, wp;
};
__host__ __device__ __forceinline__ ChainPart chain_part(const ChainLayer& L, int c, int G, int nw = kQConsumers) {
  ChainPart p;
  const int32_t t0 = static_cast<int32_t>((2ll * c * L.MT + G) / (2ll * G));
  const int32_t t1 = static_cast<int32_t>((2ll * (c + 1) * L.MT + G) / (2ll * G));
  const int32_t Uo = L.U - L.Up;
  p.pu0 = t0 * L.KT;
  p.pu1 = t1 * L.KT;
  p.ou0 = L.Up + static_cast<int32_t>(static_cast<int64_t>(c) * Uo / G);
  p.ou1 = L.Up + static_cast<int32_t>(static_cast<int64_t>(c + 1) * Uo / G);
  const int32_t np = p.pu1 - p.pu0, no = p.ou1 - p.ou0;
  if (no == 0) {
    p.wp = nw;
  } else if (np == 0) {
    p.wp = 0;
  } else {
    int wo = static_cast<int>((2ll * nw * no + (np + no)) / (2ll * (np + no)));
    wo = wo < 1 ? 1 : (wo > nw - 1 ? nw - 1 : wo);
    p.wp = nw - wo;
  }
  // Every packed warp gets at least one unit, so the warps sharing a tile are exactly the parts
  // between the parts of its first and last unit (the split-tile contributor count relies on it).
  if (p.wp > np) p.wp = np;
  return p;
}
// Warp w's unit range within its CTA's share, for nw consumer warps (32-bit arithmetic: a CTA's
// share times the warps stays below 2^31, host-checked).
__host__ __device__ __forceinline__ void chain_warp_range(const ChainPart& p, int w, int32_t* u0, int32_t* u1,
                                                         int nw = kQConsumers) {
  if (w < p.wp) {
    const int32_t np = p.pu1 - p.pu0;
    *u0 = p.pu0 + w * np / p.wp;
    *u1 = p.pu0 + (w + 1) * np / p.wp;
  } else {
    const int32_t no = p.ou1 - p.ou0, nwo = nw - p.wp;
    *u0 = p.ou0 + (w - p.wp) * no / nwo;
    *u1 = p.ou0 + (w - p.wp + 1) * no / nwo;
  }
}

// A segment's metadata for lane group g, loaded without using any loaded value: for a packed tile
// row[0] is the base row and row[1] the raw tile mask (the output rows are resolved when the tile
// is finished, so no instruction waits on these loads until then); for an outlier tile the rows
// and exponents of its slots.
__device__ __forceinline__ MetaQ chain_load_meta(const GemvQArgs& a, int32_t seg, int g) {
  MetaQ m;
  if (seg < a.MT) {
    const int r0 = seg * kTileRows + g;
    const uint4 c0 = ld_nc_v4(a.cbq + r0), c1 = ld_nc_v4(a.cbq + r0 + 8);
    m.qh[0] = c0.x; m.ql[0] = c0.y; m.e[0] = static_cast<int32_t>(c0.z);
    m.qh[1] = c1.x; m.ql[1] = c1.y; m.e[1] = static_cast<int32_t>(c1.z);
    m.row[0] = r0;
    m.row[1] = static_cast<int32_t>(ld_nc_u16(a.tile_mask + seg));
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

// Unit cursor over a layer (segments: packed tiles of KT units, outlier tiles of KO units).
struct ChainCursor {
  int32_t u, seg, begin, end;
};
__device__ __forceinline__ ChainCursor chain_cursor_at(const ChainLayer& L, int32_t u, int32_t seg) {
  ChainCursor c;
  c.u = u;
  c.seg = seg;
  c.begin = seg < L.MT ? seg * L.KT : L.Up + (seg - L.MT) * L.KO;
  c.end = c.begin + (seg < L.MT ? L.KT : L.KO);
  return c;
}
__device__ __forceinline__ int32_t chain_chunk(const ChainCursor& c, int32_t u1) {
  int32_t n = c.end - c.u;
  if (u1 - c.u < n) n = u1 - c.u;
  return n < kQChunkUnits ? n : kQChunkUnits;
}
__device__ __forceinline__ void chain_next_segment(const ChainLayer& L, ChainCursor& c) {
  c.seg += 1;
  c.begin = c.end;
  c.end = c.begin + (c.seg < L.MT ? L.KT : L.KO);
}

// Memory-model helpers.  One GPU: GPU scope.  Several GPUs: system scope for everything peers
// read or write (exchange words, fp16 rows, flags).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_scope(bool sys) {
  if (sys) fence_acq_rel_sys();
  else fence_acq_rel_gpu();
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Four consecutive words, each a single-copy-atomic relaxed load.
__device__ __forceinline__ uint4 ld_relaxed_v4(const uint32_t* p, bool sys) {
  uint4 v;
  if (sys)
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned int* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u32(unsigned int* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One warp polls n flags (lane l: flags l, l+32, ...; independent relaxed loads, all in flight
// together) until every one has reached target (modulo 2^32), bounded by kWaitLimitNs; then an
// acquire fence orders the caller's later accesses.
__device__ __noinline__ bool poll_flags_warp(const unsigned int* flags, int n, int lane, uint32_t target, bool sys) {
  uint64_t t0 = 0;
  for (;;) {
    bool reached = true;
#pragma unroll 4
    for (int t = lane; t < n; t += 32) {
      const uint32_t v = sys ? ld_relaxed_sys_u32(flags + t) : ld_relaxed_u32(flags + t);
      reached &= static_cast<int32_t>(v - target) >= 0;
    }
    if (__all_sync(0xffffffffu, reached)) {
      fence_scope(sys);
      return true;
    }
    const uint64_t now = globaltimer_ns();
    if (t0 == 0) t0 = now;
    else if (now - t0 > kWaitLimitNs) return false;
  }
}

// Exact 2^e for e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// Code size matters here: the kernel's once-per-layer paths (staging, tails, the producer) run
// while the weight stream saturates the memory system, and their code is fetched again for every
// layer (running the x-conversion pass twice in a row measured 2.0 us for the first pass and
// 0.54 us for the second), so they are kept small.  What measured smaller and faster: helpers
// with one call site inlined (digit stores, segment finishing), the polling and the row writes
// (several call sites) out of line, and loops over chunks calling them rather than unrolled
// copies of their bodies.

// Eight exchange words of k..k+7 (the first n_valid inside the row): do all carry `tag`?  Then
// their fp16 values, packed in pairs, go to v.
__device__ __forceinline__ bool chain_take_words(const uint4& a, const uint4& c, uint32_t tag, int n_valid, uint4* v) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
  bool ok = true;
#pragma unroll
  for (int e = 0; e < 8; ++e) ok &= (e >= n_valid) || ((w[e] >> 16) == tag);
  if (!ok) return false;
  uint32_t h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) h[e] = e < n_valid ? (w[e] & 0xffffu) : 0u;
  *v = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
  return true;
}

// One poll of x chunk (batch row b, columns k..k+7) of a layer >= 1: ok when every word carries
// `tag`, with the fp16 values in v (returned by value: no address, so no local memory).
struct ChainChunk {
  uint4 v;
  int ok;
};
template <bool sys>
__device__ __noinline__ ChainChunk chain_poll_chunk(const uint32_t* xw, int64_t ldxw, int b, int k, int K,
                                                    uint32_t tag) {
  const uint32_t* src = xw + b * ldxw + k;
  const uint4 a = ld_relaxed_v4(src, sys), d = ld_relaxed_v4(src + 4, sys);
  ChainChunk r;
  r.v = make_uint4(0, 0, 0, 0);
  r.ok = chain_take_words(a, d, tag, K - k, &r.v) ? 1 : 0;
  return r;
}

// Layer 0: x chunk (columns k..k+7 of row b) from the fp16 input.
__device__ __noinline__ uint4 chain_load_x0(const __half* x, int64_t ldx, int b, int k, int K, int vec16) {
  const __half* src = x + b * ldx + k;
  if (vec16) return ld_cg_v4(src);
  uint16_t h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) h[e] = (k + e < K) ? __ldcg(reinterpret_cast<const unsigned short*>(src) + e) : 0;
  return make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16), h[4] | (uint32_t(h[5]) << 16),
                    h[6] | (uint32_t(h[7]) << 16));
}

// max |x| over a chunk's eight fp16 values
__device__ __forceinline__ float chain_chunk_amax(const uint4& v) {
  // |x| by clearing the sign bits, maxima of half2 pairs (exact, NaN ignored like fmaxf), one
  // conversion at the end
  const uint32_t w[4] = {v.x & 0x7fff7fffu, v.y & 0x7fff7fffu, v.z & 0x7fff7fffu, v.w & 0x7fff7fffu};
  const __half2* h = reinterpret_cast<const __half2*>(w);
  const __half2 m = __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3]));
  return fmaxf(__low2float(m), __high2float(m));
}

// A chunk's eight values as offset integers x*2^ex + 2^22 (x_digits_q), stored at their staged
// positions in the three unsigned digit columns of batch row b.
__device__ __forceinline__ void chain_store_digits(const uint4 v, float sc, uint32_t col0, uint32_t colb, uint32_t pos) {
  const XDigitsQ d = x_digits_q(v, sc);
#pragma unroll
  for (int dd = 0; dd < 3; ++dd) sts64(col0 + dd * colb + pos, d.d[dd][0], d.d[dd][1]);
}

// sub_vector_size 8: per consumer warp two 1 KB slices of shared memory (current and next row
// tile's vector codebooks, 16 rows x 64 bytes), filled with cp.async.
constexpr int kChainVq8SliceBytes = kQConsumers * 2048 + 16;
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// Row tile seg's vector codebooks (1 KB) into slice dst: 32 bytes per lane.
__device__ __forceinline__ void chain_vq8_slice(uint32_t dst, const uint4* cbv, int32_t seg, int lane) {
  const uint4* src = cbv + static_cast<int64_t>(seg) * kTileRows * 4 + 2 * lane;
  cp_async16(dst + 32 * lane, src);
  cp_async16(dst + 32 * lane + 16, src + 1);
  cp_async_commit();
}

constexpr int kChainSplitSlots = 32;  // packed tiles per CTA and layer (host-checked)

struct ChainShared {
  ChainLayer layer[2];                    // descriptors of layers j (slot j&1) and j+1
  int4 part[2][kChainSharePieces];        // this CTA's warp shares of layers j and j+1
  uint32_t amax_bits[2][kQMaxBatch];      // staging: max |x| (float bits) of layers with parity 0 / 1
  unsigned long long tile_acc[kChainSplitSlots][kTileRows][kQMaxBatch];  // split packed tiles (count-carrying)
  int32_t abort;
  uint32_t epoch;
};

// Rows r0, r1 (local; -1 = none) with exponents e0, e1 and dot products t0, t1: exchange words
// into every rank's copy (one relaxed store per word) and, unless a later layer overwrites it,
// the fp16 output.  Scalars only, so nothing of the caller goes through local memory.
template <bool sys>
__device__ __noinline__ void chain_write_rows(const ChainLayer& L, int P, int B, int r0, int r1, int e0, int e1,
                                              long long t0, long long t1, int q, int ex0, int ex1, uint32_t tag) {
  const int b = q >> 1;
  if ((q & 1) || b >= B) return;
  const int ex = b ? ex1 : ex0;
  const __half h0 = scale_to_half(t0, e0 + ex), h1 = scale_to_half(t1, e1 + ex);
  const uint32_t w0 = (tag << 16) | __half_as_ushort(h0), w1 = (tag << 16) | __half_as_ushort(h1);
  for (int p = 0; p < (sys ? P : 1); ++p) {
    unsigned int* wb = L.yw_peer[p] + b * L.ldyw;
    if (L.write_y) {
      __half* yb = L.y_peer[p] + b * L.ldy;
      if (r0 >= 0) yb[r0] = h0;
      if (r1 >= 0) yb[r1] = h1;
    }
    if (sys) {
      if (r0 >= 0) st_relaxed_sys_u32(wb + r0, w0);
      if (r1 >= 0) st_relaxed_sys_u32(wb + r1, w1);
    } else {
      if (r0 >= 0) st_relaxed_u32(wb + r0, w0);
      if (r1 >= 0) st_relaxed_u32(wb + r1, w1);
    }
  }
}

// Reductions of partial dot products carry their own completion count: every contributor adds
// 2^52 + t with ONE returning atomic per row, t its exact partial dot product.  Every partial sum of
// a row is below 2^51 in magnitude (|centroid integer| <= 2^14, |x integer| < 2^22, K <= 2^15,
// host-checked), so the top 12 bits count the contributions (up to 4095, host-checked) and the old
// value tells a contributor how many came before it and -- for the one that completes the count --
// the exact total.  No fence, no separate counter, no second round trip; the completing lane resets
// the word to zero for the next launch and publishes the row.
constexpr int kCountShift = 52;
constexpr unsigned long long kCountOne = 1ull << kCountShift;
constexpr int kMaxContributors = 4095;
__device__ __forceinline__ bool count_add_complete(unsigned long long old, unsigned long long add, int need,
                                                   long long* total) {
  const unsigned long long biased = old + add + (kCountOne >> 1);
  *total = static_cast<long long>(biased & (kCountOne - 1ull)) - static_cast<long long>(kCountOne >> 1);
  return static_cast<int>(biased >> kCountShift) == need;
}

// A warp's partial dot products of a packed tile (this CTA's local tile lt) shared with other warps
// of the CTA (`need` of them, counted on the way in): added into the tile's shared accumulators;
// the lane completing a row's count writes that row.
template <bool sys>
__device__ __forceinline__ void chain_split_add(ChainShared* sh, const ChainLayer& L, int P, int B, int r0, int r1, int e0,
                                             int e1, long long t0, long long t1, int lt, int need, int g, int q,
                                             int ex0, int ex1, uint32_t tag) {
  const int slot = lt & (kChainSplitSlots - 1);
  const int b = q >> 1;
  int w0 = -1, w1 = -1;
  long long f0 = 0, f1 = 0;
  bool any = false;
  if (!(q & 1) && b < B) {
    unsigned long long* a0 = &sh->tile_acc[slot][g][b];
    unsigned long long* a1 = &sh->tile_acc[slot][g + 8][b];
    const unsigned long long d0 = kCountOne + static_cast<unsigned long long>(t0);
    const unsigned long long d1 = kCountOne + static_cast<unsigned long long>(t1);
    const unsigned long long o0 = atomicAdd(a0, d0), o1 = atomicAdd(a1, d1);
    if (count_add_complete(o0, d0, need, &f0)) {
      *a0 = 0ull;
      w0 = r0;
      any = true;
    }
    if (count_add_complete(o1, d1, need, &f1)) {
      *a1 = 0ull;
      w1 = r1;
      any = true;
    }
  }
  if (__any_sync(0xffffffffu, any)) chain_write_rows<sys>(L, P, B, w0, w1, e0, e1, f0, f1, q, ex0, ex1, tag);
}

// Outlier tile tt done for this warp: its partials (rows r0, r1 = the slots' rows, -1 = padding)
// go into the slots' global accumulators, counted like the packed split tiles; the lane completing
// a slot's count (every warp contributing to the tile, host-counted) publishes its row.
template <bool sys>
__device__ __forceinline__ void chain_flush_outlier(const ChainLayer& L, int P, int B, int r0, int r1, int e0, int e1,
                                                 long long t0, long long t1, int tt, int g, int q, int ex0, int ex1,
                                                 uint32_t tag) {
  const int b = q >> 1;
  int w0 = -1, w1 = -1;
  long long f0 = 0, f1 = 0;
  bool any = false;
  if (!(q & 1) && b < B) {
    const int need = static_cast<int>(ld_nc_u32(L.onc + tt));  // in flight with the atomics
    const int s0 = tt * kTileRows + g, s1 = s0 + 8;
    unsigned long long* a0 = L.acc + 2 * s0 + b;
    unsigned long long* a1 = L.acc + 2 * s1 + b;
    const unsigned long long d0 = kCountOne + static_cast<unsigned long long>(t0);
    const unsigned long long d1 = kCountOne + static_cast<unsigned long long>(t1);
    unsigned long long o0 = 0, o1 = 0;
    if (r0 >= 0) o0 = atomicAdd(a0, d0);
    if (r1 >= 0) o1 = atomicAdd(a1, d1);
    if (r0 >= 0 && count_add_complete(o0, d0, need, &f0)) {
      *a0 = 0ull;
      w0 = r0;
      any = true;
    }
    if (r1 >= 0 && count_add_complete(o1, d1, need, &f1)) {
      *a1 = 0ull;
      w1 = r1;
      any = true;
    }
  }
  if (__any_sync(0xffffffffu, any)) chain_write_rows<sys>(L, P, B, w0, w1, e0, e1, f0, f1, q, ex0, ex1, tag);
}

// A finished segment of a warp's range (one call site in the kernel): outlier tiles count in,
// packed tiles the warp covered whole are written, shared ones go through the CTA's reduction
// (`need` = the packed warps whose ranges meet the tile, counted at the layer's setup).
template <bool sys>
__device__ __forceinline__ void chain_finish_segment(ChainShared* sh, const ChainLayer& L, int P, int B, int r0, int r1,
                                                  int e0, int e1, long long t0, long long t1, int seg, int whole,
                                                  int need, int tile0, int g, int q, int ex0, int ex1, uint32_t tag) {
  if (seg >= L.MT) {
    chain_flush_outlier<sys>(L, P, B, r0, r1, e0, e1, t0, t1, seg - L.MT, g, q, ex0, ex1, tag);
  } else if (whole) {
    chain_write_rows<sys>(L, P, B, r0, r1, e0, e1, t0, t1, q, ex0, ex1, tag);
  } else {
    chain_split_add<sys>(sh, L, P, B, r0, r1, e0, e1, t0, t1, seg - tile0, need, g, q, ex0, ex1, tag);
  }
}

// kMulti: several ranks (system-scope stores into every rank's copies, cross-rank flags).  The
// one-GPU instance compiles none of that, which keeps its code small.
// kVq8: the instance for chains with sub_vector_size-8 layers (their own index units); chains of
// svs-1 layers run the instance without that code.
template <int kXC, bool kMulti, bool kVq8 = false>
__global__ void __launch_bounds__(kQThreads, 1) chain_kernel(const ChainArgs args) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int S = args.stages;
  const int B = args.batch;

  const uint32_t xs_base = smem_u32(smem);
  const uint32_t ring_base = xs_base + args.xs_bytes;
  const uint32_t full_base = ring_base + kQConsumers * S * kQChunkBytes;
  const uint32_t empty_base = full_base + kQConsumers * S * 8;
  ChainShared* sh = reinterpret_cast<ChainShared*>(smem + args.xs_bytes + kQConsumers * S * (kQChunkBytes + 16));
  // sub_vector_size 8: this consumer warp's two codebook slices (after the shared state)
  const uint32_t cbs_warp = ((smem_u32(sh) + static_cast<uint32_t>(sizeof(ChainShared)) + 15u) & ~15u) + warp * 2048u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQConsumers * S; ++i) {
      mbar_init(full_base + i * 8, 1);
      mbar_init(empty_base + i * 8, 1);
    }
    fence_mbar_init();
    const uint32_t ep = ld_relaxed_u32(args.epoch);
    sh->epoch = ep & ~kChainPoisoned;
    sh->abort = (ep & kChainPoisoned) ? 1 : 0;
    if (ep & kChainPoisoned) atomicCAS(&g_opc_device_error, 0, kDevErrChainPoisoned);
  }
  for (int i = threadIdx.x; i < kChainSplitSlots * kTileRows * kQMaxBatch; i += blockDim.x)
    (&sh->tile_acc[0][0][0])[i] = 0ull;
  if (threadIdx.x < 2 * kQMaxBatch) (&sh->amax_bits[0][0])[threadIdx.x] = 0u;
  if (threadIdx.x < sizeof(ChainLayer) / 16 && args.n_layers > 0)
    reinterpret_cast<uint4*>(&sh->layer[0])[threadIdx.x] = reinterpret_cast<const uint4*>(args.layers)[threadIdx.x];
  __syncthreads();
  if (threadIdx.x < kChainSharePieces && args.n_layers > 0)
    sh->part[0][threadIdx.x] = args.parts[kChainSharePieces * blockIdx.x + threadIdx.x];
  __syncthreads();
  if (sh->abort) return;  // poisoned: no work, no flags

  // ------------------------------------------------------------------ producer warp
  // Lane i feeds consumer warp i.  Everything a lane needs about a layer lives in registers: the
  // next layer's fields are loaded when the lane starts a layer, so a layer change costs no
  // memory round trip (a stall there would hold up every lane of the warp).
  if (warp == kQProducerWarp) {
    const int i = lane;
    const uint32_t ring = ring_base + i * S * kQChunkBytes;
    const uint64_t evict_first = l2_policy_evict_first();
    // raw fields of a layer (loads in flight until first used)
    struct Raw {
      uint64_t units, ounits;
      uint32_t Up, MT, KT, KO, u0, u1, seg0;
    };
    auto fetch = [&](int jn, Raw& r) {
      if (jn >= args.n_layers || i >= kQConsumers) return;
      const ChainLayer* Ln = args.layers + jn;
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
    // the current layer of this lane, in registers
    int j = 0;
    const uint8_t* units = nullptr;
    const uint8_t* ounits = nullptr;
    int32_t Up = 0, MT = 0, KT = 1, KO = 1, u1 = 0;
    int32_t pu = 0, seg = 0, send = 0;  // cursor: unit, segment, end of segment
    Raw nx;
    fetch(0, nx);
    // advance to the next layer with a non-empty range for this consumer
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
        fetch(j + 1, nx);  // in flight while this layer streams
        if (u0 < u1) {
          pu = u0;
          send = seg < MT ? (seg + 1) * KT : Up + (seg - MT + 1) * KO;
          return true;
        }
        ++j;
      }
      return false;
    };
    bool active = i < kQConsumers;
    if (active) active = next_range();
    int slot = 0, round = 0;  // ring slot and round of this lane's next chunk
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
          if (args.l2_prefetch)
            bulk_g2s_hint(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar, evict_first);
          else
            bulk_g2s(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar);
          pu += cnt;
          if (pu == send && pu < u1) {  // next segment
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
        if (*reinterpret_cast<volatile int32_t*>(&sh->abort)) break;  // consumers gave up (error recorded)
        const uint64_t now = globaltimer_ns();
        if (t_idle == 0) t_idle = now;
        else if (now - t_idle > 2 * kWaitLimitNs) {  // longer than any consumer wait: theirs report first
          failed = true;
          break;
        }
        nanosleep_ns(64);
      }
    }
    if (failed && lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
    // Copies that consumers which gave up never waited for land before the CTA exits: wait
    // (bounded) for the last chunk issued into each ring slot.
    if (i < kQConsumers) {
      for (int s = 0; s < S; ++s) {
        const int n_in_slot = round + (s < slot ? 1 : 0);  // chunks issued into slot s
        if (n_in_slot > 0) mbar_wait_bounded(full_base + (i * S + s) * 8, static_cast<uint32_t>((n_in_slot - 1) & 1));
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  const int g = lane >> 2, q = lane & 3;
  const int tid = threadIdx.x;
  const uint32_t negz = args.negz;
  const uint32_t ring = ring_base + warp * S * kQChunkBytes + lane * 16;
  const uint32_t fullw = full_base + warp * S * 8, emptyw = empty_base + warp * S * 8;
  const int P = kMulti ? args.world : 1;
  constexpr bool sys = kMulti;
  const int n_flags = P * G;
  const uint32_t epoch = sh->epoch;
  const uint32_t f_staged0 = 2u * epoch + 1u;  // flag: this CTA staged layer 0
  const uint32_t f_done = 2u * epoch + 2u;     // flag: this CTA finished the launch (several ranks)
  const uint32_t tag_base = chain_tag_base(epoch, args.n_layers);
  int slot = 0;
  uint32_t phase = 0;
  bool ok = true;
  bool staged0_seen = false;  // every CTA has staged layer 0 (true for the rest of the launch once seen)

  // Every CTA of every rank has published at least `target` (bounded; sets abort on a timeout).
  // The polling lanes' acquire fence plus the CTA barrier order every thread's later accesses.
  auto wait_all = [&](uint32_t target) {
    if (warp == 0 && !poll_flags_warp(args.sync, n_flags, lane, target, sys) && lane == 0) {
      sh->abort = 1;
      atomicCAS(&g_opc_device_error, 0, kDevErrBarrierTimeout);
    }
    named_barrier(1, kQConsumerThreads);
  };
  // After a CTA barrier: this CTA's flag in every rank's memory.  The publishing thread's fence
  // is cumulative: it orders every access the barrier made it observe before the flag.
  auto publish = [&](uint32_t value) {
    if (sys) {
      if (tid < P) fence_acq_rel_sys();
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)  // constant indices: the pointers stay in the parameter space
        if (p == tid && p < P) st_relaxed_sys_u32(args.sync_peer[p] + args.rank * G + cta, value);
    } else if (tid == 0) {
      fence_acq_rel_gpu();
      st_relaxed_u32(args.sync + cta, value);
    }
  };

  for (int j = 0; j < args.n_layers && ok; ++j) {
    // Descriptors live in shared memory (layer j+1's is copied during layer j's staging), so
    // reading them costs no global round trip and holds no registers.
    const ChainLayer& L = sh->layer[j & 1];
    const uint32_t tag = chain_tag(tag_base, j);
    const uint32_t tag_in = j > 0 ? chain_tag(tag_base, j - 1) : 0u;
    // Everything about this warp's share that does not depend on x, before x is complete.
    GemvQArgs qa;  // the per-layer view load_metaq takes
    qa.cbq = L.cbq; qa.tile_mask = L.tile_mask; qa.orow = L.orow; qa.oexp = L.oexp; qa.M = L.M; qa.MT = L.MT;
    unsigned long long* tr = args.trace ? args.trace + (static_cast<int64_t>(j) * G + cta) * kChainTracePhases : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer_ns();
    const int32_t* sr = reinterpret_cast<const int32_t*>(sh->part[j & 1]);
    const int32_t u0 = sr[kShU0 + warp], u1 = sr[kShU1 + warp];
    ChainCursor cc = chain_cursor_at(L, u0, sr[kShSeg0 + warp]);
    MetaQ cur, nxt;
    if (u0 < u1) {  // both loads issued here, first used in the units loop (no select on them)
      cur = chain_load_meta(qa, cc.seg, g);
      nxt = chain_load_meta(qa, min(cc.seg + 1, L.MT + L.OT - 1), g);
    }
    int cbuf = 0;  // sub_vector_size 8: the slice holding the current row tile's codebooks
    if constexpr (kVq8) {
      if (L.vq8 && u0 < u1) {
        cp_async_wait_all();  // copies a previous layer left in flight land before the slices are reused
        __syncwarp();
        if (cc.seg < L.MT) chain_vq8_slice(cbs_warp, L.cbv, cc.seg, lane);
        if (cc.seg + 1 < L.MT) chain_vq8_slice(cbs_warp + 1024, L.cbv, cc.seg + 1, lane);
      }
    }
    // contributors (packed warps of this CTA) of the first and the last packed tile of this warp's
    // range -- the only ones it may share -- counted while x is not complete yet
    int need_first = 0, need_last = 0;
    const int tile0 = sr[kShTile0];
    if (u0 < u1 && cc.seg < L.MT) {
      const int32_t fb = cc.begin, fe = cc.end;
      int32_t lb = fb, le = fe;
      while (le < u1) {
        lb = le;
        le += L.KT;
      }
      const int wp = sr[kShWp];
      for (int w = 0; w < wp; ++w) {
        const int32_t a = sr[kShU0 + w], b = sr[kShU1 + w];
        need_first += (a < b && a < fe && b > fb) ? 1 : 0;
        need_last += (a < b && a < le && b > lb) ? 1 : 0;
      }
    }
    const int32_t seg_first = cc.seg;
    // next layer's descriptor and this CTA's share of it: loaded now, stored to shared memory
    // once every warp is past this layer's first staging barrier (nobody reads the slots' old
    // contents after that)
    // (the last consumer warp: with more chunks than threads, the first warps stage more of x)
    constexpr int kDescPieces = static_cast<int>(sizeof(ChainLayer) / 16);
    const int dt = tid - (kQConsumerThreads - 32);
    const bool copy_desc = j + 1 < args.n_layers && dt >= 0 && dt < kDescPieces + kChainSharePieces;
    uint4 desc_piece = make_uint4(0, 0, 0, 0);
    if (copy_desc) {
      if (dt < kDescPieces) {
        desc_piece = ld_nc_v4(reinterpret_cast<const uint4*>(args.layers + j + 1) + dt);
      } else {
        const int4* pe = args.parts + kChainSharePieces * (static_cast<int64_t>(j + 1) * G + cta) + (dt - kDescPieces);
        desc_piece = ld_nc_v4(reinterpret_cast<const uint4*>(pe));
      }
    }
    if (tr && tid == 0) tr[1] = globaltimer_ns();

    // ---- stage x_j.  Layer 0 reads the fp16 input; later layers poll the previous layer's
    // exchange words of their chunks until every tag is this launch's (bounded).
    int ex0 = 0, ex1 = 0;  // x exponents of batch rows 0, 1 (scalars: no local memory)
    {
      static_assert(kQMaxBatch == 2, "chunk c of batch row c >= per_row: no division");
      const int per_row = L.K_pad / 8;
      const int total = B * per_row;
      uint4 v[kXC];
      uint32_t pending = 0;  // chunks still to take
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        v[i] = make_uint4(0, 0, 0, 0);
        if (c < total && (c - (c >= per_row ? per_row : 0)) * 8 < L.K) pending |= 1u << i;
      }
      if (j == 0) {
#pragma unroll
        for (int i = 0; i < kXC; ++i) {
          if (pending & (1u << i)) {
            const int c = tid + i * kQConsumerThreads;
            const int b = c >= per_row ? 1 : 0, k = (c - b * per_row) * 8;  // c < 2 per_row (batch <= 2)
            v[i] = chain_load_x0(L.x, L.ldx, b, k, L.K, L.x_vec16);
          }
        }
        pending = 0;
      }
      if (tr && tid == 0) tr[2] = globaltimer_ns();
      // layers >= 1: poll the exchange words of every pending chunk until all carry this launch's
      // tag (bounded)
      uint64_t t0 = 0;
      while (pending) {
#pragma unroll
        for (int i = 0; i < kXC; ++i) {
          if (pending & (1u << i)) {
            const int c = tid + i * kQConsumerThreads;
            const int b = c >= per_row ? 1 : 0, k = (c - b * per_row) * 8;
            const ChainChunk r = chain_poll_chunk<sys>(L.xw, L.ldxw, b, k, L.K, tag_in);
            if (r.ok) {
              v[i] = r.v;
              pending &= ~(1u << i);
            }
          }
        }
        if (!pending) break;
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > kWaitLimitNs) {
          sh->abort = 1;
          atomicCAS(&g_opc_device_error, 0, kDevErrBarrierTimeout);
          break;
        }
      }
      if (tr && tid == 0) tr[3] = globaltimer_ns();
      float mx[kQMaxBatch] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        if (c < total) {
          const float m = chain_chunk_amax(v[i]);
          if (c < per_row) mx[0] = fmaxf(mx[0], m);
          else mx[1] = fmaxf(mx[1], m);
        }
      }
      // non-negative floats order like their bit patterns: one warp max and one shared-memory
      // atomic per warp and batch row (a NaN maximum counts as 0, as fmaxf would skip it)
#pragma unroll
      for (int b = 0; b < kQMaxBatch; ++b) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, mx[b] == mx[b] ? __float_as_uint(mx[b]) : 0u);
        if (lane == 0) atomicMax(&sh->amax_bits[j & 1][b], m);
      }
      if (tid < 16)  // ones block, zero block (B operands of the ones and absent columns)
        sts128(xs_base + args.xs_bytes - kQZeroBytes - kQOnesBytes + tid * 16,
               tid < 8 ? make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u) : make_uint4(0, 0, 0, 0));
      named_barrier(1, kQConsumerThreads);  // every warp is done with layer j-1 and holds its x
      if (tr && tid == 0) tr[4] = globaltimer_ns();
      if (sh->abort) {
        ok = false;
        break;
      }
      if (copy_desc) {
        if (dt < kDescPieces) reinterpret_cast<uint4*>(&sh->layer[(j + 1) & 1])[dt] = desc_piece;
        else reinterpret_cast<uint4*>(sh->part[(j + 1) & 1])[dt - kDescPieces] = desc_piece;
      }
      if (j == 0) publish(f_staged0);  // layer-0 input read by every thread of this CTA
      {
        const float m0 = __uint_as_float(sh->amax_bits[j & 1][0]), m1 = __uint_as_float(sh->amax_bits[j & 1][1]);
        ex0 = m0 > 0.f ? 22 - frexp_exponent(m0) : 0;
        ex1 = m1 > 0.f ? 22 - frexp_exponent(m1) : 0;
        // the other parity's maxima start layer j+1 at zero: their last readers (layer j-1) are
        // past this barrier, their next writers (layer j+1) behind the staged barrier below
        if (tid < kQMaxBatch) sh->amax_bits[(j + 1) & 1][tid] = 0u;
      }
      const uint32_t colb = static_cast<uint32_t>(xsq_col_bytes(kVq8 && L.vq8 ? L.cb_stride : L.KT));
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        if (c < total) {
          const int b = c >= per_row ? 1 : 0, k = (c - b * per_row) * 8;
          chain_store_digits(v[i], pow2f(b == 0 ? ex0 : ex1), xs_base + 3 * b * colb, colb,
                             static_cast<uint32_t>((k >> 7) * 128 + xs_pos8(k & 127)));
        }
      }
      if (tr && tid == 0) tr[5] = globaltimer_ns();
      // a layer writing over the chain input starts once every CTA has read that input (flags
      // only grow within a launch, so the first layer that needs it waits and later ones do not)
      if (L.y_alias_x0 && !staged0_seen) {
        if (warp == 0 && !poll_flags_warp(args.sync, n_flags, lane, f_staged0, sys) && lane == 0) {
          sh->abort = 1;
          atomicCAS(&g_opc_device_error, 0, kDevErrBarrierTimeout);
        }
        staged0_seen = true;  // uniform over the consumer warps; a failed wait aborts below
      }
      named_barrier(1, kQConsumerThreads);
      if (sh->abort) {
        ok = false;
        break;
      }
    }
    if (tr && tid == 0) tr[6] = globaltimer_ns();

    // ---- this warp's units of layer j
    const int bcol = g >> 2, dig = g & 3;
    const bool live_col = dig < 3 && bcol < B;
    const uint32_t colbase = live_col ? xs_base + (3 * bcol + dig) * xsq_col_bytes(kVq8 && L.vq8 ? L.cb_stride : L.KT)
                                      : xs_base + args.xs_bytes - (bcol < B ? kQZeroBytes + kQOnesBytes : kQZeroBytes);
    const uint32_t kts = live_col ? 128u : 0u;
    const uint32_t xq = colbase + 32 * q, xo = colbase + 4 * q;

    if (u0 < u1) {
      AccQ A;
      zero_accq(A);
      const bool vq8 = kVq8 && L.vq8 != 0;
      if (vq8) {  // the first row tile's slice has landed
        cp_async_wait_all();
        __syncwarp();
      }
      while (cc.u < u1) {
        if (!mbar_wait_bounded(fullw + slot * 8, phase)) {
          ok = false;
          break;
        }
        const int32_t cnt = chain_chunk(cc, u1);
        const uint32_t stage = ring + slot * kQChunkBytes;
        const int32_t k0 = cc.u - cc.begin;
        if (kVq8 && vq8 && cc.seg < L.MT) {
          // sub_vector_size 8: unit = four 128-byte index units of 256 columns; lane (g, q) reads
          // the 16 bytes of row pair g of each (byte b = k16 step b: bits 2w / 4+2w the vector of
          // the step's 8-column group w for rows g / g+8), and for the 32 columns of step jw of a
          // 128-column half the vector of its group 4jw+q: one 16-byte slice load per row gives the
          // hi and lo parts of both vector halves (A-fragment registers k 4q.. and 16+4q..)
          const uint32_t ub = stage - lane * 16 + g * 16;
          const uint32_t cbs = cbs_warp + cbuf * 1024;
#pragma unroll 1
          for (int i = 0; i < cnt; ++i) {
#pragma unroll 1
            for (int v = 0; v < 4; ++v) {
              const uint4 ib = lds128(ub + i * kUnitBytes + v * 128);
              const uint32_t iw[4] = {ib.x, ib.y, ib.z, ib.w};
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t xa = xq + static_cast<uint32_t>(8 * (k0 + i) + 2 * v + h) * kts;
                const uint4 b01 = lds128(xa), b23 = lds128(xa + 16);
                const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
                for (int jw = 0; jw < 4; ++jw) {
                  const int bi = 2 * jw + (q >> 1);
                  const uint32_t byte = iw[2 * h + (bi >> 2)] >> (8 * (bi & 3));
                  const uint32_t sft = 2 * (q & 1);
                  const uint32_t i0 = (byte >> sft) & 3u, i1 = (byte >> (4 + sft)) & 3u;
                  const uint4 c0 = lds128(cbs + (g * 4 + i0) * 16), c1 = lds128(cbs + ((g + 8) * 4 + i1) * 16);
                  const uint32_t Ah[4] = {c0.x, c1.x, c0.y, c1.y}, Al[4] = {c0.z, c1.z, c0.w, c1.w};
                  imma16832(A.h[jw & 1], Ah, bb[2 * jw], bb[2 * jw + 1]);
                  imma16832(A.l[jw & 1], Al, bb[2 * jw], bb[2 * jw + 1]);
                }
              }
            }
          }
        } else if (cc.seg < L.MT) {
          // not unrolled: one unit carries enough independent work for the ALU and tensor pipes
          // (unrolling 2-8 units measured no faster), and the small loop keeps the kernel's code
          // -- which every layer re-fetches -- small
#pragma unroll 1
          for (int i = 0; i < cnt; ++i) {
            const uint4 wv = lds128(stage + i * kUnitBytes);
            const uint32_t xa = xq + static_cast<uint32_t>(k0 + i) * kts;
            const uint4 b01 = lds128(xa), b23 = lds128(xa + 16);
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
        if (cc.u == cc.end || cc.u == u1) {  // a segment of the range is complete (one call site)
          long long t[2];
          finish_dot(A, q, t);
          int r0 = cur.row[0], r1 = cur.row[1];
          if (cc.seg < L.MT) {  // packed tile: base row and raw mask -> output rows (-1: masked or past M)
            const uint32_t mask = static_cast<uint32_t>(r1);
            r1 = (r0 + 8 < L.M && !((mask >> (g + 8)) & 1u)) ? r0 + 8 : -1;
            r0 = (r0 < L.M && !((mask >> g) & 1u)) ? r0 : -1;
          }
          chain_finish_segment<sys>(sh, L, P, B, r0, r1, cur.e[0], cur.e[1], t[0], t[1], cc.seg,
                                    cc.begin >= u0 && cc.end <= u1, cc.seg == seg_first ? need_first : need_last,
                                    tile0, g, q, ex0, ex1, tag);
          if (cc.u == u1) break;
          zero_accq(A);
          chain_next_segment(L, cc);
          cur = nxt;
          if (cc.seg + 1 < L.MT + L.OT) nxt = chain_load_meta(qa, cc.seg + 1, g);
          if constexpr (kVq8) {
            if (vq8 && cc.seg < L.MT) {  // the next tile's slice (issued a segment ago) lands; refill the other
              cbuf ^= 1;
              cp_async_wait_all();
              __syncwarp();
              if (cc.seg + 1 < L.MT) chain_vq8_slice(cbs_warp + (cbuf ^ 1) * 1024, L.cbv, cc.seg + 1, lane);
            }
          }
        }
      }
      if (!ok) {
        atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
        sh->abort = 1;  // every consumer sees it at the next staging barrier
        ok = true;      // this warp still takes part in the CTA's barriers until then
      }
    }
    if (tr && tid == 0) tr[7] = globaltimer_ns();
    if (tr && lane == 0) tr[8 + warp] = globaltimer_ns();
  }

  // ---- end of the launch.  Several ranks: a last barrier, so that no rank starts its next
  // launch while a peer still writes or reads this one's buffers (its fp16 outputs are complete
  // when it passes).  The last CTA of this rank to finish advances the epoch.
  named_barrier(1, kQConsumerThreads);
  if (sh->abort) ok = false;
  if (ok && sys && args.n_layers > 0) {
    publish(f_done);
    wait_all(f_done);
    if (sh->abort) ok = false;
  }
  if (tid == 0) {
    if (!ok) atomicOr(args.epoch, kChainPoisoned);
    __threadfence();
    const unsigned int done = atomicAdd(args.epoch + 1, 1u);
    if (done == static_cast<unsigned int>(G) - 1u) {
      st_relaxed_u32(args.epoch + 1, 0u);
      atomicAdd(args.epoch, 1u);
    }
  }
}

}  // namespace opc
