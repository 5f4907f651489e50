// opc_chain.cuh -- persistent decode-chain kernel: a whole sequence of dependent fused 2-bit
// GEMVs (one decode token through every projection of every block) in one cooperative launch.
//
// Each layer is the integer-split GEMV of opc_gemvq.cuh (8 PRMT + 3 ALU operations and two int8
// mma.sync per 16 weights, exact int64 dot products).  What changes is the orchestration:
//
//  * One CTA per SM stays resident for the whole chain.  A producer warp streams every layer's
//    units for the CTA's 15 consumer warps through their rings and runs ahead across layer
//    boundaries (weights do not depend on activations), so HBM keeps streaming while the
//    consumers wait for a layer's input.
//  * Layer j+1 needs all of layer j's output: a grid barrier (per-CTA flags, release/acquire at
//    GPU scope, bounded wait) separates them.  Each CTA then stages x itself from y_j.
//  * Packed row tiles are handed out whole (CTA c gets tiles round(c*MT/G) .. round((c+1)*MT/G)),
//    so a tile is split only between warps of one CTA and reduced in shared memory; no
//    cross-CTA reduction exists for them.  Outlier tiles (16 fp16 rows, 8x heavier per row) are
//    split evenly across all CTAs and their partial dot products are added exactly into int64
//    accumulators per outlier slot; the next layer's staging reads those for its outlier rows,
//    and the CTA owning slot s (s mod G) writes that row of y.
#pragma once

#include "opc_gemvq.cuh"

namespace opc {

struct ChainLayer {
  const uint8_t* units;      // packed units
  const uint8_t* ounits;     // int8 outlier units
  const uint4* cbq;          // [M_pad] integer codebooks; outlier rows {0, 0, e, slot}
  const uint16_t* tile_mask; // [MT]
  const int32_t* orow;       // [OT*16]
  const int32_t* oexp;       // [OT*16]
  const __half* x;           // layer input (layer 0: the chain input; else a prefix of the previous y)
  __half* y;                 // layer output
  unsigned long long* acc;   // [OT*16][2] outlier-slot dot products (zero at launch)
  int64_t ldx, ldy;
  int32_t Up, U, M, K, K_pad, MT, KT, OT, KO;
  int32_t x_vec16;           // x rows 16-byte loadable
};

static_assert(sizeof(ChainLayer) % 16 == 0, "ChainLayer is copied in 16-byte pieces");

struct ChainArgs {
  const ChainLayer* layers;
  unsigned int* sync;        // [grid] per-CTA "layers finished" flags (zero at launch)
  unsigned long long* trace; // optional [n_layers][grid][8] globaltimer stamps (ns) per CTA,
                             // taken by its first consumer thread: input ready, own x loads
                             // done, exponents known, x staged, own units done, own writes
                             // fenced, CTA's writes fenced, flag published
  int32_t n_layers, batch, stages, xs_bytes;
  uint32_t negz;
  int32_t l2_prefetch;       // prefetch each consumer's share of the next layer into L2
};
constexpr int kChainTracePhases = 8;

// This CTA's share of a layer: packed units [pu0, pu1) (whole tiles) and outlier units
// [ou0, ou1); warps 0..wp-1 take the packed share, the other consumer warps the outlier share.
struct ChainPart {
  int32_t pu0, pu1, ou0, ou1, wp;
};
__device__ __forceinline__ ChainPart chain_part(const ChainLayer& L, int c, int G) {
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
    p.wp = kQConsumers;
  } else if (np == 0) {
    p.wp = 0;
  } else {
    int wo = static_cast<int>((2ll * kQConsumers * no + (np + no)) / (2ll * (np + no)));
    wo = wo < 1 ? 1 : (wo > kQConsumers - 1 ? kQConsumers - 1 : wo);
    p.wp = kQConsumers - wo;
  }
  // Every packed warp gets at least one unit, so the warps sharing a tile are exactly the parts
  // between the parts of its first and last unit (the split-tile contributor count relies on it).
  if (p.wp > np) p.wp = np;
  return p;
}
__device__ __forceinline__ void chain_warp_range(const ChainPart& p, int w, int32_t* u0, int32_t* u1) {
  if (w < p.wp) {
    const int32_t np = p.pu1 - p.pu0;
    *u0 = p.pu0 + partq_start(w, np, p.wp);
    *u1 = p.pu0 + partq_start(w + 1, np, p.wp);
  } else {
    const int32_t no = p.ou1 - p.ou0, nw = kQConsumers - p.wp;
    *u0 = p.ou0 + partq_start(w - p.wp, no, nw);
    *u1 = p.ou0 + partq_start(w - p.wp + 1, no, nw);
  }
}

// Unit cursor over a layer (segments: packed tiles of KT units, outlier tiles of KO units).
struct ChainCursor {
  int32_t u, seg, begin, end;
};
__device__ __forceinline__ ChainCursor chain_cursor(const ChainLayer& L, int32_t u) {
  ChainCursor c;
  c.u = u;
  if (u < L.Up) {
    c.seg = u / L.KT;
    c.begin = c.seg * L.KT;
    c.end = c.begin + L.KT;
  } else {
    const int32_t t = (u - L.Up) / L.KO;
    c.seg = L.MT + t;
    c.begin = L.Up + t * L.KO;
    c.end = c.begin + L.KO;
  }
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

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kChainPatchMax = 512;  // outlier slots of a layer whose values go through shared memory
constexpr int kChainMaskMax = 2048;  // row tiles of the previous layer covered by x (tile masks in smem)

// Grid barrier over per-CTA flags: CTA c publishes "finished layer j" with a release store of j+1
// into flags[c]; a waiter's threads t < G each poll flags[t] with acquire loads (bounded), then
// meet at a CTA barrier.  No atomic is shared by all CTAs.
__device__ __forceinline__ void st_relaxed_u32(unsigned int* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_u32(unsigned int* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// One warp polls all G flags (lane l: flags l, l+32, ...) until every one reaches target.
__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Each lane reads its flags with independent relaxed loads (all in flight together); once every
// flag has reached target an acquire fence orders the caller's later reads after them.
__device__ __forceinline__ bool poll_flags_warp(const unsigned int* flags, int G, int lane, uint32_t target) {
  uint64_t t0 = 0;
  for (;;) {
    uint32_t lo = 0xffffffffu;
    for (int t = lane; t < G; t += 32) lo = min(lo, ld_relaxed_u32(flags + t));
    if (__all_sync(0xffffffffu, lo >= target)) {
      fence_acq_rel_gpu();
      return true;
    }
    const uint64_t now = globaltimer_ns();
    if (t0 == 0) t0 = now;
    else if (now - t0 > kWaitLimitNs) return false;
  }
}

// Exact 2^e for e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// What the staging of layer j needs from layer j-1 (kept in registers, loaded before the wait).
struct PrevInfo {
  const uint16_t* tile_mask;
  const int32_t* orow;
  const int32_t* oexp;
  const uint4* cbq;
  const unsigned long long* acc;
  __half* y;
  int64_t ldy;
  int32_t n_slots;
};
__device__ __forceinline__ __half prev_outlier_value(const PrevInfo& P, int s, int b, int ex) {
  const long long t = static_cast<long long>(__ldcg(P.acc + 2 * s + b));
  return scale_to_half(t, __ldg(P.oexp + s) + ex);
}

constexpr int kChainSplitSlots = 32;  // packed tiles per CTA and layer (host-checked)

struct ChainShared {
  ChainLayer layer[2];                    // descriptors of layers j (slot j&1) and j+1
  float amax[kQConsumers][kQMaxBatch];    // staging: per-warp max |x|
  unsigned long long tile_acc[kChainSplitSlots][kTileRows][kQMaxBatch];  // split packed tiles
  int32_t tile_cnt[kChainSplitSlots];
  int32_t patch_row[kChainPatchMax];      // previous layer's outlier rows by slot
  int32_t patch_exp[kChainPatchMax];      // and their integer-row exponents
  uint16_t patch_val[kChainPatchMax][kQMaxBatch];
  uint16_t prev_mask[kChainMaskMax];      // previous layer's tile masks of the rows x reads
  int32_t abort;
};

// A warp's partial dot products of packed tile `seg` (this CTA's local tile lt), shared with
// other warps of the CTA: added exactly into the tile's shared int64 accumulators; the warp that
// completes the count of contributors writes the tile's rows and clears the slot.
__device__ void chain_split_add(ChainShared* sh, const GemvQArgs& qa, const MetaQ& m, const long long t[2], int lt,
                                int n_contrib, int lane, int g, int q, int ex0, int ex1) {
  const int slot = lt & (kChainSplitSlots - 1);
  const int b = q >> 1;
  const bool live = !(q & 1) && b < qa.batch;
  if (live) {
    atomicAdd(&sh->tile_acc[slot][g][b], static_cast<unsigned long long>(t[0]));
    atomicAdd(&sh->tile_acc[slot][g + 8][b], static_cast<unsigned long long>(t[1]));
  }
  __threadfence_block();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(&sh->tile_cnt[slot], 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != n_contrib - 1) return;
  __threadfence_block();
  long long fin[2] = {0, 0};
  if (live) {
    fin[0] = static_cast<long long>(atomicExch(&sh->tile_acc[slot][g][b], 0ull));
    fin[1] = static_cast<long long>(atomicExch(&sh->tile_acc[slot][g + 8][b], 0ull));
  }
  if (lane == 0) sh->tile_cnt[slot] = 0;
  write_outq(qa, m, fin, q, ex0, ex1);
}

template <int kXC>
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

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQConsumers * S; ++i) {
      mbar_init(full_base + i * 8, 1);
      mbar_init(empty_base + i * 8, 1);
    }
    fence_mbar_init();
    sh->abort = 0;
  }
  for (int i = threadIdx.x; i < kChainSplitSlots * kTileRows * kQMaxBatch; i += blockDim.x)
    (&sh->tile_acc[0][0][0])[i] = 0ull;
  for (int i = threadIdx.x; i < kChainSplitSlots; i += blockDim.x) sh->tile_cnt[i] = 0;
  if (threadIdx.x < sizeof(ChainLayer) / 16 && args.n_layers > 0)
    reinterpret_cast<uint4*>(&sh->layer[0])[threadIdx.x] = reinterpret_cast<const uint4*>(args.layers)[threadIdx.x];
  __syncthreads();

  // ------------------------------------------------------------------ producer warp
  if (warp == kQProducerWarp) {
    const int i = lane;
    const uint32_t ring = ring_base + i * S * kQChunkBytes;
    int j = 0;
    int32_t u1 = 0;
    ChainCursor pc = {0, 0, 0, 0};
    const ChainLayer* Lp = nullptr;
    bool active = i < kQConsumers;
    // advance to the first layer with a non-empty range for this consumer
    const uint64_t evict_first = l2_policy_evict_first();
    // When this lane starts layer j, its consumer's share of layer j+1 is prefetched into L2, so
    // HBM streams the next layer during this one's compute and its ring refills hit L2.
    auto prefetch_next = [&](int jn) {
      if (!args.l2_prefetch || jn >= args.n_layers) return;
      const ChainLayer N = args.layers[jn];
      const ChainPart p = chain_part(N, cta, G);
      int32_t a0, a1;
      chain_warp_range(p, i, &a0, &a1);
      if (a0 >= a1) return;
      const uint8_t* src = a0 < N.Up ? N.units + static_cast<int64_t>(a0) * kUnitBytes
                                     : N.ounits + static_cast<int64_t>(a0 - N.Up) * kUnitBytes;
      int64_t bytes = static_cast<int64_t>(a1 - a0) * kUnitBytes;
      while (bytes > 0) {
        const uint32_t n = bytes > 65536 ? 65536u : static_cast<uint32_t>(bytes);
        l2_prefetch_bulk(src, n);
        src += n;
        bytes -= n;
      }
    };
    auto next_range = [&]() {
      while (j < args.n_layers) {
        Lp = args.layers + j;
        const ChainLayer L = *Lp;
        const ChainPart p = chain_part(L, cta, G);
        int32_t u0;
        chain_warp_range(p, i, &u0, &u1);
        prefetch_next(j + 1);
        if (u0 < u1) {
          pc = chain_cursor(L, u0);
          return true;
        }
        ++j;
      }
      return false;
    };
    if (active) active = next_range();
    int32_t c = 0;
    uint64_t t_idle = 0;
    bool failed = false;
    while (__any_sync(0xffffffffu, active)) {
      bool issued = false;
      if (active) {
        const int slot = c % S;
        const int round = c / S;
        if (round == 0 || mbar_test(empty_base + (i * S + slot) * 8, static_cast<uint32_t>((round - 1) & 1))) {
          const int32_t cnt = chain_chunk(pc, u1);
          const uint32_t bar = full_base + (i * S + slot) * 8;
          mbar_expect_tx(bar, static_cast<uint32_t>(cnt * kUnitBytes));
          const int32_t Up = Lp->Up;
          const uint8_t* src = pc.u < Up ? Lp->units + static_cast<int64_t>(pc.u) * kUnitBytes
                                         : Lp->ounits + static_cast<int64_t>(pc.u - Up) * kUnitBytes;
          if (args.l2_prefetch)
            bulk_g2s_hint(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar, evict_first);
          else
            bulk_g2s(ring + slot * kQChunkBytes, src, static_cast<uint32_t>(cnt * kUnitBytes), bar);
          pc.u += cnt;
          if (pc.u == pc.end && pc.u < u1) {
            const ChainLayer L = *Lp;
            chain_next_segment(L, pc);
          }
          ++c;
          issued = true;
          if (pc.u >= u1) {
            ++j;
            active = next_range();
          }
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
  const int tid = threadIdx.x;
  const uint32_t negz = args.negz;
  const uint32_t ring = ring_base + warp * S * kQChunkBytes + lane * 16;
  const uint32_t fullw = full_base + warp * S * 8, emptyw = empty_base + warp * S * 8;
  int slot = 0;
  uint32_t phase = 0;
  int32_t ex_prev[kQMaxBatch] = {0, 0};
  bool ok = true;

  for (int j = 0; j < args.n_layers && ok; ++j) {
    // Descriptors live in shared memory (layer j+1's is copied at the end of layer j), so reading
    // them costs no global round trip and holds no registers.
    const ChainLayer& L = sh->layer[j & 1];
    // Everything about this warp's share that does not depend on x, before waiting for x.
    GemvQArgs qa;  // the per-layer view the shared helpers take
    qa.units = L.units; qa.ounits = L.ounits; qa.cbq = L.cbq; qa.tile_mask = L.tile_mask; qa.orow = L.orow;
    qa.oexp = L.oexp; qa.x = L.x; qa.y = L.y; qa.acc = nullptr; qa.counters = nullptr; qa.ldx = L.ldx;
    qa.ldy = L.ldy; qa.Up = L.Up; qa.U = L.U; qa.M = L.M; qa.K = L.K; qa.K_pad = L.K_pad; qa.MT = L.MT;
    qa.KT = L.KT; qa.OT = L.OT; qa.KO = L.KO; qa.batch = B; qa.stages = S; qa.xs_bytes = args.xs_bytes;
    qa.x_vec16 = 0; qa.negz = negz;
    const ChainPart part = chain_part(L, cta, G);
    int32_t u0, u1;
    chain_warp_range(part, warp, &u0, &u1);
    ChainCursor cc = chain_cursor(L, u0 < u1 ? u0 : 0);
    MetaQ cur, nxt;
    if (u0 < u1) {  // issued before the wait; first used by the units loop
      cur = load_metaq(qa, cc.seg, g);
      nxt = (cc.seg + 1 < L.MT + L.OT) ? load_metaq(qa, cc.seg + 1, g) : cur;
    }
    PrevInfo P = {};
    if (j > 0) {
      const ChainLayer& Lp = sh->layer[(j - 1) & 1];
      P.tile_mask = Lp.tile_mask;
      P.orow = Lp.orow;
      P.oexp = Lp.oexp;
      P.cbq = Lp.cbq;
      P.acc = Lp.acc;
      P.y = Lp.y;
      P.ldy = Lp.ldy;
      P.n_slots = Lp.OT * kTileRows;
    }
    const bool mask_in_smem = j > 0 && (L.K + 15) / 16 <= kChainMaskMax;
    // ---- wait for layer j-1 everywhere
    if (j > 0) {
      if (warp == 0 && !poll_flags_warp(args.sync, G, lane, static_cast<uint32_t>(j))) {
        if (lane == 0) {
          sh->abort = 1;
          atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
        }
      }
      fence_acq_rel_gpu();
      named_barrier(1, kQConsumerThreads);
      if (sh->abort) {
        ok = false;
        break;
      }
    }
    unsigned long long* tr = args.trace ? args.trace + (static_cast<int64_t>(j) * G + cta) * kChainTracePhases : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer_ns();
    const bool has_prev = j > 0;

    // ---- stage x_j (x = the previous output when j > 0).  Round 1 issues every load at once:
    // this thread's x chunks with the previous layer's outlier flags of their rows, and (slot
    // threads) the previous layer's outlier values.  Outlier rows of y_{j-1} are read from the
    // slot accumulators, never from y, and published through a shared patch table sorted by row.
    int ex0 = 0, ex1 = 0;  // x exponents of batch rows 0, 1 (scalars: no local memory)
    {
      const int per_row = L.K_pad / 8;
      const int total = B * per_row;
      const int n_pslots = has_prev ? P.n_slots : 0;
      uint4 v[kXC];
      uint32_t tmw[kXC];
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        v[i] = make_uint4(0, 0, 0, 0);
        tmw[i] = 0;
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          if (k < L.K) {
            const __half* src = L.x + b * L.ldx + k;
            if (L.x_vec16) {
              v[i] = ld_cg_v4(src);
            } else {
              uint16_t h[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                h[e] = (k + e < L.K) ? __ldcg(reinterpret_cast<const unsigned short*>(src) + e) : 0;
              v[i] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                                h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
            }
            if (has_prev) {
              const uint32_t mw = mask_in_smem ? sh->prev_mask[k >> 4] : __ldg(P.tile_mask + (k >> 4));
              uint32_t tm = (mw >> (k & 15)) & 0xffu;
              if (k + 8 > L.K) tm &= (1u << (L.K - k)) - 1u;
              tmw[i] = tm;
            }
          }
        }
      }
      float mx[kQMaxBatch] = {0.f, 0.f};
      // slot threads: the previous layer's outlier values (y rows owned by this CTA written here)
      for (int s = tid; s < n_pslots; s += kQConsumerThreads) {
        const int row = s < kChainPatchMax ? sh->patch_row[s] : __ldg(P.orow + s);
        const int e0 = s < kChainPatchMax ? sh->patch_exp[s] : __ldg(P.oexp + s);
        const long long t0 = static_cast<long long>(__ldcg(P.acc + 2 * s));
        const long long t1 = B > 1 ? static_cast<long long>(__ldcg(P.acc + 2 * s + 1)) : 0ll;
        const __half h0 = scale_to_half(t0, e0 + ex_prev[0]);
        const __half h1 = scale_to_half(t1, e0 + ex_prev[1]);
        if (row >= 0 && s % G == cta) {
          P.y[row] = h0;
          if (B > 1) P.y[P.ldy + row] = h1;
        }
        if (s < kChainPatchMax) {
          sh->patch_row[s] = row;
          sh->patch_val[s][0] = __half_as_ushort(h0);
          sh->patch_val[s][1] = __half_as_ushort(h1);
        }
        if (row >= 0 && row < L.K) {
          mx[0] = fmaxf(mx[0], fabsf(__half2float(h0)));
          if (B > 1) mx[1] = fmaxf(mx[1], fabsf(__half2float(h1)));
        }
      }
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        if (c < total) {
          const int b = c / per_row;
          const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          float m = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if ((tmw[i] >> e) & 1u) continue;  // outlier row: its value comes from the patch table
            const __half hv = __ushort_as_half(static_cast<unsigned short>((wv[e >> 1] >> (16 * (e & 1))) & 0xffffu));
            m = fmaxf(m, fabsf(__half2float(hv)));
          }
          if (b == 0) mx[0] = fmaxf(mx[0], m);
          else mx[1] = fmaxf(mx[1], m);
        }
      }
      if (tr && tid == 0) tr[1] = globaltimer_ns();
#pragma unroll
      for (int b = 0; b < kQMaxBatch; ++b)
        for (int o = 16; o > 0; o >>= 1) mx[b] = fmaxf(mx[b], __shfl_xor_sync(0xffffffffu, mx[b], o));
      if (lane == 0) {
        sh->amax[warp][0] = mx[0];
        sh->amax[warp][1] = mx[1];
      }
      if (tid < 8) sts128(xs_base + args.xs_bytes - kQZeroBytes + tid * 16, make_uint4(0, 0, 0, 0));
      named_barrier(1, kQConsumerThreads);
      if (tr && tid == 0) tr[2] = globaltimer_ns();
      {
        float m0 = 0.f, m1 = 0.f;
        for (int w = 0; w < kQConsumers; ++w) {
          m0 = fmaxf(m0, sh->amax[w][0]);
          m1 = fmaxf(m1, sh->amax[w][1]);
        }
        ex0 = m0 > 0.f ? 22 - frexp_exponent(m0) : 0;
        ex1 = m1 > 0.f ? 22 - frexp_exponent(m1) : 0;
      }
      const uint32_t colb = static_cast<uint32_t>(xsq_col_bytes(L.KT));
#pragma unroll
      for (int i = 0; i < kXC; ++i) {
        const int c = tid + i * kQConsumerThreads;
        if (c < total) {
          const int b = c / per_row, k = (c - b * per_row) * 8;
          const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};  // outlier rows fixed below
          const float sc = pow2f(b == 0 ? ex0 : ex1);
          uint32_t d[3][2] = {{0, 0}, {0, 0}, {0, 0}};
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const __half hv = __ushort_as_half(static_cast<unsigned short>((wv[t >> 1] >> (16 * (t & 1))) & 0xffffu));
            const int n = round_small_int(__half2float(hv) * sc);
            const int d2 = ((n + 128) & 255) - 128;
            const int n1 = (n - d2) >> 8;
            const int d1 = ((n1 + 128) & 255) - 128;
            const int d0 = (n1 - d1) >> 8;
            d[0][t >> 2] |= (static_cast<uint32_t>(d0) & 0xffu) << (8 * (t & 3));
            d[1][t >> 2] |= (static_cast<uint32_t>(d1) & 0xffu) << (8 * (t & 3));
            d[2][t >> 2] |= (static_cast<uint32_t>(d2) & 0xffu) << (8 * (t & 3));
          }
          const uint32_t pos = static_cast<uint32_t>((k >> 7) * 128 + xs_pos8(k & 127));
#pragma unroll
          for (int dd = 0; dd < 3; ++dd) sts64(xs_base + (3 * b + dd) * colb + pos, d[dd][0], d[dd][1]);
        }
      }
      if (n_pslots > 0) {
        // Outlier rows of the previous layer: one thread per slot overwrites its row's digits
        // (the chunks above converted whatever y held there).
        named_barrier(1, kQConsumerThreads);
        for (int s = tid; s < n_pslots; s += kQConsumerThreads) {
          int row;
          uint32_t hv[kQMaxBatch];
          if (s < kChainPatchMax) {
            row = sh->patch_row[s];
            hv[0] = sh->patch_val[s][0];
            hv[1] = sh->patch_val[s][1];
          } else {
            row = __ldg(P.orow + s);
            hv[0] = __half_as_ushort(prev_outlier_value(P, s, 0, ex_prev[0]));
            hv[1] = B > 1 ? __half_as_ushort(prev_outlier_value(P, s, 1, ex_prev[1])) : 0u;
          }
          if (row < 0 || row >= L.K) continue;
          const uint32_t pos = static_cast<uint32_t>((row >> 7) * 128 + xs_pos8(row & 127));
#pragma unroll
          for (int b = 0; b < kQMaxBatch; ++b) {
            if (b >= B) break;
            const int n = round_small_int(__half2float(__ushort_as_half(static_cast<unsigned short>(hv[b]))) *
                                          pow2f(b ? ex1 : ex0));
            const int d2 = ((n + 128) & 255) - 128;
            const int n1 = (n - d2) >> 8;
            const int d1 = ((n1 + 128) & 255) - 128;
            const int d0 = (n1 - d1) >> 8;
            sts8(xs_base + (3 * b + 0) * colb + pos, static_cast<uint32_t>(d0));
            sts8(xs_base + (3 * b + 1) * colb + pos, static_cast<uint32_t>(d1));
            sts8(xs_base + (3 * b + 2) * colb + pos, static_cast<uint32_t>(d2));
          }
        }
      }
      named_barrier(1, kQConsumerThreads);
    }
    if (tr && tid == 0) tr[3] = globaltimer_ns();

    // ---- this warp's units of layer j
    const int bcol = g >> 2, dig = g & 3;
    const bool live_col = dig < 3 && bcol < B;
    const uint32_t colbase = live_col ? xs_base + (3 * bcol + dig) * xsq_col_bytes(L.KT) : xs_base + args.xs_bytes - kQZeroBytes;
    const uint32_t kts = live_col ? 128u : 0u;
    const uint32_t xq = colbase + 32 * q, xo = colbase + 4 * q;

    // number of packed warps whose ranges share the tile starting at unit sb
    const int32_t tile0 = part.pu0 / (L.KT > 0 ? L.KT : 1);
    auto contrib = [&](int32_t sb) {
      const int32_t n = part.pu1 - part.pu0;
      const int32_t lo = sb - part.pu0, hi = sb + L.KT - 1 - part.pu0;
      return partq_of(hi, n, part.wp) - partq_of(lo, n, part.wp) + 1;
    };
    if (u0 < u1) {
      AccQ A;
      zero_accq(A);
      // outlier segments: add this warp's partial into the slot accumulators
      auto flush_outlier = [&](int32_t seg) {
        long long t[2];
        finish_dot(A, q, t);
        const int b = q >> 1;
        if (!(q & 1) && b < B) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int s = (seg - L.MT) * kTileRows + g + 8 * r;
            if (cur.row[r] >= 0) atomicAdd(L.acc + 2 * s + b, static_cast<unsigned long long>(t[r]));
          }
        }
      };
      while (cc.u < u1) {
        if (!mbar_wait_bounded(fullw + slot * 8, phase)) {
          ok = false;
          break;
        }
        const int32_t cnt = chain_chunk(cc, u1);
        const uint32_t stage = ring + slot * kQChunkBytes;
        const int32_t k0 = cc.u - cc.begin;
        if (cc.seg < L.MT) {
#pragma unroll
          for (int i = 0; i < kQChunkUnits; ++i) {
            if (i < cnt) {
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
          if (cc.seg >= L.MT) {
            flush_outlier(cc.seg);
          } else {
            long long t[2];
            finish_dot(A, q, t);
            if (cc.begin < u0) chain_split_add(sh, qa, cur, t, cc.seg - tile0, contrib(cc.begin), lane, g, q, ex0, ex1);
            else write_outq(qa, cur, t, q, ex0, ex1);
          }
          zero_accq(A);
          chain_next_segment(L, cc);
          cur = nxt;
          if (cc.seg + 1 < L.MT + L.OT) nxt = load_metaq(qa, cc.seg + 1, g);
        }
      }
      if (ok) {
        if (cc.seg >= L.MT) {
          flush_outlier(cc.seg);
        } else {
          long long t[2];
          finish_dot(A, q, t);
          if (cc.begin >= u0 && cc.end <= u1) write_outq(qa, cur, t, q, ex0, ex1);
          else chain_split_add(sh, qa, cur, t, cc.seg - tile0, contrib(cc.begin), lane, g, q, ex0, ex1);
        }
      } else {
        atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
        sh->abort = 1;
      }
    }
    if (tr && tid == 0) tr[4] = globaltimer_ns();
    if (j + 1 < args.n_layers) {
      // For layer j+1: its descriptor, and layer j's static outlier metadata that its staging
      // reads (shared memory is free: layer j's staging is over).  Issued before the write
      // fence, so these loads overlap it.
      if (tid < sizeof(ChainLayer) / 16)
        reinterpret_cast<uint4*>(&sh->layer[(j + 1) & 1])[tid] = ld_nc_v4(reinterpret_cast<const uint4*>(args.layers + j + 1) + tid);
      const int kn = args.layers[j + 1].K;
      if ((kn + 15) / 16 <= kChainMaskMax)
        for (int t = tid; t < (kn + 15) / 16; t += kQConsumerThreads) sh->prev_mask[t] = __ldg(L.tile_mask + t);
      const int ns = L.OT * kTileRows;
      for (int s2 = tid; s2 < ns && s2 < kChainPatchMax; s2 += kQConsumerThreads) {
        sh->patch_row[s2] = __ldg(L.orow + s2);
        sh->patch_exp[s2] = __ldg(L.oexp + s2);
      }
    }
    fence_acq_rel_gpu();                  // this thread's writes of layer j are visible GPU-wide
    if (tr && tid == 0) tr[5] = globaltimer_ns();
    named_barrier(1, kQConsumerThreads);  // ... for every thread of the CTA
    if (sh->abort) ok = false;
    if (tid == 0) {
      if (tr) tr[6] = globaltimer_ns();
      st_relaxed_u32(args.sync + cta, static_cast<uint32_t>(j + 1));  // ordered by the fences above
      if (tr) tr[7] = globaltimer_ns();
    }
    ex_prev[0] = ex0;
    ex_prev[1] = ex1;
  }

  // ---- last layer's outlier rows, once every CTA has finished it
  if (ok && args.n_layers > 0) {
    if (warp == 0 && !poll_flags_warp(args.sync, G, lane, static_cast<uint32_t>(args.n_layers))) {
      if (lane == 0) {
        sh->abort = 1;
        atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
      }
    }
    __threadfence();
    named_barrier(1, kQConsumerThreads);
    if (!sh->abort) {
      const ChainLayer* Lp = args.layers + (args.n_layers - 1);
      PrevInfo P = {};
      P.orow = Lp->orow;
      P.oexp = Lp->oexp;
      P.acc = Lp->acc;
      P.y = Lp->y;
      P.ldy = Lp->ldy;
      const int n_slots = Lp->OT * kTileRows;
      for (int s = cta + G * tid; s < n_slots; s += G * kQConsumerThreads) {
        const int row = __ldg(P.orow + s);
        if (row >= 0) {
          P.y[row] = prev_outlier_value(P, s, 0, ex_prev[0]);
          if (B > 1) P.y[P.ldy + row] = prev_outlier_value(P, s, 1, ex_prev[1]);
        }
      }
    }
  }
}

}  // namespace opc
