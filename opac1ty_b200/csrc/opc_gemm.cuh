// opc_gemm.cuh -- prefill GEMM Y[tok][r] = sum_k X[tok][k] * W_hat[r][k] on the 5th-generation
// tensor cores (tcgen05.mma, fp16 x fp16 -> fp32 in tensor memory).
//
// Reference: kernels/dequant_gemm.metal:34-149 (dequantize a weight tile into threadgroup memory,
// then a scalar multiply-accumulate); semantics opacc1ty/export/converter.py:26-67 + matmul.
//
// Persistent: one CTA per SM walks the output tiles c, c + grid, c + 2 grid, ...  A tile is 128
// weight rows x N tokens (N = 16..256, chosen by the host from the token count and the SM count),
// K in stages of 64 x kSub (kSub 2 for N <= 64: the MMA warp's per-stage cost -- two barrier
// waits, the commit and the loop, ~550 cycles next to ~50 per tcgen05.mma (measured) -- bounds
// small tiles, so their stages carry twice the work).  Roles, all pipelined across tile boundaries:
//   warp 0       TMA (no multicast): the X tile (N tokens x 64 fp16, 128-byte swizzle) per stage
//   warp 22      TMA: the packed units of the tile's 8 row tiles (one 2-D copy of 8 x 512 bytes)
//                per stage into a deeper ring of its own, freed as soon as the stage is decoded
//   warp 1       allocates 2N TMEM columns (two accumulators); one lane issues 4 tcgen05.mma
//                (K = 16 each) per stage, commits each stage to its "empty" mbarrier and each
//                finished tile to its accumulator's "full" mbarrier
//   warps 2..17  decoders, four groups of four warps taking turns by stage (four stages decoded
//                at once): thread = row r decodes the stage's 64 indices of row r through the
//                row's fp16 codebook (PRMT lookups) into the A tile, written in the canonical
//                K-major 128-byte-swizzle layout
//   warps 18..21 epilogue: read a finished accumulator (each warp its TMEM lane quarter),
//                round to fp16 and store Y, then hand the accumulator back -- while the MMAs of
//                the next tile run into the other one
// sub_vector_size 8 (an index selects one of the row's four 8-element fp16 vectors): a chunk of
// 8 columns is one vector, selected from registers.  Outlier rows have all-zero codebooks, so the
// packed tiles compute 0 for them and skip their writes; dense tiles (after the packed ones) compute them from the row-major outlier copy (A
// rows copied instead of decoded) and scatter them to their output rows.
#pragma once

#include <cuda.h>

#include "opc_device.cuh"

namespace opc {

constexpr int kGmM = 128, kGmK = 64;          // weight rows per tile, K per stage
constexpr int kGmDecWarps = 16;               // decoder warps: 4 groups of 4 (one of each group per SM sub-partition)
constexpr int kGmDecGroups = kGmDecWarps / 4; // group i decodes the stages s with s % 4 == i, one row per thread
constexpr int kGmEpiWarps = 4;                // epilogue warps: one TMEM lane quarter each
constexpr int kGmDecWarp0 = 2, kGmEpiWarp0 = kGmDecWarp0 + kGmDecWarps;
constexpr int kGmUnitWarp = kGmEpiWarp0 + kGmEpiWarps;  // the packed units' producer
constexpr int kGmThreads = (kGmUnitWarp + 1) * 32;
constexpr int kGmUStages = 8;                  // packed-units ring (its own barriers, ahead of the A/B ring)
constexpr int kGmABytes = kGmM * kGmK * 2;   // 16 KB
constexpr int kGmUBytes = 8 * kUnitBytes;    // 8 row tiles x one unit
constexpr int kGmMaxSplit = 8;                // K split of a tile into at most this many items
constexpr int kGmPrefetch = 24;               // stages ahead whose packed units are prefetched into L2
constexpr int kGmSmemBudget = 227 * 1024 - 1024 - 512;  // dynamic shared memory less slack and barriers
// Token tile N: x sub-tile N*64 fp16, two accumulators of N fp32 TMEM columns; a stage holds kSub
// sub-tiles of A (128 x 64) and of x (N x 64), each in its own 128-byte-swizzled block.
__host__ __device__ constexpr int gm_b_bytes(int N) { return N * kGmK * 2; }
__host__ __device__ constexpr int gm_stage_bytes(int N, int sub = 1) { return sub * (kGmABytes + gm_b_bytes(N)); }
__host__ __device__ constexpr int gm_stages(int N, int sub = 1) {
  return (kGmSmemBudget - kGmUStages * kGmUBytes) / gm_stage_bytes(N, sub) > 8
             ? 8
             : (kGmSmemBudget - kGmUStages * kGmUBytes) / gm_stage_bytes(N, sub);
}
__host__ __device__ constexpr int gm_tmem_cols(int N) { return 2 * N < 32 ? 32 : 2 * N; }
__host__ __device__ constexpr size_t gm_smem_bytes(int N, int sub = 1) {
  return 1024 /*alignment slack*/ + static_cast<size_t>(gm_stages(N, sub)) * gm_stage_bytes(N, sub) +
         kGmUStages * kGmUBytes + 512;
}

struct GemmArgs {
  const uint8_t* units;        // packed units
  const uint2* cb;             // sub_vector_size 1: [M_pad] split fp16 codebooks
  const uint4* cb8;            // sub_vector_size 8: [MT][32 lanes][2] codebook words (opc_vq8.cuh layout)
  int32_t svs8;                // 1: sub_vector_size 8 layer (128-byte index units of 16 rows x 256 columns)
  const uint16_t* tile_mask;   // [MT]
  const __half* dense;         // [n_slots][K_pad] outlier rows (dense tiles)
  const int32_t* orow;         // [n_slots]
  __half* y;
  int64_t ldy;
  int32_t M, K_pad, MT, KT, n_tok, n_slots;
  int32_t m_tiles;             // packed M tiles; M tile indices >= m_tiles are dense (outlier rows)
  int32_t n_tiles;             // token tiles
  int32_t tiles;               // (m_tiles + dense tiles) * n_tiles
  // split K: every tile is computed as ksplit items of nk_slice stages (the last one shorter); the
  // items' fp32 partials go to part and the last item of a tile to arrive (cnt) adds them in
  // slice order (deterministic), zeroes them and writes y.  ksplit 1: no workspace.
  int32_t ksplit, nk_slice;
  float* part;                 // [tiles][ksplit][128][N] fp32
  int32_t* cnt;                // [tiles][4] arrivals per TMEM lane quarter (zero between calls)
};

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: kind::f16, A = B = fp16, D = fp32, both K-major, M = 128, N tokens.
__host__ __device__ constexpr uint32_t gm_idesc(int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(kGmM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Bring a tile of the tensor map into L2 ahead of its load (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 (or 16) consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t v[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
      "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t v[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Decode 8 indices of one row (fields f0..f7 of w, k offsets 0..7 of the word's group) into 8
// fp16 values in k order.
__device__ __forceinline__ uint4 decode_row8(uint32_t w, uint32_t lo4, uint32_t hi4) {
  uint32_t V[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t t = (w >> (2 * p)) & 0x0303u;  // fields p (bits 0,1) and 4+p (bits 8,9)
    V[p] = prmt(lo4, hi4, t * 0x11u + 0x4040u);    // k offsets p=0:(0,2) 1:(4,6) 2:(1,3) 3:(5,7)
  }
  return make_uint4(prmt(V[0], V[2], 0x5410u), prmt(V[0], V[2], 0x7632u), prmt(V[1], V[3], 0x5410u),
                    prmt(V[1], V[3], 0x7632u));
}

// sub_vector_size 8: word i (0..3) of v
__device__ __forceinline__ uint32_t gm_sel4(const uint4& v, uint32_t i) {
  const uint32_t lo = (i & 1u) ? v.y : v.x;
  const uint32_t hi = (i & 1u) ? v.w : v.z;
  return (i & 2u) ? hi : lo;
}
constexpr int kVq8UnitBytesGm = 128;  // svs-8 index unit: 16 rows x 256 columns x 2 bits

// Offset of (row r, 16-byte chunk c) in a K-major 128-byte-swizzled tile of 64 fp16 per row.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(1024 * (r >> 3) + 128 * (r & 7) + 16 * (c ^ (r & 7)));
}

// tx: x [n_tok][K] fp16, box 64 x N, 128-byte swizzle.  tu: the packed units as a [MT][KT * 512 B]
// array of 8-byte elements, box 512 B x 8 row tiles (one copy brings a k block of all 8 row tiles);
// sub_vector_size 8: [MT][KB * 128 B], box 128 B x 8 row tiles.  td: the row-major outlier rows
// [n_slots][K_pad] fp16, box 64 x 128 rows, 128-byte swizzle (a dense tile's A stage as is).
template <int kN, int kSub>
__global__ void __launch_bounds__(kGmThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tx,
                                                             const __grid_constant__ CUtensorMap tu,
                                                             const __grid_constant__ CUtensorMap td, const GemmArgs a) {
  constexpr int kBBytes = gm_b_bytes(kN);   // one x sub-tile
  constexpr int kS = gm_stages(kN, kSub);
  constexpr int kCols = gm_tmem_cols(kN);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sA = base, sB = sA + kS * kSub * kGmABytes, sU = sB + kS * kSub * kBBytes;
  const uint32_t bars = sU + kGmUStages * kGmUBytes;
  const uint32_t full_b = bars, afull_b = bars + 8 * kS, empty_b = bars + 16 * kS;
  const uint32_t ufull_b = bars + 24 * kS, uempty_b = ufull_b + 8 * kGmUStages;
  const uint32_t accf_b = uempty_b + 8 * kGmUStages, acce_b = accf_b + 16, drain_b = acce_b + 16, tmem_slot = drain_b + 8;
  unsigned char* tmem_slot_ptr = smem_raw + (tmem_slot - raw);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int nk = a.K_pad / (kGmK * kSub);  // stages of a tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(full_b + 8 * s, 1);
      mbar_init(afull_b + 8 * s, 4);  // one arrival per warp of the stage's decoder group
      mbar_init(empty_b + 8 * s, 1);
    }
    for (int u = 0; u < kGmUStages; ++u) {
      mbar_init(ufull_b + 8 * u, 1);
      mbar_init(uempty_b + 8 * u, 4);  // the decoder group of the stage
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_b + 8 * b, 1);
      mbar_init(acce_b + 8 * b, kGmEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain_b, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot), "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- x producer
    if (lane == 0) {
      int g = 0;  // stages issued (all items)
      for (int it = blockIdx.x; it < a.tiles * a.ksplit && ok; it += G) {
        const int i = it / a.ksplit, ks = it - i * a.ksplit;
        const int s0 = ks * a.nk_slice, s1 = min(nk, s0 + a.nk_slice);
        const int n0 = (i % a.n_tiles) * kN;
        for (int s = s0; s < s1; ++s, ++g) {
          const int st = g % kS;
          if (g >= kS && !mbar_wait_bounded(empty_b + 8 * st, ((g / kS) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full_b + 8 * st, kSub * kBBytes);
#pragma unroll
          for (int j = 0; j < kSub; ++j)
            tma_load_2d(sB + (st * kSub + j) * kBBytes, &tx, (s * kSub + j) * kGmK, n0, full_b + 8 * st);
        }
      }
      // copies nobody consumed (a role gave up) land before the CTA exits: wait (bounded) for
      // the last one issued into each stage
      for (int st = 0; st < kS && st < g; ++st) {
        const int last = g - 1 - ((g - 1 - st) % kS);  // last stage counter that used slot st
        mbar_wait_bounded(full_b + 8 * st, (last / kS) & 1);
      }
    }
  } else if (warp == kGmUnitWarp) {
    // ---------------------------------------------------------------- packed-units producer
    // Its ring runs ahead of the A/B stages (a slot is free once its decoder group is done), so a
    // stage's decode waits neither for the x tile nor for the MMAs of the stages before it.
    if (lane == 0) {
      const uint32_t ubytes = a.svs8 ? 8u * kVq8UnitBytesGm : static_cast<uint32_t>(kGmUBytes);
      int gu = 0;  // packed stages issued
      for (int it = blockIdx.x; it < a.tiles * a.ksplit && ok; it += G) {
        const int i = it / a.ksplit, ks = it - i * a.ksplit;
        const int mi = i / a.n_tiles;
        if (mi >= a.m_tiles) continue;  // dense tiles: no units
        const int s0 = ks * a.nk_slice, s1 = min(nk, s0 + a.nk_slice);
        for (int s = s0; s < s1; ++s, ++gu) {
          const int su = gu % kGmUStages;
          if (gu >= kGmUStages && !mbar_wait_bounded(uempty_b + 8 * su, ((gu / kGmUStages) - 1) & 1)) {
            ok = false;
            break;
          }
          // the units kGmPrefetch stages ahead (same item) go to L2 now; one prefetch per k block
          const int sf = s + kGmPrefetch / kSub;
          if (sf < s1 && ((sf * kSub) & (a.svs8 ? 3 : 1)) == 0)
            tma_prefetch_2d(&tu, a.svs8 ? ((sf * kSub) >> 2) * (kVq8UnitBytesGm / 8) : ((sf * kSub) >> 1) * (kUnitBytes / 8),
                            mi * 8);
          // a box past the last row tile is filled with zeros and still counts its full size; x
          // coordinate: the stage's k block in 8-byte elements (512-byte units of 128 columns, or
          // 128-byte svs-8 units of 256 columns: 16-byte aligned either way)
          mbar_expect_tx(ufull_b + 8 * su, ubytes);
          tma_load_2d(sU + su * kGmUBytes, &tu,
                      a.svs8 ? ((s * kSub) >> 2) * (kVq8UnitBytesGm / 8) : ((s * kSub) >> 1) * (kUnitBytes / 8), mi * 8,
                      ufull_b + 8 * su);
        }
      }
      for (int su = 0; su < kGmUStages && su < gu; ++su) {
        const int last = gu - 1 - ((gu - 1 - su) % kGmUStages);
        mbar_wait_bounded(ufull_b + 8 * su, (last / kGmUStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int g = 0, tl = 0;
      for (int it = blockIdx.x; it < a.tiles * a.ksplit && ok; it += G, ++tl) {
        const int ks = it % a.ksplit;
        const int s0 = ks * a.nk_slice, s1 = min(nk, s0 + a.nk_slice);
        const int b = tl & 1;
        // the epilogue has read accumulator b's previous tile
        if (tl >= 2 && !mbar_wait_bounded(acce_b + 8 * b, ((tl >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem + static_cast<uint32_t>(b * kN);
        for (int s = s0; s < s1; ++s, ++g) {
          const int st = g % kS;
          const uint32_t par = (g / kS) & 1;
          if (!mbar_wait_bounded(full_b + 8 * st, par) || !mbar_wait_bounded(afull_b + 8 * st, par)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < kSub; ++j) {
            const uint64_t ad = umma_desc_sw128(sA + (st * kSub + j) * kGmABytes);
            const uint64_t bd = umma_desc_sw128(sB + (st * kSub + j) * kBBytes);
#pragma unroll
            for (int kk = 0; kk < kGmK / 16; ++kk)  // +32 bytes per K = 16 step inside the swizzle atom
              umma_f16(tacc, ad + 2 * kk, bd + 2 * kk, gm_idesc(kN), (s > s0 || j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(empty_b + 8 * st);
        }
        if (!ok) break;
        umma_commit(accf_b + 8 * b);
      }
      // no tensor-core operation of this CTA is in flight past this point
      umma_commit(drain_b);
      mbar_wait_bounded(drain_b, 0);
    }
  } else if (warp < kGmEpiWarp0) {
    // ---------------------------------------------------------------- decoders
    const int d = warp - kGmDecWarp0;
    const int r = 32 * (d & 3) + lane;  // tile row
    const int grp = d >> 2;             // this warp's group: every kGmDecGroups-th stage
    const int tl_row = r >> 4, gl = (r & 15) & 7, hi = (r & 15) >> 3;
    int g = 0, gu = 0;  // stages, and packed stages (the units ring's counter)
    for (int it = blockIdx.x; it < a.tiles * a.ksplit && ok; it += G) {
      const int i = it / a.ksplit, ks = it - i * a.ksplit;
      const int s0 = ks * a.nk_slice, s1 = min(nk, s0 + a.nk_slice);
      const int mi = i / a.n_tiles;
      const bool dense = mi >= a.m_tiles;
      const int R = (dense ? mi - a.m_tiles : mi) * kGmM + r;  // weight row (packed) or outlier slot (dense)
      uint32_t lo4 = 0, hi4 = 0;
      uint4 cv[4];  // sub_vector_size 8: word c of cv[q] = the row's vector c at halves 2q, 2q+1
      bool row_live;
      if (dense) {
        row_live = R < a.n_slots;
      } else {
        row_live = (R >> 4) < a.MT;
        if (row_live && !a.svs8) {
          const uint2 c = __ldg(a.cb + R);
          lo4 = c.x;
          hi4 = c.y;
        }
      }
      if (a.svs8) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          cv[q] = (row_live && !dense) ? __ldg(a.cb8 + (static_cast<int64_t>(R >> 4) * 32 + 4 * gl + q) * 2 + hi)
                                       : make_uint4(0, 0, 0, 0);
      }
      for (int s = s0; s < s1; ++s, ++g) {
        const int gs = dense ? 0 : gu++;          // this stage's place in the units ring
        if ((g % kGmDecGroups) != grp) continue;  // another group's stage
        const int su = gs % kGmUStages;
        const int st = g % kS;
        if (g >= kS && !mbar_wait_bounded(empty_b + 8 * st, ((g / kS) - 1) & 1)) {
          ok = false;
          break;
        }
        const uint32_t dstA0 = sA + st * kSub * kGmABytes;
        if (dense) {
          // the outlier rows' A tile is a plain copy: one TMA in the same 128-byte-swizzled
          // K-major layout, completing on the stage's "A full" barrier (the first warp's
          // arrive.expect_tx is one of the group's four arrivals; rows past the slots read zeros)
          if ((d & 3) == 0) {  // the group's first warp
            if (lane == 0) {
              mbar_expect_tx(afull_b + 8 * st, kSub * kGmABytes);
#pragma unroll
              for (int j = 0; j < kSub; ++j)
                tma_load_2d(dstA0 + j * kGmABytes, &td, (s * kSub + j) * kGmK, (mi - a.m_tiles) * kGmM, afull_b + 8 * st);
            }
          } else if (lane == 0) {
            mbar_arrive(afull_b + 8 * st);
          }
          continue;
        } else {
          if (!mbar_wait_bounded(ufull_b + 8 * su, (gs / kGmUStages) & 1)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < kSub; ++j) {
          const int q64 = s * kSub + j;  // the 64-column sub-stage
          const uint32_t dstA = dstA0 + j * kGmABytes;
          if (a.svs8) {
            // word q64&3 of row pair gl's 16 bytes: byte c/2 = k16 step, bits 2(c&1) + 4hi = the index of
            // chunk c (8 columns = one codebook vector)
            const uint32_t w = row_live ? lds32(sU + su * kGmUBytes + tl_row * kVq8UnitBytesGm + gl * 16 + 4 * (q64 & 3)) : 0u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint32_t i = (w >> (8 * (c >> 1) + 2 * (c & 1) + 4 * hi)) & 3u;
              uint32_t h[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) h[q] = gm_sel4(cv[q], i);
              sts128(dstA + sw128_off(r, c), make_uint4(h[0], h[1], h[2], h[3]));
            }
          } else {
            // chunk c = 4jj + q of the stage (columns 32jj + 8q + 0..7) is in word 2(s&1) + jj of lane 4gl + q
            const uint32_t ub = sU + su * kGmUBytes + tl_row * kUnitBytes + (4 * gl) * 16 + 8 * (q64 & 1);
            uint32_t w[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) w[c] = row_live ? lds32(ub + (c & 3) * 16 + 4 * (c >> 2)) : 0u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 v = make_uint4(0, 0, 0, 0);
              if (row_live) v = decode_row8(hi ? w[c] >> 16 : w[c], lo4, hi4);
              sts128(dstA + sw128_off(r, c), v);
            }
          }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(afull_b + 8 * st);
          if (!dense) mbar_arrive(uempty_b + 8 * su);  // the units slot may be refilled
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;        // TMEM lanes 32*quarter .. +31 (a warp's lane quarter is warp % 4)
    const int r = 32 * quarter + lane;   // tile row = TMEM lane
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    constexpr int kCols = kN < 32 ? kN : 32;  // accumulator columns per tcgen05.ld
    int tl = 0;
    for (int it = blockIdx.x; it < a.tiles * a.ksplit && ok; it += G, ++tl) {
      const int i = it / a.ksplit, ks = it - i * a.ksplit;
      const int mi = i / a.n_tiles, n0 = (i - mi * a.n_tiles) * kN;
      const bool dense = mi >= a.m_tiles;
      const int R = (dense ? mi - a.m_tiles : mi) * kGmM + r;
      int out_row = -1;
      if (dense) {
        if (R < a.n_slots) out_row = __ldg(a.orow + R);
      } else if (R < a.M) {
        const bool outlier = (__ldg(a.tile_mask + (R >> 4)) >> (R & 15)) & 1u;
        out_row = outlier ? -1 : R;
      }
      const int b = tl & 1;
      if (!mbar_wait_bounded(accf_b + 8 * b, (tl >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tacc = trow + static_cast<uint32_t>(b * kN);
      // this item's partial of row r (split K only): fp32, kN consecutive values
      float* prow = a.ksplit > 1 ? a.part + (static_cast<int64_t>(i) * a.ksplit + ks) * (kGmM * kN) +
                                       static_cast<int64_t>(r) * kN
                                 : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < kN / kCols; ++cc) {
        uint32_t v[kCols];
        if constexpr (kCols == 32) tmem_ld32(tacc + cc * 32, v);
        else tmem_ld16(tacc, v);
        if (prow) {
#pragma unroll
          for (int e = 0; e < kCols; e += 4)
            *reinterpret_cast<uint4*>(prow + cc * kCols + e) = make_uint4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        } else if (out_row >= 0) {
#pragma unroll
          for (int e = 0; e < kCols; ++e) {
            const int tok = n0 + cc * kCols + e;
            if (tok < a.n_tok) a.y[static_cast<int64_t>(tok) * a.ldy + out_row] = __float2half_rn(__uint_as_float(v[e]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_b + 8 * b);
      if (prow) {
        // the warp that completes its lane quarter's count for this tile adds the slices in order
        __syncwarp();  // the lanes' partial stores are ordered before lane 0's release below
        int old = 0;
        if (lane == 0) old = atom_add_acq_rel_gpu(a.cnt + 4 * i + quarter, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        __syncwarp();
        if (old == a.ksplit - 1) {
          // The workspace holds zeros between calls outside the GEMV's scratch slots (another
          // layer's counters and accumulators may lie here), so the partials are zeroed as they
          // are read, and the count reset.
          if (lane == 0) a.cnt[4 * i + quarter] = 0;
          float* p0 = a.part + static_cast<int64_t>(i) * a.ksplit * (kGmM * kN) + static_cast<int64_t>(r) * kN;
          // every slice's values of 4 columns are loaded at once (up to kGmMaxSplit in flight),
          // then added in slice order
#pragma unroll 1
          for (int e = 0; e < kN; e += 4) {
            float4 t[kGmMaxSplit];
#pragma unroll
            for (int k2 = 0; k2 < kGmMaxSplit; ++k2)
              if (k2 < a.ksplit) t[k2] = __ldcg(reinterpret_cast<const float4*>(p0 + static_cast<int64_t>(k2) * (kGmM * kN) + e));
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k2 = 0; k2 < kGmMaxSplit; ++k2) {
              if (k2 < a.ksplit) {
                *reinterpret_cast<float4*>(p0 + static_cast<int64_t>(k2) * (kGmM * kN) + e) = make_float4(0.f, 0.f, 0.f, 0.f);
                sum.x += t[k2].x;
                sum.y += t[k2].y;
                sum.z += t[k2].z;
                sum.w += t[k2].w;
              }
            }
            if (out_row >= 0) {
              const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
                if (n0 + e + u < a.n_tok)
                  a.y[static_cast<int64_t>(n0 + e + u) * a.ldy + out_row] = __float2half_rn(vals[u]);
            }
          }
        }
      }
    }
  }
  if (!ok && lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

}  // namespace opc
