// opc_gemm.cuh -- prefill GEMM Y[tok][r] = sum_k X[tok][k] * W_hat[r][k] on the 5th-generation
// tensor cores (tcgen05.mma, fp16 x fp16 -> fp32 in tensor memory).
//
// Reference: kernels/dequant_gemm.metal:34-149 (dequantize a weight tile into threadgroup memory,
// then a scalar multiply-accumulate); semantics opacc1ty/export/converter.py:26-67 + matmul.
//
// One CTA computes a 128-row x N-token tile (N = 256, or 128 for small problems), K in stages of 64:
//   warp 0      TMA: the X tile (N tokens x 64 fp16, 128-byte swizzle) and the 8 packed units
//               of the tile's 8 row tiles (bulk copies, no multicast) into the stage
//   warp 1      allocates N TMEM columns; one lane issues 4 tcgen05.mma (K = 16 each) per
//               stage and commits them to the stage's "empty" mbarrier
//   warps 2..5  one weight row per thread: decode the row's 64 indices of the stage through its
//               fp16 codebook (PRMT lookups) into the A tile, written in the canonical K-major
//               128-byte-swizzle layout; after the last stage, read the row's 256 accumulators
//               from TMEM (the warp's TMEM lane quarter) and store Y.
// Outlier rows have all-zero codebooks, so the packed tiles compute 0 for them and skip their
// writes; extra CTAs of the same launch (blockIdx.x >= m_tiles) compute them from the row-major
// outlier copy (A tiles copied instead of decoded) and scatter them to their output rows.
#pragma once

#include <cuda.h>

#include "opc_device.cuh"

namespace opc {

constexpr int kGmM = 128, kGmK = 64;          // weight rows per tile, K per stage
constexpr int kGmStages = 4;
constexpr int kGmThreads = 192;
constexpr int kGmABytes = kGmM * kGmK * 2;   // 16 KB
constexpr int kGmUBytes = 8 * kUnitBytes;    // 8 row tiles x one unit
// Token tile N (256, or 128 when 256-token tiles would leave SMs idle): x stage N*64 fp16,
// N fp32 TMEM columns.
__host__ __device__ constexpr int gm_b_bytes(int N) { return N * kGmK * 2; }
__host__ __device__ constexpr size_t gm_smem_bytes(int N) {
  return 1024 /*alignment slack*/ + kGmStages * (kGmABytes + gm_b_bytes(N) + kGmUBytes) + 256;
}

struct GemmArgs {
  const uint8_t* units;        // packed units
  const uint2* cb;             // [M_pad] split fp16 codebooks
  const uint16_t* tile_mask;   // [MT]
  const __half* dense;         // [n_slots][K_pad] outlier rows (dense mode)
  const int32_t* orow;         // [n_slots]
  __half* y;
  int64_t ldy;
  int32_t M, K_pad, MT, KT, n_tok, n_slots;
  int32_t m_tiles;             // CTAs with blockIdx.x < m_tiles decode packed tiles; the rest copy
                               // outlier rows (dense A tiles)
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

// 32 consecutive fp32 columns of this thread's TMEM lane.
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

// Offset of (row r, 16-byte chunk c) in a K-major 128-byte-swizzled tile of 64 fp16 per row.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(1024 * (r >> 3) + 128 * (r & 7) + 16 * (c ^ (r & 7)));
}

template <int kN>
__global__ void __launch_bounds__(kGmThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tx, const GemmArgs a) {
  const bool kDense = static_cast<int>(blockIdx.x) >= a.m_tiles;
  constexpr int kGmBBytes = gm_b_bytes(kN);
  constexpr int kGmTmemCols = kN;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sA = base, sB = sA + kGmStages * kGmABytes, sU = sB + kGmStages * kGmBBytes;
  const uint32_t bars = sU + kGmStages * kGmUBytes;
  const uint32_t full_b = bars, afull_b = bars + 8 * kGmStages, empty_b = bars + 16 * kGmStages,
                 accf_b = bars + 24 * kGmStages, tmem_slot = accf_b + 8;
  unsigned char* tmem_slot_ptr = smem_raw + (tmem_slot - raw);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int m0 = (kDense ? static_cast<int>(blockIdx.x) - a.m_tiles : static_cast<int>(blockIdx.x)) * kGmM;
  const int n0 = blockIdx.y * kN;
  const int nk = a.K_pad / kGmK;
  const int t0 = m0 / kTileRows;
  const int n_rt = kDense ? 0 : min(8, a.MT - t0);  // row tiles with units in this M tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(full_b + 8 * s, 1);
      mbar_init(afull_b + 8 * s, 4);  // one arrival per decoder warp
      mbar_init(empty_b + 8 * s, 1);
    }
    mbar_init(accf_b, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(kGmTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint32_t bytes = kGmBBytes + static_cast<uint32_t>(n_rt) * kUnitBytes;
      for (int s = 0; s < nk && ok; ++s) {
        const int st = s % kGmStages;
        if (s >= kGmStages && !mbar_wait_bounded(empty_b + 8 * st, ((s / kGmStages) - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_expect_tx(full_b + 8 * st, bytes);
        tma_load_2d(sB + st * kGmBBytes, &tx, s * kGmK, n0, full_b + 8 * st);
        for (int i = 0; i < n_rt; ++i)
          bulk_g2s(sU + st * kGmUBytes + i * kUnitBytes,
                   a.units + (static_cast<int64_t>(t0 + i) * a.KT + (s >> 1)) * kUnitBytes, kUnitBytes,
                   full_b + 8 * st);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      for (int s = 0; s < nk && ok; ++s) {
        const int st = s % kGmStages;
        const uint32_t par = (s / kGmStages) & 1;
        if (!mbar_wait_bounded(full_b + 8 * st, par) || !mbar_wait_bounded(afull_b + 8 * st, par)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(sA + st * kGmABytes), bd = umma_desc_sw128(sB + st * kGmBBytes);
#pragma unroll
        for (int kk = 0; kk < kGmK / 16; ++kk)  // +32 bytes per K = 16 step inside the swizzle atom
          umma_f16(tmem, ad + 2 * kk, bd + 2 * kk, gm_idesc(kN), (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit(empty_b + 8 * st);
      }
      if (ok) umma_commit(accf_b);
    }
  } else {
    // ---------------------------------------------------------------- decoders, then epilogue
    const int quarter = warp & 3;              // TMEM lanes 32*quarter .. +31
    const int r = 32 * quarter + lane;         // tile row = TMEM lane
    const int R = m0 + r;                      // weight row (packed) or outlier slot (dense)
    uint32_t lo4 = 0, hi4 = 0;
    bool row_live = false;
    int out_row = -1;
    if (kDense) {
      row_live = R < a.n_slots;
      out_row = row_live ? __ldg(a.orow + R) : -1;
    } else {
      const int t = R / kTileRows;
      if (t < a.MT) {
        const uint2 c = __ldg(a.cb + R);
        lo4 = c.x;
        hi4 = c.y;
        row_live = true;
        const bool outlier = (__ldg(a.tile_mask + t) >> (R % kTileRows)) & 1u;
        out_row = (R < a.M && !outlier) ? R : -1;
      }
    }
    const int gl = (R % kTileRows) & 7, hi = (R % kTileRows) >> 3, tl = (R / kTileRows) - t0;
    for (int s = 0; s < nk; ++s) {
      const int st = s % kGmStages;
      const uint32_t par = (s / kGmStages) & 1;
      if (s >= kGmStages && !mbar_wait_bounded(empty_b + 8 * st, ((s / kGmStages) - 1) & 1)) {
        ok = false;
        break;
      }
      const uint32_t dstA = sA + st * kGmABytes;
      if (kDense) {
        const __half* src = a.dense + static_cast<int64_t>(R) * a.K_pad + s * kGmK;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = row_live ? __ldg(reinterpret_cast<const uint4*>(src) + c) : make_uint4(0, 0, 0, 0);
          sts128(dstA + sw128_off(r, c), v);
        }
      } else {
        if (!mbar_wait_bounded(full_b + 8 * st, par)) {
          ok = false;
          break;
        }
        // words j = 2(s&1), 2(s&1)+1 of lanes 4gl+q hold this row's k offsets 32(j - 2(s&1)) + 8q + 0..7
        const uint32_t ub = sU + st * kGmUBytes + tl * kUnitBytes + (4 * gl) * 16 + 8 * (s & 1);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (row_live) {
              uint32_t w = lds32(ub + q * 16 + 4 * jj);
              if (hi) w >>= 16;
              v = decode_row8(w, lo4, hi4);
            }
            sts128(dstA + sw128_off(r, 4 * jj + q), v);
          }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull_b + 8 * st);
    }
    // epilogue
    if (ok && mbar_wait_bounded(accf_b, 0)) {
      tc_fence_after();
      const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
#pragma unroll 1
      for (int cc = 0; cc < kN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld32(trow + cc * 32, v);
        if (out_row >= 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int tok = n0 + cc * 32 + i;
            if (tok < a.n_tok) a.y[static_cast<int64_t>(tok) * a.ldy + out_row] = __float2half_rn(__uint_as_float(v[i]));
          }
        }
      }
    } else {
      ok = false;
    }
  }
  if (!ok && lane == 0) atomicCAS(&g_opc_device_error, 0, kDevErrTmaTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGmTmemCols) : "memory");
  }
}

}  // namespace opc
