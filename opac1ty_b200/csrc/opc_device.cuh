// opc_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// the repacked 2-bit layout, the PRMT codebook decode, and thin PTX wrappers
// (mma.sync, bulk async copies, mbarriers, programmatic dependent launch).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace opc {

// ---------------------------------------------------------------------------
// Layout constants (mirrored in include/opc_b200.h, opc_layer_plan).
// ---------------------------------------------------------------------------
constexpr int kUnitBytes = 512;      // one streamed unit
constexpr int kTileRows = 16;        // output rows per tile (mma M)
constexpr int kPackedCols = 128;     // k columns per packed unit (16 rows x 128 x 2 bit)
constexpr int kDenseCols = 16;       // k columns per outlier unit (16 rows x 16 x fp16)
constexpr uint32_t kFieldMask = 0x03030303u;
constexpr int kDenseColsQ = 16;      // k positions per int8 outlier unit (16 rows x 16 x 2 parts)

// Packed index layout (shared by the fp16 and the int8 GEMV):  lane l = 4*g + q of a warp owns,
// in the unit of row tile t and k block b, the 16 bytes [16l, 16l+16): four 32-bit words, word j
// (0..3) covering the 8 columns k = 128b + 32j + 8q + (0..7) of rows 16t+g and 16t+g+8.  Its
// sixteen 2-bit fields f0..f15 (field f at bits 2f, 2f+1) are
//     f(2c)   = row g,   k offset c        f(2c+1) = row g,   k offset 4+c        (c = 0..3)
//     f(8+2c) = row g+8, k offset c        f(9+2c) = row g+8, k offset 4+c
// so that
//   * w & 0x33333333 holds, nibble by nibble, the 4 indices of row g at offsets 0..3 (low half)
//     and of row g+8 (high half); (w >> 2) & 0x33333333 the same for offsets 4..7.  Those are
//     PRMT selectors of four int8 weights each (the int8 decode, decode_word_q);
//   * (w >> 2r) & 0x03030303 holds one index pair of row g in bytes 0,1 and the matching pair of
//     row g+8 in bytes 2,3; one IMAD turns each pair into a PRMT selector of two fp16 weights
//     (the fp16 decode, decode_word).
// Which k each decoded register covers is fixed by these two routines; the kernels stage x in
// shared memory in the matching order (see xs_pos16 / xs_pos8).
__host__ __device__ constexpr int packed_field(int row_hi, int kofs) {
  // field index of (row g + 8*row_hi, k offset kofs in 0..7) within a word
  return 8 * row_hi + 2 * (kofs & 3) + (kofs >> 2);
}

// Positions of k (within its 128-column block) in the staged copies of x.  fp16: the B
// fragments of word j for lane q are the 8 halves at positions 32q + 8j + (0..7), holding
// k offsets (0,2,1,3,4,6,5,7); int8: the 8 bytes at positions 32q + 8j + (0..7) hold k offsets
// 0..7 in order.
__host__ __device__ constexpr int kofs_order16(int i) { return (i == 1 || i == 2 || i == 5 || i == 6) ? (i ^ 3) : i; }
__host__ __device__ constexpr int xs_pos16(int kin) {
  return 32 * ((kin >> 3) & 3) + 8 * ((kin >> 5) & 3) + kofs_order16(kin & 7);
}
__host__ __device__ constexpr int xs_pos8(int kin) { return 32 * ((kin >> 3) & 3) + 8 * ((kin >> 5) & 3) + (kin & 7); }
// Inverses: the k (within the block) staged at a position.
__host__ __device__ constexpr int kin_of_pos16(int p) { return 32 * ((p >> 3) & 3) + 8 * (p >> 5) + kofs_order16(p & 7); }
__host__ __device__ constexpr int kin_of_pos8(int p) { return 32 * ((p >> 3) & 3) + 8 * (p >> 5) + (p & 7); }

// A row's 4 fp16 centroids are held "split": lo4 = the 4 low bytes, hi4 = the 4 high bytes.
// PRMT(lo4, hi4, sel) with selector nibbles (i, i|4, j, j|4) then yields half2(cb[i], cb[j]).
// For an index pair (i, j) at bits (0, 8) of a masked word m that selector is m*0x11 + 0x4040
// in the low 16 bits; PRMT reads only those, so other fields of m never disturb the result.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// Half-word broadcast on the FMA pipe: HADD2 of (hi, hi) with -0.  x + (-0) == x bit for bit
// for every non-NaN fp16 value (signed zeros and subnormals included), and the words this is
// applied to never hold a NaN half (their exponent field is at most 16), so the result is
// exactly (x >> 16) | (x & 0xffff0000).  `negz` must be 0x80008000; it is passed in a register
// so the addition is not folded away.
__device__ __forceinline__ uint32_t hswz(uint32_t x, uint32_t negz) {
  uint32_t d;
  asm("{\n .reg .b16 lo, hi;\n .reg .b32 t;\n mov.b32 {lo, hi}, %1;\n mov.b32 t, {hi, hi};\n"
      " add.rn.f16x2 %0, t, %2;\n}\n"
      : "=r"(d)
      : "r"(x), "r"(negz));
  return d;
}
constexpr uint32_t kNegZero2 = 0x80008000u;

// fp16 decode of one packed word into the A-fragment registers of two m16n8k16 k-steps
// (A0: step 0, A1: step 1).  cbl/cbh: split codebooks of rows g (index 0) and g+8 (index 1).
// Register r of a step is (row g + 8*(r&1), mma columns 2q+8*(r>>1), +1); the pairs used are
//   step 0: r>>1 = 0 -> k offsets (0, 2), r>>1 = 1 -> (1, 3)
//   step 1: r>>1 = 0 -> k offsets (4, 6), r>>1 = 1 -> (5, 7)
// i.e. the B fragment of step 0 is x at offsets (0,2 | 1,3), of step 1 (4,6 | 5,7).
// Pair p = 0..3 = fields (p, 4+p) of row g, bytes 0/1 of (w >> 2p) & 0x03030303, and fields
// (8+p, 12+p) of row g+8 in bytes 2/3.  Work split: ALU 8 PRMT + 4 LOP3 + 2 SHF, FMA 5 IMAD +
// 6 HADD2 (the two pipes issue in parallel):
//   p = 0..2: t = (w >> 2p) & 0x03030303; P = t*0x11 + 0x40404040 holds the row-g selector in
//             its low half and the row-(g+8) selector in its high half; hswz(P) moves the latter.
//   p = 3:    m = w & 0xC0C0C0C0; m*0x4400 + 0x40400000 lifts the (6, 14) pair into the high
//             half (the (22, 30) pair overflows out of 32 bits), hswz brings it down; the
//             (22, 30) pair goes through hswz(m) first.
__device__ __forceinline__ void decode_word(uint32_t w, const uint32_t cbl[2], const uint32_t cbh[2],
                                            uint32_t negz, uint32_t A0[4], uint32_t A1[4]) {
  uint32_t S[4][2];  // [pair][row half] selectors in the low 16 bits
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    const uint32_t t = (w >> (2 * p)) & kFieldMask;
    uint32_t P;
    asm("mad.lo.u32 %0, %1, 17, 1077952576;" : "=r"(P) : "r"(t));  // t*0x11 + 0x40404040
    S[p][0] = P;
    S[p][1] = hswz(P, negz);
  }
  const uint32_t m = w & 0xC0C0C0C0u;
  uint32_t qa, qb;
  asm("mad.lo.u32 %0, %1, 17408, 1077936128;" : "=r"(qa) : "r"(m));  // m*0x4400 + 0x40400000
  const uint32_t mh = hswz(m, negz);
  asm("mad.lo.u32 %0, %1, 17408, 1077936128;" : "=r"(qb) : "r"(mh));
  S[3][0] = hswz(qa, negz);
  S[3][1] = hswz(qb, negz);
  // pair p: k offsets (p=0: 0,2) (p=1: 4,6) (p=2: 1,3) (p=3: 5,7)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    A0[h] = prmt(cbl[h], cbh[h], S[0][h]);
    A0[2 + h] = prmt(cbl[h], cbh[h], S[2][h]);
    A1[h] = prmt(cbl[h], cbh[h], S[1][h]);
    A1[2 + h] = prmt(cbl[h], cbh[h], S[3][h]);
  }
}

// int8 decode of one packed word into the A fragments (4 registers x 4 int8) of one
// m16n8k32 step, for the two 8-bit parts of the rows' integer codebooks:
//   qh/ql[0]: row g (4 int8 centroids), qh/ql[1]: row g+8.
// Register r: row g + 8*(r&1), mma columns 4q + 16*(r>>1) + (0..3) = k offsets 4*(r>>1) + (0..3).
// ALU: 8 PRMT + 2 LOP3 + 1 SHF; FMA: 2 HADD2.  PRMT(a, a, s) reads each selector nibble's low
// 3 bits; the masks leave bit 3 clear and bit 2 only selects the second copy of a.
__device__ __forceinline__ void decode_word_q(uint32_t w, const uint32_t qh[2], const uint32_t ql[2], uint32_t negz,
                                              uint32_t Ah[4], uint32_t Al[4]) {
  const uint32_t s0 = w & 0x33333333u;
  const uint32_t s2 = (w >> 2) & 0x33333333u;
  const uint32_t s1 = hswz(s0, negz);
  const uint32_t s3 = hswz(s2, negz);
  Ah[0] = prmt(qh[0], qh[0], s0);
  Ah[1] = prmt(qh[1], qh[1], s1);
  Ah[2] = prmt(qh[0], qh[0], s2);
  Ah[3] = prmt(qh[1], qh[1], s3);
  Al[0] = prmt(ql[0], ql[0], s0);
  Al[1] = prmt(ql[1], ql[1], s1);
  Al[2] = prmt(ql[0], ql[0], s2);
  Al[3] = prmt(ql[1], ql[1], s3);
}

// ---------------------------------------------------------------------------
// Tensor cores: legacy-warp MMA, fp16 x fp16 -> fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  float d0, d1, d2, d3;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d0), "=f"(d1), "=f"(d2), "=f"(d3)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
  c[0] = d0; c[1] = d1; c[2] = d2; c[3] = d3;
}
// int8 (A, signed) x uint8 (B, unsigned) -> int32 (exact).  m16n8k32: A 4 regs (row g / g+8,
// k 4q.., 16+4q..), B 2 regs.
__device__ __forceinline__ void imma16832(int32_t c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// m16n8k16, A signed, B unsigned: A 2 regs (row g / g+8, k 4q..4q+3), B 1 reg.
__device__ __forceinline__ void imma16816(int32_t c[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// ---------------------------------------------------------------------------
// Shared memory, bulk async copies and mbarriers (sm_90+ PTX).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts64(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void sts8(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// One contiguous global -> shared copy performed by the TMA unit (no multicast).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Non-blocking completion test of the given phase parity.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same copy with an L2 cache-policy operand (e.g. evict-first for data read exactly once).
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Bring [src, src+bytes) into L2 ahead of use (bytes a multiple of 16, src 16-byte aligned).
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Arrival count with acquire-release semantics at GPU scope: releases the caller's (and, through
// a preceding __syncwarp, its warp's) earlier writes and acquires those released by earlier
// arrivals -- one atomic instead of a fence on each side of a relaxed one.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Every wait in this library is bounded: after kWaitLimitNs the caller records an error in
// the device error word and gives up instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Programmatic dependent launch (sm_90+): let the next kernel on the stream start its
// prologue, and wait for the previous one's memory before touching its outputs.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `threads` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void nanosleep_ns(uint32_t ns) { asm volatile("nanosleep.u32 %0;" ::"r"(ns)); }

// Global loads the compiler may not re-issue: under register pressure it may otherwise
// rematerialize a load instead of keeping its value live, putting a fresh L2 round trip on a
// latency-critical path.  .cg: L2 only (data written by other SMs); .nc: read-only data.
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint64_t ld_nc_u64(const void* p) {
  uint64_t v;
  asm volatile("ld.global.nc.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_nc_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_nc_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Binary exponent e of a finite normal float m > 0 with m = f * 2^e, f in [0.5, 1) (the frexp
// convention), from its bits; no address-taken output argument, so nothing goes to local memory.
__device__ __forceinline__ int frexp_exponent(float m) { return ((__float_as_int(m) >> 23) & 0xff) - 126; }


// Device error word (one per device, lives in the module; the library is one translation
// unit).  Codes:
//   1  a ring / shared-memory barrier wait gave up
//   2  an index out of range was skipped
//   3  a grid or cross-rank barrier of the decode chain gave up (a CTA or rank did not arrive)
//   4  a decode chain launch found the chain poisoned by an earlier failed launch
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrTmaTimeout = 1,
  kDevErrBadIndex = 2,
  kDevErrBarrierTimeout = 3,
  kDevErrChainPoisoned = 4
};
__device__ int g_opc_device_error = 0;

}  // namespace opc
