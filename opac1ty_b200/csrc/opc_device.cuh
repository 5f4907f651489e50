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

// Lane l = 4*g + q of a warp owns, in every packed unit, the 2-bit indices of
//   rows  {16t + g, 16t + g + 8}
//   cols  {128b + 16s + 4q + c : s = 0..7 k-steps, c = 0..3}
// i.e. exactly the weights of its mma.sync m16n8k16 A fragments for the 8 k-steps, under the
// k-permutation  mma column 2q+e -> 4q+e,  mma column 2q+8+e -> 4q+2+e  (e = 0,1).  With that
// permutation the matching B fragment (x) is 4 consecutive fp16 values, one 8-byte load.
//
// Word j (0..3) of the lane's 16 bytes covers k-steps s = 2j (h = 0) and 2j+1 (h = 1).  The
// index of (register r = 0..3, parity h, odd column o) sits at bit 2r + 16h + 8o, where
// register r is the A-fragment register: r&1 selects row g (0) or g+8 (1), r>>1 selects
// columns 4q,4q+1 (0) or 4q+2,4q+3 (1).
__host__ __device__ constexpr int field_shift(int r, int h, int odd) { return 2 * r + 16 * h + 8 * odd; }

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

// Decode one packed word into the A-fragment registers of its two k-steps (parity 0 -> A0,
// parity 1 -> A1).  cbl/cbh: split codebooks of rows g (index 0) and g+8 (index 1).
//
// Field (r, h) pairs sit at bits (2r + 16h, 2r + 16h + 8).  The work is split between the ALU
// pipe (8 PRMT, 4 LOP3, 2 SHF) and the FMA pipe (5 IMAD, 6 HADD2), which issue in parallel:
//   r = 0..2: t = (w >> 2r) & 0x03030303; P = t*0x11 + 0x40404040 holds the parity-0 selector in
//             its low half and the parity-1 selector in its high half; hswz(P) moves the latter.
//   r = 3:    m = w & 0xC0C0C0C0; m*0x4400 + 0x40400000 lifts the (6, 14) pair into the high
//             half (the (22, 30) pair overflows out of 32 bits), hswz brings it down; the
//             (22, 30) pair goes through hswz(m) first.
__device__ __forceinline__ void decode_word(uint32_t w, const uint32_t cbl[2], const uint32_t cbh[2],
                                            uint32_t negz, uint32_t A0[4], uint32_t A1[4]) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const uint32_t t = (w >> (2 * r)) & kFieldMask;
    uint32_t P;
    asm("mad.lo.u32 %0, %1, 17, 1077952576;" : "=r"(P) : "r"(t));  // t*0x11 + 0x40404040
    A0[r] = prmt(cbl[r & 1], cbh[r & 1], P);
    A1[r] = prmt(cbl[r & 1], cbh[r & 1], hswz(P, negz));
  }
  const uint32_t m = w & 0xC0C0C0C0u;
  uint32_t qa, qb;
  asm("mad.lo.u32 %0, %1, 17408, 1077936128;" : "=r"(qa) : "r"(m));  // m*0x4400 + 0x40400000
  const uint32_t mh = hswz(m, negz);
  asm("mad.lo.u32 %0, %1, 17408, 1077936128;" : "=r"(qb) : "r"(mh));
  A0[3] = prmt(cbl[1], cbh[1], hswz(qa, negz));
  A1[3] = prmt(cbl[1], cbh[1], hswz(qb, negz));
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

// Device error word (one per device, lives in the module; the library is one translation
// unit).  Codes:
enum DeviceError : int { kDevErrNone = 0, kDevErrTmaTimeout = 1, kDevErrBadIndex = 2 };
__device__ int g_opc_device_error = 0;

}  // namespace opc
