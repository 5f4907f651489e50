// opc_coo.cuh -- element-wise (COO) outliers: individual weights kept exactly in fp16 next to the
// 2-bit codebook form, as an epilogue of the GEMV / GEMM and a scatter after the dequant.
//
// The reference keeps outliers as whole rows (opacc1ty/quantize/outlier.py:84-168,
// export/converter.py:59-63) and reserves a "sparse_outlier" layer type for element outliers
// (format/header.py:57-60, quantize/vq.py:103-109) that it never produces.  Here such a layer is
// W_hat = codebook lookup, then W_hat[r][c] = v for each (r, c, v) (the last entry of a repeated
// position wins).  The GEMV computes the codebook part with the regular kernels and then adds,
// per output row r, sum_j delta_j * x[col_j] with delta_j = v_j - codebook value at (r, col_j),
// from a row-compressed (CSR) list built once on the host (opc_coo_build).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace opc {

constexpr int kCooWarps = 8;

// y[b][r] = fp16(y[b][r] + sum_{j in row r} delta[j] * x[b][cols[j]]): one thread per (row, batch
// column), consecutive threads on consecutive rows; the row's entries are summed in CSR order
// (deterministic), four loads in flight.
__global__ void __launch_bounds__(kCooWarps * 32) coo_gemv_kernel(int32_t M, const int32_t* __restrict__ row_ptr,
                                                                  const int32_t* __restrict__ cols,
                                                                  const float* __restrict__ delta,
                                                                  const __half* __restrict__ x, int64_t ldx,
                                                                  __half* __restrict__ y, int64_t ldy, int32_t batch) {
  const int64_t total = static_cast<int64_t>(M) * batch;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t b = static_cast<int32_t>(t / M), r = static_cast<int32_t>(t - static_cast<int64_t>(b) * M);
    const int32_t j0 = row_ptr[r], j1 = row_ptr[r + 1];
    if (j0 == j1) continue;
    const __half* xb = x + static_cast<int64_t>(b) * ldx;
    float s = 0.f;
    int32_t j = j0;
    for (; j + 4 <= j1; j += 4) {
      const int32_t c0 = cols[j], c1 = cols[j + 1], c2 = cols[j + 2], c3 = cols[j + 3];
      const float d0 = delta[j], d1 = delta[j + 1], d2 = delta[j + 2], d3 = delta[j + 3];
      const float x0 = __half2float(xb[c0]), x1 = __half2float(xb[c1]), x2 = __half2float(xb[c2]),
                  x3 = __half2float(xb[c3]);
      s = fmaf(d0, x0, s);
      s = fmaf(d1, x1, s);
      s = fmaf(d2, x2, s);
      s = fmaf(d3, x3, s);
    }
    for (; j < j1; ++j) s = fmaf(delta[j], __half2float(xb[cols[j]]), s);
    __half* yp = y + static_cast<int64_t>(b) * ldy + r;
    *yp = __float2half_rn(__half2float(*yp) + s);
  }
}

// w[r][cols[j]] = values[j] for the CSR entries (positions are unique after opc_coo_build).
__global__ void coo_scatter_kernel(int32_t M, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ cols,
                                   const __half* __restrict__ values, __half* __restrict__ w, int64_t ldw) {
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < M; r += warps)
    for (int32_t j = row_ptr[r] + lane; j < row_ptr[r + 1]; j += 32) w[r * ldw + cols[j]] = values[j];
}

}  // namespace opc
