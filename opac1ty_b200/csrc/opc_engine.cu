// opc_engine.cu -- the bf_engine_* C API (include/opc_engine.h): a Llama-style decoder over the
// fused dequant library.  The reference declares the same calls (runtime/include/opacc1ty.h:69-212)
// and implements them as stubs (runtime/src/inference.c:183-245, bf2_format.c:131-314); this file
// loads a .bf2 model onto the GPU and runs it.  Projections go through the library's public C ABI
// (opc_repack_layer, opc_gemv, opc_dequant); the small per-token operations (RMSNorm, rotary
// embedding, attention over the KV cache, SiLU gating, residual adds) are the kernels below.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "opc_b200.h"
#include "opc_engine.h"

extern "C" const BFSamplingParams BF_DEFAULT_SAMPLING = {1.0f, 0.0f, 0, 1.0f, 0u};

namespace {

constexpr uint32_t kChunk = 512;         // tokens per prompt chunk
constexpr int kGemvMaxBatch = 64;        // opc_gemv's largest batch; larger chunks call opc_gemm
constexpr uint32_t kDefaultContext = 4096;
constexpr int kAttnThreads = 128;        // attention_kernel: threads per CTA
constexpr int kAttnTile = 256;           // attention_kernel: positions per tile
constexpr int kAttnSplits = 16;          // attention_kernel: at most this many context ranges per (head, token)
constexpr int kAttnMinCtas = 512;        // attention_kernel: CTAs a launch should have when the context allows
constexpr int kNormThreads = 512;        // add_rmsnorm_kernel: one CTA per token
constexpr int kNormPer = 16;             // values per thread held in registers (rows up to 8192)
constexpr int kRopeSplit = 4;            // rope_cache_kernel: CTAs per token
constexpr int kMaxHeadDim = 256;

// ------------------------------------------------------------------------------------------------
// .bf2 file (opacc1ty/format/header.py:63-178, bf2.py:78-150): "BF2\0", u32 version, u32 flags,
// u32 model-JSON length twice, JSON, u32 quantize-JSON length, JSON, u32 layer count, then per
// layer a 64-byte header "<H B I I I B B H Q Q Q Q 13s", the name, and the payload.
// ------------------------------------------------------------------------------------------------
constexpr int kLayerHeader = 64;
constexpr uint8_t kQuantized = 0, kSparse = 1, kPassthrough = 2;  // kSparse: element-wise (COO) outliers

struct FileLayer {
  std::string name;
  uint8_t type = 0;
  uint32_t out_f = 0, in_f = 0, n_groups = 0;
  uint8_t entries = 0, svs = 0;
  uint16_t n_out = 0;
  uint64_t nnz = 0;     // kSparse: entries (u64 in the first reserved bytes)
  size_t data = 0;      // file offset of the payload (after header and name)
  int id_bytes = 4;     // outlier id width (the reference's own files carry int64)
};

template <typename T>
T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

// Payload bytes of a layer as its header describes it; SIZE_MAX when the fields describe more
// than any file can hold (the sums are formed in 128 bits, so no header value wraps them around).
size_t payload_bytes(const FileLayer& l, int id_bytes) {
  using u128 = unsigned __int128;
  u128 n = 0;
  if (l.type == kSparse) {  // codebooks, indices, values [nnz] fp16, positions [nnz][2] int32
    n = static_cast<u128>(l.n_groups) * l.entries * l.svs * 2 +
        (l.svs ? static_cast<u128>(l.n_groups) * (l.in_f / l.svs) : 0) + static_cast<u128>(l.nnz) * 10;
  } else if (l.type == kQuantized) {
    n = static_cast<u128>(l.n_groups) * l.entries * l.svs * 2;
    if (l.svs) n += static_cast<u128>(l.n_groups) * (l.in_f / l.svs);
    if (l.n_out) n += static_cast<u128>(l.n_out) * l.in_f * 2 + static_cast<u128>(l.n_out) * id_bytes;
  } else if (l.type == kPassthrough) {
    n = static_cast<u128>(l.out_f) * l.in_f * 2;
  }
  return n >= static_cast<u128>(SIZE_MAX) ? SIZE_MAX : static_cast<size_t>(n);
}

// Parse the layer header at `pos` (false when it is not a plausible header).
bool parse_layer_at(const uint8_t* base, size_t size, size_t pos, FileLayer* out) {
  if (pos > size || size - pos < kLayerHeader) return false;
  const uint8_t* h = base + pos;
  FileLayer l;
  const uint16_t nlen = rd<uint16_t>(h);
  l.type = h[2];
  l.out_f = rd<uint32_t>(h + 3);
  l.in_f = rd<uint32_t>(h + 7);
  l.n_groups = rd<uint32_t>(h + 11);
  l.entries = h[15];
  l.svs = h[16];
  l.n_out = rd<uint16_t>(h + 17);
  l.nnz = l.type == kSparse ? rd<uint64_t>(h + 51) : 0;
  if (nlen == 0 || l.type > 2 || size - pos - kLayerHeader < nlen) return false;
  if (l.out_f > 0x7fffffffu || l.in_f > 0x7fffffffu || l.n_groups > 0x7fffffffu) return false;
  l.name.assign(reinterpret_cast<const char*>(h + kLayerHeader), nlen);
  l.data = pos + kLayerHeader + nlen;
  *out = l;
  return true;
}

// Value of "key" in a flat JSON object: a number (true) or, with `str`, a string.
bool json_number(const std::string& js, const char* key, double* v) {
  const std::string k = std::string("\"") + key + "\"";
  size_t p = js.find(k);
  if (p == std::string::npos) return false;
  p = js.find(':', p + k.size());
  if (p == std::string::npos) return false;
  const char* s = js.c_str() + p + 1;
  while (*s == ' ' || *s == '\t' || *s == '\n' || *s == '\r') ++s;
  char* end = nullptr;
  const double d = std::strtod(s, &end);
  if (end == s) return false;
  *v = d;
  return true;
}
bool json_string(const std::string& js, const char* key, std::string* v) {
  const std::string k = std::string("\"") + key + "\"";
  size_t p = js.find(k);
  if (p == std::string::npos) return false;
  p = js.find(':', p + k.size());
  if (p == std::string::npos) return false;
  p = js.find('"', p);
  if (p == std::string::npos) return false;
  const size_t e = js.find('"', p + 1);
  if (e == std::string::npos) return false;
  *v = js.substr(p + 1, e - p - 1);
  return true;
}

// ------------------------------------------------------------------------------------------------
// Kernels.  Rows are tokens of the current chunk; the residual stream h is fp32 [n][hidden].
// ------------------------------------------------------------------------------------------------
// Programmatic dependent launch: the kernels below (but the first of a chunk) are launched with
// programmatic stream serialization (launch_pdl), so each may be resident before the previous
// kernel of the stream has finished.  Each waits for that kernel's completion (griddepcontrol.wait)
// before it touches any buffer and only then lets the next kernel launch
// (griddepcontrol.launch_dependents); the next kernel's prologue -- a GEMV's weight prefetch --
// then overlaps this one.  The library's GEMV kernels also wait before reading x, and a kernel
// completes only after its wait has returned, so every kernel still sees all earlier results.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// The chunk's tokens and first position live in device memory ([kChunk] tokens, then the position),
// copied from pinned host memory at the start of every chunk, so that a captured decode step
// (CUDA graph) replays with new values.  Launched plainly (it follows that copy).
__global__ void embed_kernel(const __half* __restrict__ table, int hidden, const int32_t* __restrict__ tokpos,
                             float* __restrict__ h) {
  pdl_begin();
  const int r = blockIdx.x;
  const __half* src = table + static_cast<int64_t>(tokpos[r]) * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) h[static_cast<int64_t>(r) * hidden + i] = __half2float(src[i]);
}

__device__ float block_sum(float v) {
  __shared__ float part[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) part[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += part[i];
  __syncthreads();
  return s;
}

// Residual add fused with the RMSNorm that follows it.  Row r = row0 + blockIdx.x: with kAdd,
// h[r][i] += y[r][i] (fp32, written back); then
// out[blockIdx.x][i] = fp16(w[i] * h[r][i] / sqrt(mean_i h[r][i]^2 + eps)), without kW w = ones
// (LlamaRMSNorm: the statistics in fp32, the scaled value times the weight).  A row of up to
// kNormPer * blockDim.x values is held in registers, all of its loads (h, y and w) in flight at
// once; longer rows take a loop in which each thread reads back only the elements it wrote.
template <bool kAdd, bool kW>
__global__ void add_rmsnorm_kernel(float* __restrict__ h, int hidden, const __half* __restrict__ y, int ldy,
                                   int row0, const __half* __restrict__ w, float eps, __half* __restrict__ out,
                                   int ldo) {
  pdl_begin();
  const int r = row0 + static_cast<int>(blockIdx.x);
  float* x = h + static_cast<int64_t>(r) * hidden;
  const __half* yr = kAdd ? y + static_cast<int64_t>(r) * ldy : nullptr;
  __half* o = out + static_cast<int64_t>(blockIdx.x) * ldo;
  const int nt = blockDim.x;
  float ss = 0.f;
  if (hidden <= kNormPer * nt) {
    float v[kNormPer], t[kNormPer], wv[kNormPer];
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
      const int i = threadIdx.x + j * nt;
      const bool in = i < hidden;
      v[j] = in ? x[i] : 0.f;
      if (kAdd) t[j] = in ? __half2float(yr[i]) : 0.f;
      if (kW) wv[j] = in ? __half2float(w[i]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
      const int i = threadIdx.x + j * nt;
      if (kAdd) {
        v[j] += t[j];
        if (i < hidden) x[i] = v[j];
      }
      ss += v[j] * v[j];
    }
    const float inv = rsqrtf(block_sum(ss) / static_cast<float>(hidden) + eps);
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
      const int i = threadIdx.x + j * nt;
      if (i < hidden) o[i] = __float2half_rn(kW ? wv[j] * (v[j] * inv) : v[j] * inv);
    }
    return;
  }
  for (int i = threadIdx.x; i < hidden; i += nt) {
    const float v = kAdd ? x[i] + __half2float(yr[i]) : x[i];
    if (kAdd) x[i] = v;
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum(ss) / static_cast<float>(hidden) + eps);
  for (int i = threadIdx.x; i < hidden; i += nt) {
    const float v = x[i] * inv;
    o[i] = __float2half_rn(kW ? __half2float(w[i]) * v : v);
  }
}

// Rotary embedding (rotate-half pairing: dims i and i + hd/2 of a head, angle
// pos * theta^(-2i/hd)) on q in place and on k, then k and v appended to the layer's cache
// [kv_heads][ctx][hd] at position pos0 + r.  Token r = blockIdx.x; blockIdx.y splits its pairs.
__global__ void rope_cache_kernel(__half* __restrict__ q, int ldq, const __half* __restrict__ k,
                                  const __half* __restrict__ v, int ldkv, int heads, int kv_heads, int hd,
                                  const int32_t* __restrict__ pos0p, float theta, __half* __restrict__ kc,
                                  __half* __restrict__ vc, int ctx) {
  pdl_begin();
  const int r = blockIdx.x;
  const int pos = *pos0p + r;
  const int half = hd / 2;
  const int nq = heads * half, nk = kv_heads * half;
  const int t0 = blockIdx.y * blockDim.x + threadIdx.x, dt = gridDim.y * blockDim.x;
  for (int i = t0; i < nq + nk; i += dt) {
    const bool isq = i < nq;
    const int j = isq ? i : i - nq;
    const int head = j / half, d = j - head * half;
    const float inv_freq = powf(theta, -2.0f * static_cast<float>(d) / static_cast<float>(hd));
    float s, c;
    sincosf(static_cast<float>(pos) * inv_freq, &s, &c);
    const __half* src = isq ? q + static_cast<int64_t>(r) * ldq : k + static_cast<int64_t>(r) * ldkv;
    const float x0 = __half2float(src[head * hd + d]), x1 = __half2float(src[head * hd + d + half]);
    const __half y0 = __float2half_rn(x0 * c - x1 * s), y1 = __float2half_rn(x1 * c + x0 * s);
    if (isq) {
      q[static_cast<int64_t>(r) * ldq + head * hd + d] = y0;
      q[static_cast<int64_t>(r) * ldq + head * hd + d + half] = y1;
    } else {
      __half* dst = kc + (static_cast<int64_t>(head) * ctx + pos) * hd;
      dst[d] = y0;
      dst[d + half] = y1;
    }
  }
  for (int i = t0; i < kv_heads * hd; i += dt) {
    const int head = i / hd, d = i - head * hd;
    vc[(static_cast<int64_t>(head) * ctx + pos) * hd + d] = v[static_cast<int64_t>(r) * ldkv + i];
  }
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ void unpack8(const uint4& raw, float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xffffu)));
    f[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
  }
}

// Causal grouped-query attention of token r = blockIdx.y (position pos0 + r) for query head
// blockIdx.x: softmax(q.k / sqrt(hd)) . v over cache positions 0..pos0+r.  The positions are split
// into gridDim.z equal ranges (split z = blockIdx.z) so that long contexts spread over many SMs.
// A CTA walks its range in tiles of kAttnTile positions, with a running max M and sum T:
//   scores: thread j takes positions j, j + kAttnThreads, ... (a full dot product each, its k row
//           read with 16-byte loads, q from shared memory);
//   weights: the tile's max updates M (earlier sums rescaled), w = exp(score - M);
//   values: thread (g, c) adds w * v over positions g, g + G, ... for dims [8c, 8c + 8) (a warp
//           reads whole rows of v), the G position groups summed at the end.
// Every load of a phase is independent of the others, so they are in flight together.  The CTA
// writes its record (M, T, unnormalised sums) to part[r][head][z]; the CTA that completes
// count[r][head] (one atomic per CTA after a fence) merges the ranges' records, writes the output
// and sets the count back to 0 for the next launch.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __half* __restrict__ q, int ldq,
                                                                 const __half* __restrict__ kc,
                                                                 const __half* __restrict__ vc, int heads,
                                                                 int kv_heads, int hd, int ctx,
                                                                 const int32_t* __restrict__ pos0p,
                                                                 __half* __restrict__ out, int ldo,
                                                                 float* __restrict__ part, int* __restrict__ count) {
  __shared__ float sq[kMaxHeadDim];
  __shared__ float sp[kAttnTile];
  __shared__ float red[kAttnThreads / 32];
  __shared__ float sacc[kAttnThreads * 8];  // [G][hd]: G * hd <= 8 * kAttnThreads
  __shared__ int sm_last;
  pdl_begin();
  const int head = blockIdx.x, r = blockIdx.y, z = blockIdx.z, S = gridDim.z;
  const int tid = threadIdx.x;
  const int kvh = head / (heads / kv_heads);
  const int L = *pos0p + r + 1;
  const int per = (L + S - 1) / S;
  const int pb = min(L, z * per), pe = min(L, pb + per);
  const float scale = rsqrtf(static_cast<float>(hd));
  for (int d = tid; d < hd; d += kAttnThreads) sq[d] = __half2float(q[static_cast<int64_t>(r) * ldq + head * hd + d]) * scale;
  const __half* kb = kc + static_cast<int64_t>(kvh) * ctx * hd;
  const __half* vb = vc + static_cast<int64_t>(kvh) * ctx * hd;
  const int nc = hd / 8;               // 16-byte chunks per row
  const int G = kAttnThreads / nc;     // position groups of the values phase
  const int c = tid % nc, g = tid / nc;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float M = -INFINITY, T = 0.f;
  __syncthreads();
  for (int t0 = pb; t0 < pe; t0 += kAttnTile) {
    const int tn = min(kAttnTile, pe - t0);
    for (int j = tid; j < tn; j += kAttnThreads) {
      const uint4* kp = reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(t0 + j) * hd);
      float dot = 0.f;
#pragma unroll 8
      for (int cc = 0; cc < nc; ++cc) {
        float f[8];
        unpack8(kp[cc], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += sq[8 * cc + i] * f[i];
      }
      sp[j] = dot;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = tid; j < tn; j += kAttnThreads) mx = fmaxf(mx, sp[j]);
    const float Mn = fmaxf(M, block_max(mx, red));
    const float corr = expf(M - Mn);
    float ts = 0.f;
    for (int j = tid; j < tn; j += kAttnThreads) {
      const float w = expf(sp[j] - Mn);
      sp[j] = w;
      ts += w;
    }
    T = T * corr + block_sum(ts);  // its barriers also publish the weights
    M = Mn;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= corr;
    if (g < G) {
#pragma unroll 4
      for (int j = g; j < tn; j += G) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(t0 + j) * hd + 8 * c), f);
        const float w = sp[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += w * f[i];
      }
    }
    __syncthreads();  // the next tile overwrites sp
  }
  if (g < G) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[g * hd + 8 * c + i] = acc[i];
  }
  __syncthreads();
  __half* orow = out + static_cast<int64_t>(r) * ldo + head * hd;
  if (S == 1) {
    for (int d = tid; d < hd; d += kAttnThreads) {
      float o = 0.f;
      for (int gg = 0; gg < G; ++gg) o += sacc[gg * hd + d];
      orow[d] = __float2half_rn(o / T);
    }
    return;
  }
  const int rec = hd + 2;
  float* mine = part + ((static_cast<int64_t>(r) * heads + head) * S + z) * rec;
  for (int d = tid; d < hd; d += kAttnThreads) {
    float o = 0.f;
    for (int gg = 0; gg < G; ++gg) o += sacc[gg * hd + d];
    mine[2 + d] = o;
  }
  if (tid == 0) {
    mine[0] = M;  // -inf for an empty range
    mine[1] = T;
  }
  __threadfence();
  __syncthreads();
  int* cnt = count + static_cast<int64_t>(r) * heads + head;
  if (tid == 0) sm_last = atomicAdd(cnt, 1) == S - 1;
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
  const float* all = part + (static_cast<int64_t>(r) * heads + head) * S * rec;
  float MM = -INFINITY;
  for (int j = 0; j < S; ++j) MM = fmaxf(MM, __ldcg(all + j * rec));
  float TT = 0.f;
  for (int j = 0; j < S; ++j) {
    const float mj = __ldcg(all + j * rec);
    if (mj != -INFINITY) TT += __ldcg(all + j * rec + 1) * expf(mj - MM);
  }
  for (int d = tid; d < hd; d += kAttnThreads) {
    float o = 0.f;
    for (int j = 0; j < S; ++j) {
      const float mj = __ldcg(all + j * rec);
      if (mj != -INFINITY) o += __ldcg(all + j * rec + 2 + d) * expf(mj - MM);
    }
    orow[d] = __float2half_rn(o / TT);
  }
  if (tid == 0) *cnt = 0;
}

// a[r][i] = fp16(silu(g[r][i]) * u[r][i]), silu(g) = g / (1 + exp(-g)), for rows < rows and
// i < n: one thread per element over the whole grid.
__global__ void silu_mul_kernel(const __half* __restrict__ g, const __half* __restrict__ u, int ldg, int n, int rows,
                                __half* __restrict__ a, int lda) {
  pdl_begin();
  const int64_t total = static_cast<int64_t>(rows) * n;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(t / n), i = static_cast<int>(t - static_cast<int64_t>(r) * n);
    const float gv = __half2float(g[static_cast<int64_t>(r) * ldg + i]), uv = __half2float(u[static_cast<int64_t>(r) * ldg + i]);
    a[static_cast<int64_t>(r) * lda + i] = __float2half_rn(gv / (1.0f + expf(-gv)) * uv);
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// Engine state
// ------------------------------------------------------------------------------------------------
namespace {

struct DevLayer {
  opc_layer L{};
  bool present = false;
  // element-wise outliers (kSparse layers), row-compressed by opc_coo_build
  int64_t nnz = 0;
  int32_t *row_ptr = nullptr, *cols = nullptr;
  float* delta = nullptr;
  __half* values = nullptr;
};

struct Block {
  DevLayer q, k, v, o, gate, up, down;
  DevLayer qkv, gu;               // q|k|v and gate|up as one layer each (rows stacked) when fusable
  const __half* ln_in = nullptr;    // device; NULL = ones
  const __half* ln_post = nullptr;
};

int pad8(int v) { return (v + 7) & ~7; }

// The next-token logits come back from the device as fp16 and are widened to fp32 on the host
// every step (32000 to 128256 values).  One value at a time, from the IEEE-754 binary16 layout:
// sign, 5-bit exponent (bias 15), 10-bit fraction; exact (every binary16 value is a binary32 one).
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16, ex = (h >> 10) & 0x1fu, fr = h & 0x3ffu;
  uint32_t bits;
  if (ex == 0x1fu) {
    bits = sign | 0x7f800000u | (fr << 13);  // infinities and NaNs (payload kept)
  } else if (ex != 0) {
    bits = sign | ((ex + 112u) << 23) | (fr << 13);  // normal: rebias 15 -> 127
  } else if (fr == 0) {
    bits = sign;  // signed zero
  } else {  // subnormal fr * 2^-24: normalise around its leading bit p
    const int p = 31 - __builtin_clz(fr);
    bits = sign | (static_cast<uint32_t>(p + 103) << 23) | ((fr << (23 - p)) & 0x7fffffu);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

#if defined(__x86_64__)
// Eight values per instruction with the x86 F16C conversion (same results: exact widening).
__attribute__((target("avx,f16c"))) void halves_to_floats_f16c(const uint16_t* h, float* f, size_t n) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    _mm256_storeu_ps(f + i, _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(h + i))));
  for (; i < n; ++i) f[i] = half_bits_to_float(h[i]);
}
#endif

void halves_to_floats(const __half* h, float* f, size_t n) {
  const uint16_t* b = reinterpret_cast<const uint16_t*>(h);
#if defined(__x86_64__)
  static const bool f16c = __builtin_cpu_supports("f16c") && __builtin_cpu_supports("avx");
  if (f16c) {
    halves_to_floats_f16c(b, f, n);
    return;
  }
#endif
  for (size_t i = 0; i < n; ++i) f[i] = half_bits_to_float(b[i]);
}

// Context ranges per (head, token) of an attention launch over n tokens: enough CTAs to cover the
// SMs a few times (a decode step: kAttnSplits per head), one range per CTA for long prompt chunks.
int attention_splits(int n, int heads) {
  const int want = (kAttnMinCtas + n * heads - 1) / (n * heads);
  return std::max(1, std::min(kAttnSplits, want));
}

}  // namespace

struct BFEngine {
  std::string error;
  BFModelConfig cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  float eps = 1e-5f;
  uint32_t ctx = 0, pos = 0;
  int hidden = 0, heads = 0, kv_heads = 0, hd = 0, inter = 0, vocab = 0, n_layers = 0;
  std::vector<Block> blocks;
  DevLayer embed, lm_head;
  bool lm_from_embed = false;
  __half* embed_table = nullptr;
  const __half* final_norm = nullptr;
  __half *kcache = nullptr, *vcache = nullptr;
  size_t kv_bytes = 0;
  // per-chunk scratch, kChunk rows each
  float* h = nullptr;
  __half *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *y = nullptr, *g = nullptr,
         *u = nullptr, *a = nullptr, *logits16 = nullptr, *qkv = nullptr, *gu = nullptr;
  int ld_x = 0, ld_q = 0, ld_kv = 0, ld_i = 0, ld_y = 0, ld_qkv = 0, ld_gu = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  float* att_part = nullptr;      // attention: per (token, head, context range) records of hd + 2 floats
  int* att_count = nullptr;       // attention: ranges finished per (token, head); 0 between launches
  __half* host_logits = nullptr;  // pinned
  int32_t* d_tokpos = nullptr;    // [kChunk] tokens, then the chunk's first position
  int32_t* h_tokpos = nullptr;    // pinned mirror
  cudaGraphExec_t step_exec = nullptr;  // the captured one-token step (tokens and position from d_tokpos)
  bool graph_tried = false;
  uint32_t step_launches = 0;
  uint32_t direct_steps = 0;  // one-token steps launched directly (the first one sets up the kernels)
  std::vector<void*> allocs;
  size_t dev_bytes = 0;
  std::vector<int32_t> history;   // tokens in the cache (repetition penalty)
  BFStats stats{};
};

namespace {

int fail(BFEngine* e, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  e->error = buf;
  return -1;
}

#define ENG_CUDA(e, call)                                                                     \
  do {                                                                                        \
    cudaError_t _r = (call);                                                                  \
    if (_r != cudaSuccess) return fail((e), "%s: %s", #call, cudaGetErrorString(_r));          \
  } while (0)

#define ENG_OPC(e, call)                                                                      \
  do {                                                                                        \
    if ((call) != OPC_OK) return fail((e), "%s: %s", #call, opc_last_error());                \
  } while (0)

int dalloc(BFEngine* e, void** p, size_t bytes) {
  *p = nullptr;
  if (bytes == 0) bytes = 16;
  ENG_CUDA(e, cudaMalloc(p, bytes));
  e->allocs.push_back(*p);
  e->dev_bytes += bytes;
  return 0;
}

// The .bf2 file, memory-mapped for the duration of bf_engine_create.
struct MappedFile {
  int fd = -1;
  const uint8_t* p = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (p) munmap(const_cast<uint8_t*>(p), size);
    if (fd >= 0) close(fd);
  }
};

struct Model {
  std::string model_json;
  std::map<std::string, FileLayer> layers;
};

int parse_file(BFEngine* e, const MappedFile& f, Model* m) {
  const uint8_t* b = f.p;
  const size_t size = f.size;
  if (size < 4 || std::memcmp(b, "BF2\0", 4) != 0) return fail(e, "Not a valid BF2 file (bad magic)");
  if (size < 24) return fail(e, "Not a valid BF2 file (truncated file header: %zu bytes)", size);
  const uint32_t version = rd<uint32_t>(b + 4), flags = rd<uint32_t>(b + 8);
  if (version != 1) return fail(e, "Unsupported BF2 version: %u (expected 1)", version);
  size_t pos = 16;
  const uint32_t mlen = rd<uint32_t>(b + pos);
  pos += 4;
  if (pos + mlen + 4 > size) return fail(e, "BF2 header truncated (model JSON)");
  m->model_json.assign(reinterpret_cast<const char*>(b + pos), mlen);
  pos += mlen;
  const uint32_t qlen = rd<uint32_t>(b + pos);
  pos += 4;
  if (pos + qlen + 4 > size) return fail(e, "BF2 header truncated (quantize JSON)");
  pos += qlen;
  const uint32_t count = rd<uint32_t>(b + pos);
  pos += 4;
  size_t end = size;
  if (flags & 1u) {  // XXH64 trailer over everything before it
    if (end < pos + 8) return fail(e, "BF2 file too short for its checksum");
    end -= 8;
    const uint64_t stored = rd<uint64_t>(b + end), computed = opc_xxh64(b, end, 0);
    if (stored != computed)
      return fail(e, "checksum mismatch (stored %016llx, computed %016llx)", static_cast<unsigned long long>(stored),
                  static_cast<unsigned long long>(computed));
  }
  for (uint32_t i = 0; i < count; ++i) {
    FileLayer l;
    if (!parse_layer_at(b, end, pos, &l)) return fail(e, "layer %u header at byte %zu is invalid or truncated", i, pos);
    l.id_bytes = 4;
    // the offset `n` payload bytes after the layer's name, SIZE_MAX past the end
    auto after = [&](size_t n) { return n <= end - l.data ? l.data + n : SIZE_MAX; };
    if (l.type == kQuantized && l.n_out > 0) {  // which outlier-id width is followed by a layer (or the end)
      FileLayer probe;
      const size_t e4 = after(payload_bytes(l, 4)), e8 = after(payload_bytes(l, 8));
      const bool last = i + 1 == count;
      const bool ok4 = last ? e4 == end : parse_layer_at(b, end, e4, &probe);
      const bool ok8 = last ? e8 == end : parse_layer_at(b, end, e8, &probe);
      if (!ok4 && ok8) l.id_bytes = 8;
      else if (!ok4 && !ok8 && !last) return fail(e, "cannot locate the layer after '%s'", l.name.c_str());
    }
    const size_t next = after(payload_bytes(l, l.id_bytes));
    if (next > end) return fail(e, "layer '%s' is truncated", l.name.c_str());
    m->layers[l.name] = l;
    pos = next;
  }
  return 0;
}

int load_sparse_part(BFEngine* e, const MappedFile& f, const FileLayer& l, DevLayer* d);

// Copy one quantized layer to the device and repack it.
int load_quantized(BFEngine* e, const MappedFile& f, const FileLayer& l, DevLayer* d) {
  if (l.type != kQuantized && l.type != kSparse)
    return fail(e, "layer '%s' is not quantized (type %u)", l.name.c_str(), l.type);
  if (l.entries != 4 || (l.svs != 1 && l.svs != 8) || l.n_groups != l.out_f)
    return fail(e, "layer '%s': unsupported layout (entries %u, sub_vector_size %u)", l.name.c_str(), l.entries, l.svs);
  const int M = static_cast<int>(l.out_f), K = static_cast<int>(l.in_f);
  const size_t cb_bytes = static_cast<size_t>(M) * 4 * l.svs * 2, idx_bytes = static_cast<size_t>(M) * (K / l.svs);
  const size_t ov_bytes = static_cast<size_t>(l.n_out) * K * 2;
  const uint8_t* src = f.p + l.data;
  std::vector<int64_t> ids(l.n_out);
  const uint8_t* id_src = src + cb_bytes + idx_bytes + ov_bytes;
  for (int i = 0; i < l.n_out; ++i)
    ids[i] = l.id_bytes == 8 ? rd<int64_t>(id_src + 8 * i) : static_cast<int64_t>(rd<int32_t>(id_src + 4 * i));
  const int32_t n_distinct = opc_count_distinct_ids(ids.empty() ? nullptr : ids.data(), l.n_out);
  opc_layer_plan plan;
  ENG_OPC(e, opc_plan_layer(M, K, n_distinct, l.svs, &plan));
  d->L.plan = plan;
  if (dalloc(e, &d->L.units, plan.units_bytes) || dalloc(e, &d->L.codebooks, plan.codebook_bytes) ||
      dalloc(e, &d->L.tile_mask, plan.tile_mask_bytes) ||
      dalloc(e, reinterpret_cast<void**>(&d->L.outlier_rows), plan.outlier_rows_bytes))
    return -1;
  void* tmp = nullptr;
  const size_t tmp_bytes = cb_bytes + idx_bytes + ov_bytes;
  ENG_CUDA(e, cudaMalloc(&tmp, tmp_bytes));
  int rc = 0;
  cudaError_t cr = cudaMemcpyAsync(tmp, src, tmp_bytes, cudaMemcpyHostToDevice, e->stream);
  if (cr != cudaSuccess) {
    rc = fail(e, "copying layer '%s' to the device: %s", l.name.c_str(), cudaGetErrorString(cr));
  } else {
    const uint8_t* t = static_cast<const uint8_t*>(tmp);
    if (opc_repack_layer(&d->L, t, t + cb_bytes, l.n_out ? t + cb_bytes + idx_bytes : nullptr,
                         l.n_out ? ids.data() : nullptr, l.n_out, e->stream) != OPC_OK)
      rc = fail(e, "repacking layer '%s': %s", l.name.c_str(), opc_last_error());
  }
  cudaStreamSynchronize(e->stream);
  cudaFree(tmp);
  if (rc) return rc;
  d->present = true;
  return l.type == kSparse ? load_sparse_part(e, f, l, d) : 0;
}

// Several quantized layers with the same K and sub_vector_size as one layer, rows stacked in order
// (q|k|v, gate|up): one GEMV launch instead of several.  Only plain quantized layers (no element
// outliers) are fused.
int load_stacked(BFEngine* e, const MappedFile& f, const std::vector<const FileLayer*>& parts, DevLayer* d) {
  const FileLayer& l0 = *parts[0];
  const int K = static_cast<int>(l0.in_f), svs = l0.svs;
  int M = 0, n_out = 0;
  for (const FileLayer* l : parts) {
    if (l->type != kQuantized || l->in_f != l0.in_f || l->svs != l0.svs || l->entries != 4 || l->n_groups != l->out_f)
      return fail(e, "layer '%s' cannot be stacked", l->name.c_str());
    M += static_cast<int>(l->out_f);
    n_out += l->n_out;
  }
  std::vector<uint8_t> cb, idx, ov;
  std::vector<int64_t> ids;
  int row0 = 0;
  for (const FileLayer* l : parts) {
    const int Mi = static_cast<int>(l->out_f);
    const size_t cbb = static_cast<size_t>(Mi) * 4 * svs * 2, ib = static_cast<size_t>(Mi) * (K / svs);
    const size_t ob = static_cast<size_t>(l->n_out) * K * 2;
    const uint8_t* src = f.p + l->data;
    cb.insert(cb.end(), src, src + cbb);
    idx.insert(idx.end(), src + cbb, src + cbb + ib);
    ov.insert(ov.end(), src + cbb + ib, src + cbb + ib + ob);
    const uint8_t* id_src = src + cbb + ib + ob;
    for (int i = 0; i < l->n_out; ++i)
      ids.push_back(row0 + (l->id_bytes == 8 ? rd<int64_t>(id_src + 8 * i) : static_cast<int64_t>(rd<int32_t>(id_src + 4 * i))));
    row0 += Mi;
  }
  const int32_t n_distinct = opc_count_distinct_ids(ids.empty() ? nullptr : ids.data(), n_out);
  opc_layer_plan plan;
  ENG_OPC(e, opc_plan_layer(M, K, n_distinct, svs, &plan));
  d->L.plan = plan;
  if (dalloc(e, &d->L.units, plan.units_bytes) || dalloc(e, &d->L.codebooks, plan.codebook_bytes) ||
      dalloc(e, &d->L.tile_mask, plan.tile_mask_bytes) ||
      dalloc(e, reinterpret_cast<void**>(&d->L.outlier_rows), plan.outlier_rows_bytes))
    return -1;
  void* tmp = nullptr;
  ENG_CUDA(e, cudaMalloc(&tmp, cb.size() + idx.size() + ov.size()));
  uint8_t* t = static_cast<uint8_t*>(tmp);
  cudaError_t cr = cudaMemcpy(t, cb.data(), cb.size(), cudaMemcpyHostToDevice);
  if (cr == cudaSuccess) cr = cudaMemcpy(t + cb.size(), idx.data(), idx.size(), cudaMemcpyHostToDevice);
  if (cr == cudaSuccess && !ov.empty()) cr = cudaMemcpy(t + cb.size() + idx.size(), ov.data(), ov.size(), cudaMemcpyHostToDevice);
  int rc = 0;
  if (cr != cudaSuccess) rc = fail(e, "copying '%s' and the layers after it: %s", l0.name.c_str(), cudaGetErrorString(cr));
  else if (opc_repack_layer(&d->L, t, t + cb.size(), n_out ? t + cb.size() + idx.size() : nullptr,
                            n_out ? ids.data() : nullptr, n_out, e->stream) != OPC_OK)
    rc = fail(e, "repacking '%s' stacked: %s", l0.name.c_str(), opc_last_error());
  cudaStreamSynchronize(e->stream);
  cudaFree(tmp);
  if (rc) return rc;
  d->present = true;
  return 0;
}

bool stackable(const std::vector<const FileLayer*>& parts) {
  for (const FileLayer* l : parts)
    if (!l || l->type != kQuantized || l->svs != parts[0]->svs || l->in_f != parts[0]->in_f) return false;
  return true;
}

// The element outliers of a kSparse layer: row-compressed on the host, then copied to the device.
int load_sparse_part(BFEngine* e, const MappedFile& f, const FileLayer& l, DevLayer* d) {
  const int M = static_cast<int>(l.out_f), K = static_cast<int>(l.in_f);
  const size_t cb_bytes = static_cast<size_t>(M) * 4 * l.svs * 2, idx_bytes = static_cast<size_t>(M) * (K / l.svs);
  const uint8_t* src = f.p + l.data;
  const int64_t n = static_cast<int64_t>(l.nnz);
  const uint8_t* vals = src + cb_bytes + idx_bytes;
  const uint8_t* posb = vals + 2 * n;
  std::vector<int64_t> pos(static_cast<size_t>(2 * n));
  for (int64_t i = 0; i < 2 * n; ++i) pos[i] = rd<int32_t>(posb + 4 * i);
  std::vector<uint16_t> cb(cb_bytes / 2), vin(static_cast<size_t>(n)), vout(static_cast<size_t>(std::max<int64_t>(n, 1)));
  std::memcpy(cb.data(), src, cb_bytes);
  if (n) std::memcpy(vin.data(), vals, static_cast<size_t>(2 * n));
  std::vector<int32_t> row_ptr(M + 1), cols(static_cast<size_t>(std::max<int64_t>(n, 1)));
  std::vector<float> delta(cols.size());
  int64_t nnz = 0;
  ENG_OPC(e, opc_coo_build(M, K, l.svs, cb.data(), src + cb_bytes, n ? pos.data() : nullptr, n ? vin.data() : nullptr, n,
                           row_ptr.data(), cols.data(), vout.data(), delta.data(), &nnz));
  d->nnz = nnz;
  if (dalloc(e, reinterpret_cast<void**>(&d->row_ptr), sizeof(int32_t) * (M + 1)) ||
      dalloc(e, reinterpret_cast<void**>(&d->cols), sizeof(int32_t) * std::max<int64_t>(nnz, 1)) ||
      dalloc(e, reinterpret_cast<void**>(&d->delta), sizeof(float) * std::max<int64_t>(nnz, 1)) ||
      dalloc(e, reinterpret_cast<void**>(&d->values), 2 * std::max<int64_t>(nnz, 1)))
    return -1;
  ENG_CUDA(e, cudaMemcpy(d->row_ptr, row_ptr.data(), sizeof(int32_t) * (M + 1), cudaMemcpyHostToDevice));
  if (nnz) {
    ENG_CUDA(e, cudaMemcpy(d->cols, cols.data(), sizeof(int32_t) * nnz, cudaMemcpyHostToDevice));
    ENG_CUDA(e, cudaMemcpy(d->delta, delta.data(), sizeof(float) * nnz, cudaMemcpyHostToDevice));
    ENG_CUDA(e, cudaMemcpy(d->values, vout.data(), 2 * nnz, cudaMemcpyHostToDevice));
  }
  return 0;
}

// A fp16 pass-through vector of `n` values on the device (NULL when the file lacks it).
int load_vector(BFEngine* e, const MappedFile& f, const Model& m, const std::string& name, int n,
                const __half** out) {
  *out = nullptr;
  auto it = m.layers.find(name);
  if (it == m.layers.end()) return 0;
  const FileLayer& l = it->second;
  if (l.type != kPassthrough || static_cast<size_t>(l.out_f) * l.in_f != static_cast<size_t>(n))
    return fail(e, "'%s': expected a pass-through fp16 vector of %d values", name.c_str(), n);
  void* p = nullptr;
  if (dalloc(e, &p, static_cast<size_t>(n) * 2)) return -1;
  ENG_CUDA(e, cudaMemcpy(p, f.p + l.data, static_cast<size_t>(n) * 2, cudaMemcpyHostToDevice));
  *out = static_cast<const __half*>(p);
  return 0;
}

const FileLayer* find(const Model& m, const std::string& name) {
  auto it = m.layers.find(name);
  return it == m.layers.end() ? nullptr : &it->second;
}

int load_model(BFEngine* e, const char* path, uint32_t max_context) {
  MappedFile f;
  f.fd = open(path, O_RDONLY);
  if (f.fd < 0) return fail(e, "Cannot open file: %s", path);
  struct stat st;
  if (fstat(f.fd, &st) != 0 || st.st_size <= 0) return fail(e, "Cannot stat file: %s", path);
  f.size = static_cast<size_t>(st.st_size);
  void* mp = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
  if (mp == MAP_FAILED) return fail(e, "Cannot mmap file: %s", path);
  f.p = static_cast<const uint8_t*>(mp);
  Model m;
  if (parse_file(e, f, &m)) return -1;

  // ---- model numbers: JSON first, then the layer shapes
  const std::string& js = m.model_json;
  BFModelConfig& c = e->cfg;
  std::string arch;
  std::snprintf(c.architecture, sizeof(c.architecture), "%s", json_string(js, "architecture", &arch) ? arch.c_str() : "unknown");
  double v;
  const FileLayer* emb = find(m, "model.embed_tokens.weight");
  if (!emb) return fail(e, "no 'model.embed_tokens.weight' layer");
  e->hidden = static_cast<int>(emb->in_f);
  e->vocab = static_cast<int>(emb->out_f);
  if (json_number(js, "hidden_size", &v) && static_cast<int>(v) != e->hidden)
    return fail(e, "hidden_size %d in the model JSON, %d in the embedding", static_cast<int>(v), e->hidden);
  int n_layers = 0;
  if (json_number(js, "num_hidden_layers", &v)) n_layers = static_cast<int>(v);
  else
    while (find(m, "model.layers." + std::to_string(n_layers) + ".self_attn.q_proj.weight")) ++n_layers;
  if (n_layers <= 0) return fail(e, "the model has no decoder layers");
  e->n_layers = n_layers;
  const std::string p0 = "model.layers.0.";
  const FileLayer* q0 = find(m, p0 + "self_attn.q_proj.weight");
  const FileLayer* k0 = find(m, p0 + "self_attn.k_proj.weight");
  const FileLayer* g0 = find(m, p0 + "mlp.gate_proj.weight");
  if (!q0 || !k0 || !g0) return fail(e, "layer 0 lacks q_proj, k_proj or gate_proj");
  e->heads = json_number(js, "num_attention_heads", &v) ? static_cast<int>(v) : static_cast<int>(q0->out_f) / 128;
  if (e->heads <= 0) return fail(e, "cannot determine num_attention_heads");
  e->hd = json_number(js, "head_dim", &v) ? static_cast<int>(v) : static_cast<int>(q0->out_f) / e->heads;
  if (json_number(js, "num_kv_heads", &v) || json_number(js, "num_key_value_heads", &v)) e->kv_heads = static_cast<int>(v);
  else e->kv_heads = e->hd > 0 ? static_cast<int>(k0->out_f) / e->hd : 0;
  e->inter = static_cast<int>(g0->out_f);
  const float theta = json_number(js, "rope_theta", &v) ? static_cast<float>(v) : 10000.0f;
  e->eps = json_number(js, "rms_norm_eps", &v) ? static_cast<float>(v) : 1e-5f;
  const uint32_t max_pos = json_number(js, "max_position_embeddings", &v) ? static_cast<uint32_t>(v) : 0u;
  if (e->hd <= 0 || e->hd % 32 || e->hd > kMaxHeadDim || e->heads * e->hd != static_cast<int>(q0->out_f))
    return fail(e, "head_dim %d with %d heads does not fit q_proj (%u rows); head_dim must be a multiple of 32 up to %d",
                e->hd, e->heads, q0->out_f, kMaxHeadDim);
  if (e->kv_heads <= 0 || e->heads % e->kv_heads || e->kv_heads * e->hd != static_cast<int>(k0->out_f))
    return fail(e, "%d kv heads do not fit k_proj (%u rows) and %d query heads", e->kv_heads, k0->out_f, e->heads);
  c.vocab_size = static_cast<uint32_t>(e->vocab);
  c.hidden_size = static_cast<uint32_t>(e->hidden);
  c.intermediate_size = static_cast<uint32_t>(e->inter);
  c.num_hidden_layers = static_cast<uint32_t>(e->n_layers);
  c.num_attention_heads = static_cast<uint32_t>(e->heads);
  c.num_kv_heads = static_cast<uint32_t>(e->kv_heads);
  c.max_position_embeddings = max_pos;
  c.rope_theta = theta;
  c.head_dim = static_cast<uint32_t>(e->hd);
  e->ctx = max_context ? max_context : (max_pos ? std::min(max_pos, kDefaultContext) : kDefaultContext);

  // ---- device
  ENG_CUDA(e, cudaSetDevice(e->device));
  ENG_CUDA(e, cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));

  // ---- weights
  const int qd = e->heads * e->hd, kvd = e->kv_heads * e->hd;
  e->blocks.resize(e->n_layers);
  for (int i = 0; i < e->n_layers; ++i) {
    Block& B = e->blocks[i];
    const std::string p = "model.layers." + std::to_string(i) + ".";
    struct {
      const char* name;
      DevLayer* d;
      int M, K;
    } want[] = {{"self_attn.q_proj.weight", &B.q, qd, e->hidden},   {"self_attn.k_proj.weight", &B.k, kvd, e->hidden},
                {"self_attn.v_proj.weight", &B.v, kvd, e->hidden},  {"self_attn.o_proj.weight", &B.o, e->hidden, qd},
                {"mlp.gate_proj.weight", &B.gate, e->inter, e->hidden}, {"mlp.up_proj.weight", &B.up, e->inter, e->hidden},
                {"mlp.down_proj.weight", &B.down, e->hidden, e->inter}};
    std::vector<const FileLayer*> fl;
    for (auto& w : want) {
      const FileLayer* l = find(m, p + w.name);
      if (!l) return fail(e, "missing layer '%s%s'", p.c_str(), w.name);
      if (static_cast<int>(l->out_f) != w.M || static_cast<int>(l->in_f) != w.K)
        return fail(e, "'%s%s' is %ux%u, expected %dx%d", p.c_str(), w.name, l->out_f, l->in_f, w.M, w.K);
      fl.push_back(l);
    }
    const std::vector<const FileLayer*> qkv = {fl[0], fl[1], fl[2]}, gu = {fl[4], fl[5]};
    if (stackable(qkv)) {
      if (load_stacked(e, f, qkv, &B.qkv)) return -1;
    } else if (load_quantized(e, f, *fl[0], &B.q) || load_quantized(e, f, *fl[1], &B.k) ||
               load_quantized(e, f, *fl[2], &B.v)) {
      return -1;
    }
    if (load_quantized(e, f, *fl[3], &B.o)) return -1;
    if (stackable(gu)) {
      if (load_stacked(e, f, gu, &B.gu)) return -1;
    } else if (load_quantized(e, f, *fl[4], &B.gate) || load_quantized(e, f, *fl[5], &B.up)) {
      return -1;
    }
    if (load_quantized(e, f, *fl[6], &B.down)) return -1;
    if (load_vector(e, f, m, p + "input_layernorm.weight", e->hidden, &B.ln_in) ||
        load_vector(e, f, m, p + "post_attention_layernorm.weight", e->hidden, &B.ln_post))
      return -1;
  }
  if (load_vector(e, f, m, "model.norm.weight", e->hidden, &e->final_norm)) return -1;
  void* table = nullptr;
  if (dalloc(e, &table, static_cast<size_t>(e->vocab) * e->hidden * 2)) return -1;
  e->embed_table = static_cast<__half*>(table);
  if (emb->type == kPassthrough) {
    ENG_CUDA(e, cudaMemcpy(table, f.p + emb->data, static_cast<size_t>(e->vocab) * e->hidden * 2, cudaMemcpyHostToDevice));
  } else {
    if (load_quantized(e, f, *emb, &e->embed)) return -1;
    ENG_OPC(e, opc_dequant(&e->embed.L, table, e->hidden, e->stream));
    if (e->embed.nnz)
      ENG_OPC(e, opc_coo_scatter(e->vocab, e->embed.row_ptr, e->embed.cols, e->embed.values, table, e->hidden, e->stream));
    ENG_CUDA(e, cudaStreamSynchronize(e->stream));
  }
  const FileLayer* lm = find(m, "lm_head.weight");
  if (lm) {
    if (static_cast<int>(lm->out_f) != e->vocab || static_cast<int>(lm->in_f) != e->hidden)
      return fail(e, "lm_head is %ux%u, expected %dx%d", lm->out_f, lm->in_f, e->vocab, e->hidden);
    if (load_quantized(e, f, *lm, &e->lm_head)) return -1;
  } else {
    if (!e->embed.present) return fail(e, "no lm_head and the embedding is not quantized (tied fp16 head unsupported)");
    e->lm_from_embed = true;
  }

  // ---- KV cache and scratch
  e->kv_bytes = 2ull * e->n_layers * e->kv_heads * static_cast<size_t>(e->ctx) * e->hd * 2;
  void* kv = nullptr;
  if (dalloc(e, &kv, e->kv_bytes)) return -1;
  e->kcache = static_cast<__half*>(kv);
  e->vcache = e->kcache + e->kv_bytes / 4;
  ENG_CUDA(e, cudaMemset(kv, 0, e->kv_bytes));
  e->ld_x = pad8(e->hidden);
  e->ld_q = pad8(qd);
  e->ld_kv = pad8(kvd);
  e->ld_i = pad8(e->inter);
  e->ld_y = pad8(std::max(e->hidden, qd));
  e->ld_qkv = pad8(qd + 2 * kvd);
  e->ld_gu = pad8(2 * e->inter);
  struct {
    __half** p;
    int ld;
  } bufs[] = {{&e->xn, e->ld_x}, {&e->q, e->ld_q}, {&e->k, e->ld_kv}, {&e->v, e->ld_kv}, {&e->att, e->ld_q},
              {&e->y, e->ld_y},  {&e->g, e->ld_i}, {&e->u, e->ld_i},   {&e->a, e->ld_i},
              {&e->qkv, e->ld_qkv}, {&e->gu, e->ld_gu}};
  for (auto& b : bufs) {
    void* p = nullptr;
    if (dalloc(e, &p, static_cast<size_t>(kChunk) * b.ld * 2)) return -1;
    ENG_CUDA(e, cudaMemset(p, 0, static_cast<size_t>(kChunk) * b.ld * 2));
    *b.p = static_cast<__half*>(p);
  }
  void* ap = nullptr;
  size_t records = 0;  // the most (token, head, range) records one attention launch writes
  for (int n = 1; n <= static_cast<int>(kChunk); ++n) {
    const int sp = attention_splits(n, e->heads);
    if (sp > 1) records = std::max(records, static_cast<size_t>(n) * e->heads * sp);
  }
  if (dalloc(e, &ap, std::max<size_t>(records, 1) * (e->hd + 2) * 4)) return -1;
  e->att_part = static_cast<float*>(ap);
  void* ac = nullptr;
  if (dalloc(e, &ac, static_cast<size_t>(kChunk) * e->heads * sizeof(int))) return -1;
  ENG_CUDA(e, cudaMemset(ac, 0, static_cast<size_t>(kChunk) * e->heads * sizeof(int)));
  e->att_count = static_cast<int*>(ac);
  void* hp = nullptr;
  if (dalloc(e, &hp, static_cast<size_t>(kChunk) * e->hidden * 4)) return -1;
  e->h = static_cast<float*>(hp);
  void* lp = nullptr;
  if (dalloc(e, &lp, static_cast<size_t>(e->vocab) * 2)) return -1;
  e->logits16 = static_cast<__half*>(lp);
  ENG_CUDA(e, cudaMallocHost(reinterpret_cast<void**>(&e->host_logits), static_cast<size_t>(e->vocab) * 2));
  ENG_CUDA(e, cudaMallocHost(reinterpret_cast<void**>(&e->h_tokpos), (kChunk + 1) * sizeof(int32_t)));
  void* tp = nullptr;
  if (dalloc(e, &tp, (kChunk + 1) * sizeof(int32_t))) return -1;
  e->d_tokpos = static_cast<int32_t*>(tp);

  // one workspace for every projection and chunk size (calls are ordered on the engine's stream)
  std::vector<const DevLayer*> all;
  for (auto& B : e->blocks)
    for (const DevLayer* d : {&B.q, &B.k, &B.v, &B.o, &B.gate, &B.up, &B.down, &B.qkv, &B.gu})
      if (d->present) all.push_back(d);
  all.push_back(e->lm_from_embed ? &e->embed : &e->lm_head);
  for (const DevLayer* d : all)
    for (int b = 1; b <= kGemvMaxBatch; ++b)
      e->ws_bytes = std::max(e->ws_bytes, opc_gemv_workspace_bytes(&d->L.plan, b, e->device));
  if (dalloc(e, &e->ws, e->ws_bytes)) return -1;
  ENG_OPC(e, opc_workspace_init(e->ws, e->ws_bytes, e->stream));
  ENG_CUDA(e, cudaStreamSynchronize(e->stream));
  e->stats.peak_memory_bytes = e->dev_bytes;
  return 0;
}

// Append n (<= kChunk) tokens at positions pos.. and, with `logits`, write the last one's
// next-token logits (fp32, vocab values) to the host.
// Every launch of a chunk of n tokens, stream-ordered and asynchronous (no host synchronisation),
// reading the tokens and the first position from d_tokpos; with want_logits the last token's
// next-token logits are copied to host_logits.
// add_rmsnorm_kernel for `rows` rows from row0, with the residual add when y is given and the
// weight when w is given.
cudaError_t launch_norm(cudaStream_t s, int rows, float* h, int hidden, const __half* y, int ldy, int row0,
                        const __half* w, float eps, __half* out, int ldo) {
  auto k = y ? (w ? add_rmsnorm_kernel<true, true> : add_rmsnorm_kernel<true, false>)
             : (w ? add_rmsnorm_kernel<false, true> : add_rmsnorm_kernel<false, false>);
  return launch_pdl(k, dim3(rows), dim3(kNormThreads), s, h, hidden, y, ldy, row0, w, eps, out, ldo);
}

int enqueue_chunk(BFEngine* e, int n, bool want_logits, uint32_t* n_launches) {
  cudaStream_t s = e->stream;
  const int32_t* pos0 = e->d_tokpos + kChunk;
  const int qd = e->heads * e->hd;
  uint32_t launches = 0;
  auto gemv = [&](const DevLayer& d, const __half* x, int ldx, __half* y, int ldy, int rows) -> int {
    ++launches;
    const int rc = rows <= kGemvMaxBatch ? opc_gemv(&d.L, x, ldx, y, ldy, rows, e->ws, e->ws_bytes, s)
                                         : opc_gemm(&d.L, x, ldx, y, ldy, rows, s);
    if (rc != OPC_OK)
      return fail(e, "%s (%d x %d, %d tokens): %s", rows <= kGemvMaxBatch ? "opc_gemv" : "opc_gemm", d.L.plan.M,
                  d.L.plan.K, rows, opc_last_error());
    if (d.nnz) {  // element-wise outliers: the CSR epilogue
      ++launches;
      if (opc_coo_gemv(d.L.plan.M, d.row_ptr, d.cols, d.delta, x, ldx, y, ldy, rows, s) != OPC_OK)
        return fail(e, "opc_coo_gemv: %s", opc_last_error());
    }
    return 0;
  };
  ENG_CUDA(e, cudaMemcpyAsync(e->d_tokpos, e->h_tokpos, (kChunk + 1) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  embed_kernel<<<n, 256, 0, s>>>(e->embed_table, e->hidden, e->d_tokpos, e->h);
  ++launches;
  const __half* res = nullptr;  // the previous block's down projection, still to be added into h
  const int64_t silu_n = static_cast<int64_t>(n) * e->inter;
  const unsigned silu_grid = static_cast<unsigned>(std::min<int64_t>((silu_n + 255) / 256, 4 * 148));
  for (int l = 0; l < e->n_layers; ++l) {
    const Block& B = e->blocks[l];
    __half* kc = e->kcache + static_cast<size_t>(l) * e->kv_heads * e->ctx * e->hd;
    __half* vc = e->vcache + static_cast<size_t>(l) * e->kv_heads * e->ctx * e->hd;
    ENG_CUDA(e, launch_norm(s, n, e->h, e->hidden, res, e->ld_y, 0, B.ln_in, e->eps, e->xn, e->ld_x));
    __half *qb = e->q, *kb = e->k, *vb = e->v;
    int ldq = e->ld_q, ldkv = e->ld_kv;
    if (B.qkv.present) {  // one GEMV for q|k|v
      if (gemv(B.qkv, e->xn, e->ld_x, e->qkv, e->ld_qkv, n)) return -1;
      qb = e->qkv;
      kb = qb + qd;
      vb = kb + e->kv_heads * e->hd;
      ldq = ldkv = e->ld_qkv;
    } else if (gemv(B.q, e->xn, e->ld_x, e->q, e->ld_q, n) || gemv(B.k, e->xn, e->ld_x, e->k, e->ld_kv, n) ||
               gemv(B.v, e->xn, e->ld_x, e->v, e->ld_kv, n)) {
      return -1;
    }
    ENG_CUDA(e, launch_pdl(rope_cache_kernel, dim3(n, kRopeSplit), dim3(256), s, qb, ldq, kb, vb, ldkv, e->heads,
                           e->kv_heads, e->hd, pos0, e->cfg.rope_theta, kc, vc, static_cast<int>(e->ctx)));
    ENG_CUDA(e, launch_pdl(attention_kernel, dim3(e->heads, n, attention_splits(n, e->heads)), dim3(kAttnThreads), s, qb, ldq, kc, vc,
                           e->heads, e->kv_heads, e->hd, static_cast<int>(e->ctx), pos0, e->att, e->ld_q,
                           e->att_part, e->att_count));
    if (gemv(B.o, e->att, e->ld_q, e->y, e->ld_y, n)) return -1;
    ENG_CUDA(e, launch_norm(s, n, e->h, e->hidden, e->y, e->ld_y, 0, B.ln_post, e->eps, e->xn, e->ld_x));
    if (B.gu.present) {  // one GEMV for gate|up
      if (gemv(B.gu, e->xn, e->ld_x, e->gu, e->ld_gu, n)) return -1;
      ENG_CUDA(e, launch_pdl(silu_mul_kernel, dim3(silu_grid), dim3(256), s, e->gu, e->gu + e->inter, e->ld_gu,
                             e->inter, n, e->a, e->ld_i));
    } else {
      if (gemv(B.gate, e->xn, e->ld_x, e->g, e->ld_i, n) || gemv(B.up, e->xn, e->ld_x, e->u, e->ld_i, n)) return -1;
      ENG_CUDA(e, launch_pdl(silu_mul_kernel, dim3(silu_grid), dim3(256), s, e->g, e->u, e->ld_i, e->inter, n, e->a,
                             e->ld_i));
    }
    if (gemv(B.down, e->a, e->ld_i, e->y, e->ld_y, n)) return -1;
    res = e->y;
    launches += 5;  // two RMSNorms (each with the residual add before it), rotary + cache append, attention, SiLU
  }

  if (want_logits) {  // the last residual add and the final norm, for the chunk's last token only
    ENG_CUDA(e, launch_norm(s, 1, e->h, e->hidden, res, e->ld_y, n - 1, e->final_norm, e->eps, e->xn, e->ld_x));
    ++launches;
    if (gemv(e->lm_from_embed ? e->embed : e->lm_head, e->xn, e->ld_x, e->logits16, e->vocab, 1)) return -1;
    ENG_CUDA(e, cudaMemcpyAsync(e->host_logits, e->logits16, static_cast<size_t>(e->vocab) * 2,
                                cudaMemcpyDeviceToHost, s));
  }
  ENG_CUDA(e, cudaGetLastError());
  *n_launches = launches;
  return 0;
}

// Capture the one-token step with logits into a CUDA graph (once); on any failure the engine
// keeps launching directly.
void capture_step(BFEngine* e) {
  e->graph_tried = true;
  cudaGraph_t g = nullptr;
  if (cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  const std::string saved = e->error;
  uint32_t launches = 0;
  const int rc = enqueue_chunk(e, 1, true, &launches);
  const cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (rc == 0 && ce == cudaSuccess && g && cudaGraphInstantiate(&e->step_exec, g, 0) == cudaSuccess) {
    e->step_launches = launches;
  } else {
    e->step_exec = nullptr;
    e->error = saved;
  }
  if (g) cudaGraphDestroy(g);
  cudaGetLastError();
}

int run_chunk(BFEngine* e, const int32_t* tokens, int n, float* logits) {
  cudaStream_t s = e->stream;
  for (int i = 0; i < n; ++i) e->h_tokpos[i] = tokens[i];
  e->h_tokpos[kChunk] = static_cast<int32_t>(e->pos);
  uint32_t launches = 0;
  if (n == 1 && logits && !e->graph_tried && e->direct_steps > 0) capture_step(e);
  if (n == 1 && logits && e->step_exec) {
    ENG_CUDA(e, cudaGraphLaunch(e->step_exec, s));
    launches = e->step_launches;
  } else {
    if (enqueue_chunk(e, n, logits != nullptr, &launches)) return -1;
    if (n == 1 && logits) ++e->direct_steps;
  }
  ENG_CUDA(e, cudaStreamSynchronize(s));
  int32_t derr = 0;
  if (opc_take_device_error(e->device, &derr) != OPC_OK || derr != 0)
    return fail(e, "device error %d reported by a kernel", derr);
  if (logits)
    halves_to_floats(e->host_logits, logits, static_cast<size_t>(e->vocab));
  e->pos += static_cast<uint32_t>(n);
  e->history.insert(e->history.end(), tokens, tokens + n);
  e->stats.n_kernel_dispatches += launches;
  return 0;
}

int ready(BFEngine* e) {
  if (!e) return -1;
  if (!e->error.empty() && e->blocks.empty()) return -1;  // failed at load: stays failed
  return 0;
}

// Append tokens in chunks; logits of the last token when `logits` is non-NULL.
int run_tokens(BFEngine* e, const int32_t* tokens, uint32_t n, float* logits) {
  if (static_cast<uint64_t>(e->pos) + n > e->ctx)
    return fail(e, "context full: %u cached + %u new tokens exceed the %u-position cache", e->pos, n, e->ctx);
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= e->vocab) return fail(e, "token id %d outside [0, %d)", tokens[i], e->vocab);
  cudaSetDevice(e->device);
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0; i < n; i += kChunk) {
    const int c = static_cast<int>(std::min<uint32_t>(kChunk, n - i));
    if (run_chunk(e, tokens + i, c, (logits && i + c == n) ? logits : nullptr)) return -1;
  }
  e->stats.total_time_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return 0;
}

int32_t sample_token(const std::vector<float>& logits_in, const BFSamplingParams& p, const std::vector<int32_t>& hist,
                     std::mt19937_64& rng) {
  std::vector<float> l(logits_in);
  const int V = static_cast<int>(l.size());
  if (p.repetition_penalty > 0.f && p.repetition_penalty != 1.f) {
    std::vector<char> seen(V, 0);
    for (int32_t t : hist)
      if (t >= 0 && t < V && !seen[t]) {
        seen[t] = 1;
        l[t] = l[t] > 0.f ? l[t] / p.repetition_penalty : l[t] * p.repetition_penalty;
      }
  }
  if (!(p.temperature > 1e-6f)) return static_cast<int32_t>(std::max_element(l.begin(), l.end()) - l.begin());
  const bool cut_k = p.top_k > 0 && p.top_k < V, cut_p = p.top_p > 0.f && p.top_p < 1.f;
  if (!cut_k && !cut_p) {  // the whole softmax: a draw needs no ordering of the vocabulary
    const double mx = *std::max_element(l.begin(), l.end());
    std::vector<double> w(V);
    double sum = 0.0;
    for (int i = 0; i < V; ++i) sum += (w[i] = std::exp((static_cast<double>(l[i]) - mx) / p.temperature));
    const double r = std::uniform_real_distribution<double>(0.0, sum)(rng);
    double c = 0.0;
    for (int i = 0; i < V; ++i) {
      c += w[i];
      if (r < c) return i;
    }
    return V - 1;
  }
  // candidates by descending logit (ties: lower id first); with top-k only the first k are ordered
  std::vector<int> idx(V);
  std::iota(idx.begin(), idx.end(), 0);
  const auto before = [&](int a, int b) { return l[a] > l[b] || (l[a] == l[b] && a < b); };
  int keep = V;
  if (cut_k) {
    keep = p.top_k;
    std::partial_sort(idx.begin(), idx.begin() + keep, idx.end(), before);
  } else {
    std::sort(idx.begin(), idx.end(), before);
  }
  std::vector<double> w(keep);
  const double mx = l[idx[0]];
  double sum = 0.0;
  for (int i = 0; i < keep; ++i) sum += (w[i] = std::exp((static_cast<double>(l[idx[i]]) - mx) / p.temperature));
  if (p.top_p > 0.f && p.top_p < 1.f) {
    double c = 0.0;
    int k = 0;
    while (k < keep) {
      c += w[k++] / sum;
      if (c >= p.top_p) break;
    }
    keep = std::max(k, 1);
    sum = 0.0;
    for (int i = 0; i < keep; ++i) sum += w[i];
  }
  const double r = std::uniform_real_distribution<double>(0.0, sum)(rng);
  double c = 0.0;
  for (int i = 0; i < keep; ++i) {
    c += w[i];
    if (r < c) return idx[i];
  }
  return idx[keep - 1];
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// C API
// ------------------------------------------------------------------------------------------------
extern "C" {

BFEngine* bf_engine_create_ex(const char* path, int32_t device, uint32_t max_context) {
  if (!path) return nullptr;
  BFEngine* e = new (std::nothrow) BFEngine();
  if (!e) return nullptr;
  e->device = device;
  if (load_model(e, path, max_context) != 0) {
    // keep the message; release what was allocated (the handle stays, as in the reference)
    const std::string msg = e->error;
    for (void* p : e->allocs) cudaFree(p);
    e->allocs.clear();
    if (e->host_logits) cudaFreeHost(e->host_logits);
    e->host_logits = nullptr;
    if (e->h_tokpos) cudaFreeHost(e->h_tokpos);
    e->h_tokpos = nullptr;
    if (e->stream) cudaStreamDestroy(e->stream);
    e->stream = nullptr;
    e->blocks.clear();
    e->dev_bytes = 0;
    e->error = msg.empty() ? "load failed" : msg;
  }
  return e;
}

BFEngine* bf_engine_create(const char* path) { return bf_engine_create_ex(path, 0, 0); }

void bf_engine_destroy(BFEngine* e) {
  if (!e) return;
  if (!e->allocs.empty() || e->stream) {
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    if (e->step_exec) cudaGraphExecDestroy(e->step_exec);
    for (void* p : e->allocs) cudaFree(p);
    if (e->host_logits) cudaFreeHost(e->host_logits);
    if (e->h_tokpos) cudaFreeHost(e->h_tokpos);
    if (e->stream) cudaStreamDestroy(e->stream);
  }
  delete e;
}

const BFModelConfig* bf_engine_get_config(const BFEngine* e) { return e ? &e->cfg : nullptr; }
const char* bf_engine_get_error(const BFEngine* e) { return (e && !e->error.empty()) ? e->error.c_str() : nullptr; }
uint32_t bf_engine_vocab_size(const BFEngine* e) { return e ? e->cfg.vocab_size : 0u; }

int bf_engine_forward(BFEngine* e, const int32_t* tokens, uint32_t seq_len, float* logits_out, uint32_t vocab_size) {
  if (ready(e)) return -1;
  if (!tokens || seq_len == 0 || !logits_out) return fail(e, "bf_engine_forward: need tokens and a logits buffer");
  if (vocab_size != e->cfg.vocab_size) return fail(e, "logits buffer holds %u values, the vocabulary %u", vocab_size, e->cfg.vocab_size);
  bf_engine_reset_kv_cache(e);
  e->error.clear();
  return run_tokens(e, tokens, seq_len, logits_out);
}

int bf_engine_prefill(BFEngine* e, const int32_t* tokens, uint32_t seq_len) {
  if (ready(e)) return -1;
  if (seq_len == 0) return 0;
  if (!tokens) return fail(e, "bf_engine_prefill: NULL tokens");
  e->error.clear();
  return run_tokens(e, tokens, seq_len, nullptr);
}

int bf_engine_forward_step(BFEngine* e, int32_t token, float* logits_out, uint32_t vocab_size) {
  if (ready(e)) return -1;
  if (!logits_out) return fail(e, "bf_engine_forward_step: NULL logits buffer");
  if (vocab_size != e->cfg.vocab_size) return fail(e, "logits buffer holds %u values, the vocabulary %u", vocab_size, e->cfg.vocab_size);
  e->error.clear();
  return run_tokens(e, &token, 1, logits_out);
}

int32_t bf_engine_generate_tokens(BFEngine* e, const int32_t* prompt, uint32_t prompt_len, uint32_t max_new_tokens,
                                  const BFSamplingParams* params, int32_t* out_tokens) {
  if (ready(e)) return -1;
  if ((prompt_len && !prompt) || (max_new_tokens && !out_tokens)) return fail(e, "bf_engine_generate: NULL buffer");
  const BFSamplingParams& p = params ? *params : BF_DEFAULT_SAMPLING;
  std::mt19937_64 rng(p.seed ? p.seed : static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count()));
  bf_engine_reset_kv_cache(e);
  e->error.clear();
  const int32_t start = 0;  // an empty prompt starts from token 0
  const int32_t* pr = prompt_len ? prompt : &start;
  const uint32_t n = prompt_len ? prompt_len : 1u;
  std::vector<float> logits(e->vocab);
  const auto t0 = std::chrono::steady_clock::now();
  if (n > 1 && run_tokens(e, pr, n - 1, nullptr)) return -1;
  if (max_new_tokens == 0) return 0;
  if (run_tokens(e, pr + n - 1, 1, logits.data())) return -1;
  int32_t generated = 0;
  for (uint32_t i = 0; i < max_new_tokens; ++i) {
    const int32_t t = sample_token(logits, p, e->history, rng);
    out_tokens[generated++] = t;
    if (t == 0 || i + 1 == max_new_tokens) break;
    if (run_tokens(e, &t, 1, logits.data())) return generated;
  }
  e->stats.total_tokens_generated += static_cast<uint64_t>(generated);
  (void)t0;
  e->stats.tokens_per_second =
      e->stats.total_time_seconds > 0 ? static_cast<double>(e->stats.total_tokens_generated) / e->stats.total_time_seconds : 0.0;
  return generated;
}

int32_t bf_engine_generate(BFEngine* e, const char* prompt, uint32_t max_new_tokens, const BFSamplingParams* params,
                           FILE* output) {
  if (ready(e) || !prompt) return -1;
  std::vector<int32_t> toks;
  for (const unsigned char* c = reinterpret_cast<const unsigned char*>(prompt); *c; ++c) toks.push_back(*c);
  std::vector<int32_t> out(max_new_tokens);
  const int32_t n = bf_engine_generate_tokens(e, toks.data(), static_cast<uint32_t>(toks.size()), max_new_tokens, params,
                                              out.data());
  if (n > 0 && output) {
    for (int32_t i = 0; i < n; ++i) {
      if (out[i] >= 0 && out[i] < 256) std::fputc(out[i], output);
      else std::fputs("?", output);
    }
    std::fflush(output);
  }
  return n;
}

void bf_engine_reset_kv_cache(BFEngine* e) {
  if (!e) return;
  e->pos = 0;
  e->history.clear();
  if (e->kcache && e->stream) {
    cudaSetDevice(e->device);
    cudaMemsetAsync(e->kcache, 0, e->kv_bytes, e->stream);
    cudaStreamSynchronize(e->stream);
  }
}

size_t bf_engine_kv_cache_size(const BFEngine* e) { return e ? e->kv_bytes : 0; }
uint32_t bf_engine_position(const BFEngine* e) { return e ? e->pos : 0u; }

void bf_engine_get_stats(const BFEngine* e, BFStats* s) {
  if (!e || !s) return;
  *s = e->stats;
  s->peak_memory_bytes = e->dev_bytes;
  s->tokens_per_second = s->total_time_seconds > 0 ? static_cast<double>(s->total_tokens_generated) / s->total_time_seconds : 0.0;
}

void bf_engine_reset_stats(BFEngine* e) {
  if (!e) return;
  e->stats = BFStats{};
}

const char* bf_version(void) { return "opc_b200 engine 1.0 (runtime API of opacc1ty 1.0.2)"; }

int bf_has_metal_gpu(void) { return 0; }

int bf_has_cuda_gpu(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int d = 0; d < n; ++d) {
    cudaDeviceProp pr;
    if (cudaGetDeviceProperties(&pr, d) == cudaSuccess && pr.major == 10) return 1;
  }
  return 0;
}

}  // extern "C"
