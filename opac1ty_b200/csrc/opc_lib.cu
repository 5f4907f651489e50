// opc_lib.cu -- C ABI (include/opc_b200.h) over the sm_100a kernels.  Single translation
// unit: the kernels live in the included .cuh files.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/opc_b200.h"
#include "opc_device.cuh"
#include "opc_chain.cuh"
#include "opc_chain2.cuh"
#include "opc_coo.cuh"
#include "opc_gemm.cuh"
#include "opc_gemv.cuh"
#include "opc_gemvd.cuh"
#include "opc_gemvq.cuh"
#include "opc_layer.cuh"
#include "opc_vq8.cuh"

#define OPC_VERSION_STRING "opc_b200 0.2.0 abi 1"

namespace {

thread_local char g_last_error[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(OPC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define OPC_CUDA(call, what)                           \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct DeviceCache {
  int sm_count = 0;
  int max_smem_optin = 0;
};
std::mutex g_mu;
std::map<int, DeviceCache> g_dev;

int device_cache(int dev, DeviceCache* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceCache& c = g_dev[dev];
  if (c.sm_count == 0) {
    OPC_CUDA(cudaDeviceGetAttribute(&c.sm_count, cudaDevAttrMultiProcessorCount, dev),
             "cudaDeviceGetAttribute(SM count)");
    OPC_CUDA(cudaDeviceGetAttribute(&c.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
             "cudaDeviceGetAttribute(smem optin)");
  }
  *out = c;
  return OPC_OK;
}

// k columns per index unit: 128 (svs = 1, 512-byte units), 256 (svs = 8, 128-byte units)
int unit_cols(int svs) { return svs == 8 ? opc::kVq8BlockCols : opc::kPackedCols; }

bool plan_ok(const opc_layer_plan* p) {
  return p && p->M > 0 && p->K > 0 && p->n_outliers >= 0 && p->n_outliers <= p->M &&
         (p->sub_vector_size == 1 || (p->sub_vector_size == 8 && p->K % 8 == 0)) &&
         p->row_tiles == ceil_div(p->M, opc::kTileRows) && p->k_units == ceil_div(p->K, unit_cols(p->sub_vector_size)) &&
         p->M_pad == p->row_tiles * opc::kTileRows && p->K_pad == p->k_units * unit_cols(p->sub_vector_size) &&
         p->outlier_tiles == ceil_div(p->n_outliers, opc::kTileRows) &&
         p->outlier_k_units == p->K_pad / opc::kDenseCols &&
         p->packed_units == static_cast<int64_t>(p->row_tiles) * p->k_units &&
         p->total_units == p->packed_units + static_cast<int64_t>(p->outlier_tiles) * p->outlier_k_units;
}

opc::Vq8Geom vq8_geom_of(const opc_layer_plan& p) {
  opc::Vq8Geom G;
  G.M = p.M;
  G.K = p.K;
  G.K_pad = p.K_pad;
  G.MT = p.row_tiles;
  G.KB = p.k_units;
  G.n_slots = std::max(p.outlier_tiles, 1) * opc::kTileRows;
  return G;
}

opc::LayerGeom geom_of(const opc_layer_plan& p) {
  opc::LayerGeom G;
  G.Up = p.packed_units;
  G.U = p.total_units;
  G.M = p.M;
  G.K = p.K;
  G.K_pad = p.K_pad;
  G.M_pad = p.M_pad;
  G.MT = p.row_tiles;
  G.KT = p.k_units;
  G.OT = p.outlier_tiles;
  G.KO = p.outlier_k_units;
  return G;
}

// ---------------------------------------------------------------------------
// GEMV launch configuration.
// ---------------------------------------------------------------------------
constexpr int kCtasPerSm = 2;
#ifndef OPC_XS_MAX_BYTES
#define OPC_XS_MAX_BYTES (96 * 1024)  // largest x copy staged in shared memory
#endif
constexpr int kXsMaxBytes = OPC_XS_MAX_BYTES;
constexpr int kMaxBatch = 64;
// opc_gemv runs batches above this on the prefill GEMM (opc_set_gemm_crossover)
std::atomic<int> g_gemm_crossover{8};

int nt_for_batch(int batch) {
  if (batch <= 8) return 1;
  if (batch <= 16) return 2;
  if (batch <= 32) return 4;
  return 8;
}

// At most kCtasPerSm CTAs per SM and at least one unit per warp where the layer allows (the
// kernel's partition needs grid <= total units, which this guarantees).
int64_t gemv_grid(const opc_layer_plan& p, int sm_count) {
  const int64_t by_units = std::max<int64_t>(1, p.total_units / opc::kGemvWarps);
  return std::min<int64_t>(static_cast<int64_t>(sm_count) * kCtasPerSm, by_units);
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Cross-CTA partial sums: two slots of NT*128 floats per CTA.
size_t slots_bytes(int sm_count, int nt) {
  const int64_t ctas_max = static_cast<int64_t>(sm_count) * kCtasPerSm;
  return static_cast<size_t>(ctas_max) * 2 * nt * 128 * sizeof(float);
}

// Workspace layout: [fp16-kernel partial-sum slots sized for the largest batch | per-segment
// counters | int8-kernel int64 accumulators].  The counters sit at the same offset for every
// batch and every layer, so one zeroed workspace can serve any sequence of calls: counters and
// accumulators are zero between calls (each finisher resets what it used) and the slot area is
// plain scratch.  The accumulators of a large layer may overlap the counters of a smaller one;
// both are zero whenever no call is running.
size_t counters_offset(int sm_count) { return align_up(slots_bytes(sm_count, nt_for_batch(kMaxBatch)), 256); }
size_t acc_offset(const opc_layer_plan& p, int sm_count) {
  return counters_offset(sm_count) + align_up(static_cast<size_t>(p.row_tiles + p.outlier_tiles) * sizeof(int32_t), 256);
}

// Launch shape of the prefill GEMM for n_tok tokens: token tile tn (16..256), stage depth (64 x sub
// columns; sub 2 for tiles of up to 64 tokens) and K split, chosen by the least estimated time --
// waves of persistent items (one CTA per SM) times the 64-column steps of an item times the cost
// of a step: the largest of the MMA warp's per-stage work ((550 + 200 sub) / sub cycles: barrier
// waits, commit and loop ~550, each tcgen05.mma ~50, measured), the decode (~330) and the tensor
// time (~2.8 N for 128 x N x 64 on one SM).  A K split (only with a workspace, split_ok) cuts a tile
// into items of at least 16 steps whose fp32 partials are added in a fixed order.
struct GemmPlan {
  int tn = 16, sub = 1, ksplit = 1, nk_slice = 1;   // nk_slice in stages of 64 x sub columns
  int64_t tiles = 0;        // (packed M tiles + dense tiles) x token tiles
  size_t split_bytes = 0;   // workspace of the split: [tiles][4] counters, then the fp32 partials
};
// Stage depth of a token tile: two 64-column sub-tiles for N <= 64 (their stages still fit four
// deep in shared memory), one above.
int gemm_sub(int N) { return N <= 64 ? 2 : 1; }

GemmPlan gemm_plan(const opc_layer_plan& p, int n_tok, int sm_count, bool split_ok) {
  const int64_t m_tiles = ceil_div(p.M_pad, opc::kGmM);
  const int64_t d_tiles = p.n_outliers > 0 ? ceil_div(static_cast<int64_t>(p.outlier_tiles) * opc::kTileRows, opc::kGmM) : 0;
  GemmPlan best;
  double best_cost = -1.0;
  for (int N = 16; N <= 256; N *= 2) {
    if (N > 16 && N / 2 >= n_tok) break;  // a smaller tile already covers every token
    const int sub = gemm_sub(N);
    const int nk = p.K_pad / (opc::kGmK * sub);  // K_pad is a multiple of 128
    const double step = std::max({(550.0 + 200.0 * sub) / sub, 330.0, 2.8 * N});
    const int64_t tiles = (m_tiles + d_tiles) * ceil_div(n_tok, N);
    for (int S = 1; S <= (split_ok ? opc::kGmMaxSplit : 1); ++S) {
      const int slice = static_cast<int>(ceil_div(nk, S));
      // a split only for layers with fewer tiles than SMs, into one wave of items of >= 16 steps
      if (S > 1 && (tiles >= sm_count || tiles * S > sm_count || slice * sub < 16 || ceil_div(nk, slice) != S)) continue;
      const double waves = static_cast<double>(ceil_div(tiles * S, sm_count));
      // + the split's epilogue: partials out, and the last arrival reading and adding them
      const double cost = waves * slice * sub * step + (S > 1 ? 3000.0 + 500.0 * S : 0.0);
      if (best_cost < 0.0 || cost < best_cost) {
        best_cost = cost;
        best.tn = N;
        best.sub = sub;
        best.ksplit = S;
        best.nk_slice = slice;
        best.tiles = tiles;
      }
    }
  }
  if (best.ksplit > 1)
    best.split_bytes = align_up(static_cast<size_t>(best.tiles) * 4 * sizeof(int32_t), 256) +
                       static_cast<size_t>(best.tiles) * best.ksplit * opc::kGmM * best.tn * sizeof(float);
  return best;
}

int gemm_run(const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t n_tok, void* ws,
             size_t ws_bytes, void* stream_v);

// The opc_gemv workspace proper (partial-sum slots, counters, int64 accumulators), before the
// part a GEMM with a K split uses for batches routed to it.
size_t gemv_workspace_base(const opc_layer_plan& p, int sm_count);

size_t workspace_bytes(const opc_layer_plan& p, int batch, int sm_count) {
  // batches above 8 may be routed to the GEMM (opc_set_gemm_crossover): room for its K split
  const size_t split = batch > 8 ? align_up(gemm_plan(p, batch, sm_count, true).split_bytes, 256) : 0;
  return gemv_workspace_base(p, sm_count) + split;
}

size_t gemv_workspace_base(const opc_layer_plan& p, int sm_count) {
  return acc_offset(p, sm_count) + static_cast<size_t>(p.M_pad) * opc::kQMaxBatch * sizeof(unsigned long long);
}

// Byte offsets inside the layer buffers (see opc_layer.cuh).
int64_t outlier_units(const opc_layer_plan& p) { return p.total_units - p.packed_units; }
const uint8_t* ounits_q(const opc_layer* L) { return static_cast<const uint8_t*>(L->units) + L->plan.packed_units * opc::kUnitBytes; }
const uint8_t* ounits_h(const opc_layer* L) {
  return static_cast<const uint8_t*>(L->units) + (L->plan.packed_units + outlier_units(L->plan)) * opc::kUnitBytes;
}
const uint4* codebooks_q(const opc_layer* L) {
  return reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(L->codebooks) + static_cast<int64_t>(L->plan.M_pad) * 8);
}
int n_slots_of(const opc_layer_plan& p) { return std::max(p.outlier_tiles, 1) * opc::kTileRows; }
const __half* dense_outliers(const opc_layer* L) {
  return reinterpret_cast<const __half*>(static_cast<const uint8_t*>(L->units) +
                                         (2 * L->plan.total_units - L->plan.packed_units) * opc::kUnitBytes);
}

template <int NT, bool XS>
int launch_gemv_t(const opc::GemvArgs& args, int64_t grid, size_t smem, cudaStream_t stream, int dev) {
  auto kern = opc::gemv_kernel<NT, XS>;
  static std::mutex mu;
  static std::map<int, size_t> configured;  // device -> dynamic smem limit already set
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = configured.find(dev);
    if (it == configured.end() || it->second < smem) {
      OPC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
               "cudaFuncSetAttribute(max dynamic smem)");
      configured[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(opc::kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OPC_CUDA(cudaLaunchKernelEx(&cfg, kern, args), "launch gemv_kernel");
  return OPC_OK;
}

template <int NT>
int launch_gemv_nt(const opc::GemvArgs& a, bool xs, int64_t grid, size_t smem, cudaStream_t s, int dev) {
  return xs ? launch_gemv_t<NT, true>(a, grid, smem, s, dev) : launch_gemv_t<NT, false>(a, grid, smem, s, dev);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// int8 kernel: shared memory for `stages` ring stages per consumer warp.
size_t gemvq_smem(int xs_bytes, int stages) {
  return static_cast<size_t>(xs_bytes) + static_cast<size_t>(opc::kQConsumers) * stages * (opc::kQChunkBytes + 16) +
         sizeof(opc::SmemSlotsQ);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <int kN, int kSub>
int launch_gemm_t(const CUtensorMap& tx, const CUtensorMap& tu, const CUtensorMap& td, const opc::GemmArgs& a,
                  unsigned grid, cudaStream_t stream, int dev) {
  static std::mutex mu;
  static std::map<int, bool> configured;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      OPC_CUDA(cudaFuncSetAttribute(opc::gemm_kernel<kN, kSub>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(opc::gm_smem_bytes(kN, kSub))),
               "cudaFuncSetAttribute(max dynamic smem, gemm)");
      configured[dev] = true;
    }
  }
  opc::gemm_kernel<kN, kSub><<<grid, opc::kGmThreads, opc::gm_smem_bytes(kN, kSub), stream>>>(tx, tu, td, a);
  OPC_CUDA(cudaGetLastError(), "launch gemm_kernel");
  return OPC_OK;
}

int launch_gemvq(const opc::GemvQArgs& args, int64_t grid, size_t smem, cudaStream_t stream, int dev) {
  static std::mutex mu;
  static std::map<int, size_t> configured;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = configured.find(dev);
    if (it == configured.end() || it->second < smem) {
      OPC_CUDA(cudaFuncSetAttribute(opc::gemvq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
               "cudaFuncSetAttribute(max dynamic smem, gemvq)");
      configured[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(opc::kQThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::gemvq_kernel, args), "launch gemvq_kernel");
  return OPC_OK;
}

}  // namespace

extern "C" {

const char* opc_version(void) { return OPC_VERSION_STRING; }

const char* opc_last_error(void) { return g_last_error; }

int opc_device_info(int32_t device, opc_device_props* out) {
  if (!out) return fail(OPC_ERR_INVALID, "opc_device_info: out is NULL");
  int n = 0;
  OPC_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(OPC_ERR_INVALID, "opc_device_info: device %d of %d", device, n);
  cudaDeviceProp p;
  OPC_CUDA(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
  memset(out, 0, sizeof(*out));
  strncpy(out->name, p.name, sizeof(out->name) - 1);
  out->device = device;
  out->sm_count = p.multiProcessorCount;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->total_mem_bytes = static_cast<int64_t>(p.totalGlobalMem);
  out->max_smem_per_block_optin = static_cast<int32_t>(p.sharedMemPerBlockOptin);
  out->max_threads_per_block = p.maxThreadsPerBlock;
  out->l2_bytes = p.l2CacheSize;
  out->warp_size = p.warpSize;
  return OPC_OK;
}

int opc_plan_layer(int32_t M, int32_t K, int32_t n_outliers, int32_t sub_vector_size, opc_layer_plan* plan) {
  if (!plan) return fail(OPC_ERR_INVALID, "opc_plan_layer: plan is NULL");
  if (M <= 0 || K <= 0) return fail(OPC_ERR_INVALID, "opc_plan_layer: bad shape M=%d K=%d", M, K);
  if (n_outliers < 0 || n_outliers > M)
    return fail(OPC_ERR_INVALID, "opc_plan_layer: n_outliers=%d outside [0, M=%d]", n_outliers, M);
  if (sub_vector_size != 1 && sub_vector_size != 8)
    return fail(OPC_ERR_UNSUPPORTED, "opc_plan_layer: sub_vector_size=%d (1 and 8 are implemented)", sub_vector_size);
  if (sub_vector_size == 8 && K % 8)
    return fail(OPC_ERR_UNSUPPORTED, "opc_plan_layer: K=%d is not a multiple of sub_vector_size 8", K);
  memset(plan, 0, sizeof(*plan));
  plan->M = M;
  plan->K = K;
  plan->n_outliers = n_outliers;
  plan->sub_vector_size = sub_vector_size;
  plan->row_tiles = static_cast<int32_t>(ceil_div(M, opc::kTileRows));
  plan->k_units = static_cast<int32_t>(ceil_div(K, unit_cols(sub_vector_size)));
  plan->M_pad = plan->row_tiles * opc::kTileRows;
  plan->K_pad = plan->k_units * unit_cols(sub_vector_size);
  plan->outlier_tiles = static_cast<int32_t>(ceil_div(n_outliers, opc::kTileRows));
  plan->outlier_k_units = plan->K_pad / opc::kDenseCols;
  plan->packed_units = static_cast<int64_t>(plan->row_tiles) * plan->k_units;
  plan->total_units = plan->packed_units + static_cast<int64_t>(plan->outlier_tiles) * plan->outlier_k_units;
  // units: packed, then the outlier units of the int8 kernel, then those of the fp16 kernel
  // and the row-major outlier rows of the prefill GEMM
  plan->units_bytes = (2 * plan->total_units - plan->packed_units) * opc::kUnitBytes +
                      static_cast<int64_t>(std::max(plan->outlier_tiles, 1)) * opc::kTileRows * plan->K_pad * 2;
  plan->codebook_bytes = static_cast<int64_t>(plan->M_pad) * (8 + 16);
  plan->tile_mask_bytes = static_cast<int64_t>(plan->row_tiles) * 2;
  plan->outlier_rows_bytes = static_cast<int64_t>(std::max(plan->outlier_tiles, 1)) * opc::kTileRows * 8;
  if (sub_vector_size == 8) {
    // 128-byte index units, then the outlier rows row-major; codebooks 64 bytes per row
    plan->units_bytes = plan->packed_units * opc::kVq8UnitBytes +
                        static_cast<int64_t>(std::max(plan->outlier_tiles, 1)) * opc::kTileRows * plan->K_pad * 2;
    plan->codebook_bytes = static_cast<int64_t>(plan->M_pad) * 64;
  }
  return OPC_OK;
}

int32_t opc_count_distinct_ids(const int64_t* ids, int32_t n) {
  if (!ids || n <= 0) return 0;
  std::vector<int64_t> v(ids, ids + n);
  std::sort(v.begin(), v.end());
  return static_cast<int32_t>(std::unique(v.begin(), v.end()) - v.begin());
}

int opc_repack_layer(const opc_layer* L, const void* codebooks_f16, const uint8_t* indices_u8, const void* outlier_f16,
                     const int64_t* outlier_ids, int32_t n_rows, void* stream_v) {
  if (!L || !plan_ok(&L->plan)) return fail(OPC_ERR_INVALID, "opc_repack_layer: invalid layer plan");
  const opc_layer_plan& p = L->plan;
  if (!L->units || !L->codebooks || !L->tile_mask || !L->outlier_rows)
    return fail(OPC_ERR_INVALID, "opc_repack_layer: layer buffers not allocated");
  if (!codebooks_f16 || !indices_u8) return fail(OPC_ERR_INVALID, "opc_repack_layer: codebooks/indices NULL");
  if (n_rows < 0 || (n_rows > 0 && (!outlier_ids || !outlier_f16)))
    return fail(OPC_ERR_INVALID, "opc_repack_layer: %d outlier rows but ids/values NULL", n_rows);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);

  // Effective outlier list: a repeated id keeps its last row; sorted by id.
  std::map<int64_t, int32_t> last_src;
  for (int32_t i = 0; i < n_rows; ++i) {
    const int64_t id = outlier_ids[i];
    if (id < 0 || id >= p.M)
      return fail(OPC_ERR_INVALID, "opc_repack_layer: outlier id %lld outside [0, %d)", static_cast<long long>(id), p.M);
    last_src[id] = i;
  }
  if (static_cast<int32_t>(last_src.size()) != p.n_outliers)
    return fail(OPC_ERR_INVALID, "opc_repack_layer: plan has %d outliers but the id list has %zu distinct ids",
                p.n_outliers, last_src.size());

  std::vector<uint16_t> mask(p.row_tiles, 0);
  const int n_slots = n_slots_of(p);
  std::vector<int32_t> orow(n_slots, -1), src(n_slots, -1);
  int s = 0;
  for (const auto& kv : last_src) {
    mask[kv.first / opc::kTileRows] |= static_cast<uint16_t>(1u << (kv.first % opc::kTileRows));
    orow[s] = static_cast<int32_t>(kv.first);
    src[s] = kv.second;
    ++s;
  }

  int32_t* d_src = nullptr;
  int* d_bad = nullptr;
  int rc = OPC_OK;
  auto cleanup = [&]() {
    if (d_src) cudaFree(d_src);
    if (d_bad) cudaFree(d_bad);
  };
#define OPC_REPACK_CUDA(call, what)      \
  do {                                   \
    cudaError_t e_ = (call);             \
    if (e_ != cudaSuccess) {             \
      rc = cuda_fail(e_, what);          \
      cleanup();                         \
      return rc;                         \
    }                                    \
  } while (0)

  OPC_REPACK_CUDA(cudaMalloc(&d_src, n_slots * sizeof(int32_t)), "cudaMalloc(repack slots)");
  OPC_REPACK_CUDA(cudaMalloc(&d_bad, sizeof(int)), "cudaMalloc(repack flag)");
  OPC_REPACK_CUDA(cudaMemsetAsync(d_bad, 0, sizeof(int), stream), "cudaMemsetAsync");
  OPC_REPACK_CUDA(cudaMemcpyAsync(L->tile_mask, mask.data(), mask.size() * 2, cudaMemcpyHostToDevice, stream),
                  "copy tile mask");
  OPC_REPACK_CUDA(cudaMemcpyAsync(L->outlier_rows, orow.data(), n_slots * 4, cudaMemcpyHostToDevice, stream),
                  "copy outlier rows");
  OPC_REPACK_CUDA(cudaMemcpyAsync(d_src, src.data(), n_slots * 4, cudaMemcpyHostToDevice, stream),
                  "copy outlier sources");

  const int tpb = 256;
  if (p.sub_vector_size == 8) {
    const opc::Vq8Geom V = vq8_geom_of(p);
    const int64_t n_idx_words = p.packed_units * (opc::kVq8UnitBytes / 4);
    opc::vq8_repack_indices_kernel<<<static_cast<unsigned>(ceil_div(n_idx_words, tpb)), tpb, 0, stream>>>(
        V, indices_u8, static_cast<uint32_t*>(L->units), d_bad);
    OPC_REPACK_CUDA(cudaGetLastError(), "launch vq8_repack_indices_kernel");
    const int64_t n_cb_words = static_cast<int64_t>(p.row_tiles) * 32 * 8;
    opc::vq8_repack_codebooks_kernel<<<static_cast<unsigned>(ceil_div(n_cb_words, tpb)), tpb, 0, stream>>>(
        V, static_cast<const uint16_t*>(codebooks_f16), static_cast<const uint16_t*>(L->tile_mask),
        static_cast<uint32_t*>(L->codebooks));
    OPC_REPACK_CUDA(cudaGetLastError(), "launch vq8_repack_codebooks_kernel");
    OPC_REPACK_CUDA(cudaMemsetAsync(L->outlier_rows + n_slots, 0, n_slots * 4, stream), "clear outlier exponents");
    const int64_t n_dense = static_cast<int64_t>(n_slots) * p.K_pad;
    opc::vq8_repack_outliers_kernel<<<static_cast<unsigned>(ceil_div(n_dense, tpb)), tpb, 0, stream>>>(
        V, static_cast<const uint16_t*>(outlier_f16), d_src,
        reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(L->units) + p.packed_units * opc::kVq8UnitBytes));
    OPC_REPACK_CUDA(cudaGetLastError(), "launch vq8_repack_outliers_kernel");
    int bad8 = 0;
    OPC_REPACK_CUDA(cudaMemcpyAsync(&bad8, d_bad, sizeof(int), cudaMemcpyDeviceToHost, stream), "read repack flag");
    OPC_REPACK_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(repack)");
    cleanup();
    if (bad8) return fail(OPC_ERR_INVALID, "opc_repack_layer: an index value is outside 0..3");
    return OPC_OK;
  }
  const opc::LayerGeom G = geom_of(p);
  const int64_t n_idx_words = p.packed_units * (opc::kUnitBytes / 4);
  opc::repack_indices_kernel<<<static_cast<unsigned>(ceil_div(n_idx_words, tpb)), tpb, 0, stream>>>(
      G, indices_u8, static_cast<uint32_t*>(L->units), d_bad);
  OPC_REPACK_CUDA(cudaGetLastError(), "launch repack_indices_kernel");
  opc::repack_codebooks_kernel<<<static_cast<unsigned>(ceil_div(p.M_pad, tpb)), tpb, 0, stream>>>(
      G, static_cast<const uint16_t*>(codebooks_f16), static_cast<const uint16_t*>(L->tile_mask),
      static_cast<uint2*>(L->codebooks), const_cast<uint4*>(codebooks_q(L)));
  OPC_REPACK_CUDA(cudaGetLastError(), "launch repack_codebooks_kernel");
  int32_t* oexp = L->outlier_rows + n_slots;
  int32_t* d_orow = L->outlier_rows;
  opc::outlier_exponent_kernel<<<static_cast<unsigned>(n_slots), tpb, 0, stream>>>(
      G, static_cast<const uint16_t*>(outlier_f16), d_src, d_orow, oexp, const_cast<uint4*>(codebooks_q(L)));
  OPC_REPACK_CUDA(cudaGetLastError(), "launch outlier_exponent_kernel");
  const int64_t n_out_words = outlier_units(p) * (opc::kUnitBytes / 4);
  if (n_out_words > 0) {
    opc::repack_outliers_kernel<<<static_cast<unsigned>(ceil_div(n_out_words, tpb)), tpb, 0, stream>>>(
        G, static_cast<const uint16_t*>(outlier_f16), d_src, oexp,
        reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(ounits_q(L))),
        reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(ounits_h(L))));
    OPC_REPACK_CUDA(cudaGetLastError(), "launch repack_outliers_kernel");
  }
  const int64_t n_dense = static_cast<int64_t>(n_slots) * p.K_pad;
  opc::repack_dense_outliers_kernel<<<static_cast<unsigned>(ceil_div(n_dense, tpb)), tpb, 0, stream>>>(
      G, static_cast<const uint16_t*>(outlier_f16), d_src, n_slots,
      reinterpret_cast<uint16_t*>(const_cast<__half*>(dense_outliers(L))));
  OPC_REPACK_CUDA(cudaGetLastError(), "launch repack_dense_outliers_kernel");
  int bad = 0;
  OPC_REPACK_CUDA(cudaMemcpyAsync(&bad, d_bad, sizeof(int), cudaMemcpyDeviceToHost, stream), "read repack flag");
  OPC_REPACK_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(repack)");
  cleanup();
#undef OPC_REPACK_CUDA
  if (bad) return fail(OPC_ERR_INVALID, "opc_repack_layer: an index value is outside 0..3");
  return OPC_OK;
}

size_t opc_gemv_workspace_bytes(const opc_layer_plan* plan, int32_t batch, int32_t device) {
  if (!plan || batch < 1) return 0;
  DeviceCache dc;
  if (device_cache(device, &dc) != OPC_OK) return 0;
  return workspace_bytes(*plan, std::min<int32_t>(batch, kMaxBatch), dc.sm_count);
}

int opc_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (!workspace && bytes) return fail(OPC_ERR_INVALID, "opc_workspace_init: NULL workspace");
  OPC_CUDA(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)), "cudaMemsetAsync(workspace)");
  return OPC_OK;
}

}  // extern "C"

namespace {
// svs = 8: one launch, no workspace (each CTA reduces its tile in shared memory).  `fn` names the
// entry point in error messages.
int launch_vq8(const char* fn, const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t batch,
               cudaStream_t s) {
  const opc_layer_plan& p = L->plan;
  opc::Vq8Args a;
  memset(&a, 0, sizeof(a));
  a.units = static_cast<const uint4*>(L->units);
  a.cb = static_cast<const uint4*>(L->codebooks);
  a.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
  a.orows = reinterpret_cast<const __half*>(static_cast<const uint8_t*>(L->units) + p.packed_units * opc::kVq8UnitBytes);
  a.orow = L->outlier_rows;
  a.x = static_cast<const __half*>(x);
  a.y = static_cast<__half*>(y);
  a.ldx = ldx;
  a.ldy = ldy;
  a.M = p.M;
  a.K = p.K;
  a.K_pad = p.K_pad;
  a.MT = p.row_tiles;
  a.KB = p.k_units;
  a.OT = p.n_outliers > 0 ? p.outlier_tiles : 0;
  a.batch = batch;
  a.x_vec16 = aligned(x, 16) && ldx % 8 == 0;
  // batch columns per CTA: as many of 8 as the staged x allows
  const size_t col_bytes = static_cast<size_t>(p.K_pad + 8) * 2;
  int nc = 8;
  while (nc > 1 && static_cast<size_t>(nc) * col_bytes > static_cast<size_t>(opc::kVq8XsMaxBytes)) nc >>= 1;
  while (nc > 1 && nc / 2 >= batch) nc >>= 1;
  if (col_bytes > static_cast<size_t>(opc::kVq8XsMaxBytes))
    return fail(OPC_ERR_UNSUPPORTED, "%s: K=%d too large for the svs=8 kernel's staged x", fn, p.K);
  a.nc = nc;
  const size_t smem = static_cast<size_t>(nc) * col_bytes;
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  {
    // the dynamic shared-memory limit is a per-device function attribute: set it once on every
    // device the kernel runs on
    static std::mutex mu;
    static std::map<int, bool> configured;
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      OPC_CUDA(cudaFuncSetAttribute(opc::vq8_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    opc::kVq8XsMaxBytes),
               "cudaFuncSetAttribute(max dynamic smem, vq8_gemv)");
      configured[dev] = true;
    }
  }
  const dim3 grid(static_cast<unsigned>(p.row_tiles + a.OT), static_cast<unsigned>(ceil_div(batch, nc)));
  opc::vq8_gemv_kernel<<<grid, opc::kVq8Warps * 32, smem, s>>>(a);
  OPC_CUDA(cudaGetLastError(), "launch vq8_gemv_kernel");
  return OPC_OK;
}
int launch_gemvd(const opc::GemvDArgs& args, int64_t grid, size_t smem, cudaStream_t stream, int dev) {
  static std::mutex mu;
  static std::map<int, size_t> configured;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = configured.find(dev);
    if (it == configured.end() || it->second < smem) {
      OPC_CUDA(cudaFuncSetAttribute(opc::gemvd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
               "cudaFuncSetAttribute(max dynamic smem, gemvd)");
      configured[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(opc::kDThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::gemvd_kernel, args), "launch gemvd_kernel");
  return OPC_OK;
}

}  // namespace

extern "C" {

int opc_gemv(const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t batch, void* workspace,
             size_t workspace_bytes_given, void* stream_v) {
  if (!L || !plan_ok(&L->plan)) return fail(OPC_ERR_INVALID, "opc_gemv: invalid layer plan");
  const opc_layer_plan& p = L->plan;
  if (!L->units || !L->codebooks || !L->tile_mask || !L->outlier_rows)
    return fail(OPC_ERR_INVALID, "opc_gemv: layer buffers not allocated");
  if (batch < 1 || batch > kMaxBatch) return fail(OPC_ERR_INVALID, "opc_gemv: batch %d outside [1, %d]", batch, kMaxBatch);
  if (!x || !y) return fail(OPC_ERR_INVALID, "opc_gemv: x or y is NULL");
  if (ldx < p.K || ldy < p.M)
    return fail(OPC_ERR_INVALID, "opc_gemv: ldx=%lld < K=%d or ldy=%lld < M=%d", static_cast<long long>(ldx), p.K,
                static_cast<long long>(ldy), p.M);
  if (!aligned(x, 2) || !aligned(y, 2)) return fail(OPC_ERR_INVALID, "opc_gemv: x/y not 2-byte aligned");
  if (!aligned(L->units, 16) || !aligned(L->codebooks, 16))
    return fail(OPC_ERR_INVALID, "opc_gemv: layer buffers misaligned (units and codebooks 16 B)");
  if (p.sub_vector_size == 8)
    return launch_vq8("opc_gemv", L, x, ldx, y, ldy, batch, static_cast<cudaStream_t>(stream_v));
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  const size_t need = workspace_bytes(p, batch, dc.sm_count);
  if (!workspace || workspace_bytes_given < need || !aligned(workspace, 256))
    return fail(OPC_ERR_WORKSPACE, "opc_gemv: workspace %zu bytes at %p, need %zu (256-byte aligned, zeroed)",
                workspace_bytes_given, workspace, need);

  const int nt = nt_for_batch(batch);
  if (p.total_units >= (int64_t(1) << 31)) return fail(OPC_ERR_UNSUPPORTED, "opc_gemv: layer too large (2^31 units)");
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);

  // Batches above the crossover (default 8): the tcgen05 GEMM when x can be read with TMA
  // (measured, L2 flushed: faster than the fp16 GEMV from batch 16 on on every Llama-3.1-8B and
  // Llama-3-70B projection -- 1.3-1.8x at 16 rows, 4-20x at 64 -- slower at 8).
  if (batch > g_gemm_crossover.load(std::memory_order_relaxed) && aligned(x, 16) && ldx % 8 == 0) {
    const size_t base = gemv_workspace_base(p, dc.sm_count);
    return gemm_run(L, x, ldx, y, ldy, batch, static_cast<char*>(workspace) + base, workspace_bytes_given - base,
                    stream_v);
  }

  // Batch 1..2: the integer kernel, when its staged x and at least two ring stages fit.
  if (batch <= opc::kQMaxBatch) {
    const int xs_q = static_cast<int>(align_up(static_cast<size_t>(3 * batch) * opc::xsq_col_bytes(p.k_units) +
                                                   opc::kQZeroBytes + opc::kQOnesBytes, 128));
    // The single-launch kernel (opc_gemvd.cuh) when its staged x and unit rings fit, its 32-bit
    // unit arithmetic holds and the count-carrying sums stay exact (K <= 2^15); else gemvq_kernel.
    const size_t smem_d = static_cast<size_t>(xs_q) + opc::kDRingBytes;
    const int64_t grid_d = std::min<int64_t>(dc.sm_count, std::max<int64_t>(1, ceil_div(p.total_units, opc::kDWarps)));
    const int64_t nw_d = std::min<int64_t>(grid_d * opc::kDWarps, p.total_units);
    if (smem_d + 1024 <= static_cast<size_t>(dc.max_smem_optin) && p.K <= 32768 &&
        static_cast<uint64_t>(nw_d) * static_cast<uint64_t>(p.total_units) < (1ull << 32)) {
      opc::GemvDArgs d;
      memset(&d, 0, sizeof(d));
      d.units = static_cast<const uint8_t*>(L->units);
      d.ounits = ounits_q(L);
      d.cbq = codebooks_q(L);
      d.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
      d.orow = L->outlier_rows;
      d.oexp = L->outlier_rows + n_slots_of(p);
      d.x = static_cast<const __half*>(x);
      d.y = static_cast<__half*>(y);
      d.acc = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + acc_offset(p, dc.sm_count));
      d.ldx = ldx;
      d.ldy = ldy;
      d.Up = static_cast<int32_t>(p.packed_units);
      d.U = static_cast<int32_t>(p.total_units);
      d.NW = static_cast<int32_t>(nw_d);
      d.M = p.M;
      d.K = p.K;
      d.K_pad = p.K_pad;
      d.MT = p.row_tiles;
      d.KT = p.k_units;
      d.OT = p.outlier_tiles;
      d.KO = p.outlier_k_units;
      d.batch = batch;
      d.xs_bytes = xs_q;
      d.x_vec16 = (p.K % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16);
      d.negz = opc::kNegZero2;
      return launch_gemvd(d, grid_d, smem_d, s, dev);
    }
    int stages = opc::kQMaxStages;
    while (stages >= 2 && gemvq_smem(xs_q, stages) > static_cast<size_t>(dc.max_smem_optin)) --stages;
    if (stages >= 2) {
      opc::GemvQArgs q;
      memset(&q, 0, sizeof(q));
      q.units = static_cast<const uint8_t*>(L->units);
      q.ounits = ounits_q(L);
      q.cbq = codebooks_q(L);
      q.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
      q.orow = L->outlier_rows;
      q.oexp = L->outlier_rows + n_slots_of(p);
      q.x = static_cast<const __half*>(x);
      q.y = static_cast<__half*>(y);
      q.acc = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + acc_offset(p, dc.sm_count));
      q.counters = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + counters_offset(dc.sm_count));
      q.ldx = ldx;
      q.ldy = ldy;
      q.Up = static_cast<int32_t>(p.packed_units);
      q.U = static_cast<int32_t>(p.total_units);
      q.M = p.M;
      q.K = p.K;
      q.K_pad = p.K_pad;
      q.MT = p.row_tiles;
      q.KT = p.k_units;
      q.OT = p.outlier_tiles;
      q.KO = p.outlier_k_units;
      q.batch = batch;
      q.stages = stages;
      q.xs_bytes = xs_q;
      q.x_vec16 = (p.K % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16);
      q.negz = opc::kNegZero2;
      const int64_t grid = std::min<int64_t>(dc.sm_count, std::max<int64_t>(1, p.total_units / opc::kQConsumers));
      return launch_gemvq(q, grid, gemvq_smem(xs_q, stages), s, dev);
    }
  }

  opc::GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.units = static_cast<const uint8_t*>(L->units);
  a.ounits = ounits_h(L);
  a.cb = static_cast<const uint2*>(L->codebooks);
  a.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
  a.orow = L->outlier_rows;
  a.x = static_cast<const __half*>(x);
  a.y = static_cast<__half*>(y);
  a.gslots = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + counters_offset(dc.sm_count));
  a.ldx = ldx;
  a.ldy = ldy;
  a.Up = static_cast<int32_t>(p.packed_units);
  a.U = static_cast<int32_t>(p.total_units);
  a.M = p.M;
  a.K = p.K;
  a.K_pad = p.K_pad;
  a.MT = p.row_tiles;
  a.KT = p.k_units;
  a.OT = p.outlier_tiles;
  a.KO = p.outlier_k_units;
  a.batch = batch;
  a.x_vec16 = (p.K % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16);
  a.x_vec8 = (p.K % 4 == 0) && (ldx % 4 == 0) && aligned(x, 8);
  a.negz = opc::kNegZero2;
  // x rows 0..batch-1 plus a 64-byte zero block (the B operand of absent batch columns).
  const size_t xs_bytes = align_up(static_cast<size_t>(batch) * opc::xs_row_bytes(p.k_units) + 64, 128);
  const bool xs = xs_bytes <= static_cast<size_t>(kXsMaxBytes);
  a.xs_bytes = xs ? static_cast<int32_t>(xs_bytes) : 0;
  const size_t slots_smem = static_cast<size_t>(opc::kGemvWarps) * 2 * nt * 128 * sizeof(float) + opc::kGemvWarps * 2 * sizeof(int32_t);
  const size_t smem = a.xs_bytes + static_cast<size_t>(opc::kGemvWarps) * (opc::kRingBytesPerWarp + opc::kBarBytesPerWarp) + slots_smem;
  if (smem > static_cast<size_t>(dc.max_smem_optin))
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemv: needs %zu bytes of shared memory, device allows %d", smem,
                dc.max_smem_optin);
  const int64_t grid = gemv_grid(p, dc.sm_count);
  switch (nt) {
    case 1: return launch_gemv_nt<1>(a, xs, grid, smem, s, dev);
    case 2: return launch_gemv_nt<2>(a, xs, grid, smem, s, dev);
    case 4: return launch_gemv_nt<4>(a, xs, grid, smem, s, dev);
    default: return launch_gemv_nt<8>(a, xs, grid, smem, s, dev);
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Allocation-free GEMV.  Some callers of this library cannot allocate device memory: a plugin
// host that hands its plugins only preallocated input and output buffers, or a serving process
// whose whole device memory is owned by its own pool, where a cudaMalloc would fail or would
// go unaccounted.  For them the GEMV's scratch (cross-CTA partial sums and per-tile counters)
// lives in this file-scope device array instead of a caller workspace.  It is 448 KiB, and
// every GPU that loads the library keeps it until the process exits.
// ---------------------------------------------------------------------------------------------
namespace {

constexpr int kStaticMaxCtas = 384;         // grid cap of the allocation-free variant
constexpr int kStaticMaxSegments = 16384;   // row tiles + outlier tiles of the largest layer
constexpr int kStaticMaxBatch = 8;          // one n-tile of partial sums per slot
constexpr size_t kStaticSlotsBytes = static_cast<size_t>(kStaticMaxCtas) * 2 * 128 * sizeof(float);
constexpr size_t kStaticScratchBytes = kStaticSlotsBytes + static_cast<size_t>(kStaticMaxSegments) * sizeof(int32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kStaticScratchBytes];

std::mutex g_noalloc_mu;
std::map<int, void*> g_noalloc_ptr;  // device -> device address of g_noalloc_scratch

// Device address of the scratch array on the current device.  In host code the array's name
// only stands in for the symbol, so the address is looked up once per device, with that device
// current, and cached.
int noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_ptr.find(dev);
  if (it == g_noalloc_ptr.end()) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(allocation-free GEMV scratch)");
    it = g_noalloc_ptr.emplace(dev, p).first;
  }
  *out = it->second;
  return OPC_OK;
}

}  // namespace

extern "C" {

int opc_gemv_noalloc(const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t batch,
                     void* stream_v) {
  if (!L || !plan_ok(&L->plan)) return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: invalid layer plan");
  const opc_layer_plan& p = L->plan;
  if (!L->units || !L->codebooks || !L->tile_mask || !L->outlier_rows)
    return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: layer buffers not allocated");
  if (batch < 1 || batch > kStaticMaxBatch)
    return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: batch %d outside [1, %d] (the static scratch holds one n-tile)",
                batch, kStaticMaxBatch);
  if (!x || !y) return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: x or y is NULL");
  if (ldx < p.K || ldy < p.M)
    return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: ldx=%lld < K=%d or ldy=%lld < M=%d", static_cast<long long>(ldx),
                p.K, static_cast<long long>(ldy), p.M);
  if (!aligned(x, 2) || !aligned(y, 2)) return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: x/y not 2-byte aligned");
  if (!aligned(L->units, 16) || !aligned(L->codebooks, 16))
    return fail(OPC_ERR_INVALID, "opc_gemv_noalloc: layer buffers misaligned (units and codebooks 16 B)");
  // sub_vector_size 8 reduces each tile inside its CTA and needs no scratch at all
  if (p.sub_vector_size == 8)
    return launch_vq8("opc_gemv_noalloc", L, x, ldx, y, ldy, batch, static_cast<cudaStream_t>(stream_v));
  if (static_cast<int64_t>(p.row_tiles) + p.outlier_tiles > kStaticMaxSegments)
    return fail(OPC_ERR_INVALID,
                "opc_gemv_noalloc: %d row tiles + %d outlier tiles exceed the static scratch limit of %d tiles "
                "(M up to %d rows); use opc_gemv with a workspace",
                p.row_tiles, p.outlier_tiles, kStaticMaxSegments, kStaticMaxSegments * opc::kTileRows);
  if (p.total_units >= (int64_t(1) << 31))
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemv_noalloc: layer too large (2^31 units)");
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc != OPC_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  int32_t* counters = reinterpret_cast<int32_t*>(static_cast<char*>(scratch) + kStaticSlotsBytes);
  // The counters must start at zero.  Each call's finishers leave them zero, but the array
  // outlives any one call, so clear this layer's counters explicitly (no allocation involved).
  OPC_CUDA(cudaMemsetAsync(counters, 0, (static_cast<size_t>(p.row_tiles) + p.outlier_tiles) * sizeof(int32_t), s),
           "cudaMemsetAsync(static scratch counters)");

  opc::GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.units = static_cast<const uint8_t*>(L->units);
  a.ounits = ounits_h(L);
  a.cb = static_cast<const uint2*>(L->codebooks);
  a.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
  a.orow = L->outlier_rows;
  a.x = static_cast<const __half*>(x);
  a.y = static_cast<__half*>(y);
  a.gslots = static_cast<float*>(scratch);
  a.counters = counters;
  a.ldx = ldx;
  a.ldy = ldy;
  a.Up = static_cast<int32_t>(p.packed_units);
  a.U = static_cast<int32_t>(p.total_units);
  a.M = p.M;
  a.K = p.K;
  a.K_pad = p.K_pad;
  a.MT = p.row_tiles;
  a.KT = p.k_units;
  a.OT = p.outlier_tiles;
  a.KO = p.outlier_k_units;
  a.batch = batch;
  a.x_vec16 = (p.K % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16);
  a.x_vec8 = (p.K % 4 == 0) && (ldx % 4 == 0) && aligned(x, 8);
  a.negz = opc::kNegZero2;
  const size_t xs_bytes = align_up(static_cast<size_t>(batch) * opc::xs_row_bytes(p.k_units) + 64, 128);
  const bool xs = xs_bytes <= static_cast<size_t>(kXsMaxBytes);
  a.xs_bytes = xs ? static_cast<int32_t>(xs_bytes) : 0;
  const size_t slots_smem = static_cast<size_t>(opc::kGemvWarps) * 2 * 128 * sizeof(float) + opc::kGemvWarps * 2 * sizeof(int32_t);
  const size_t smem = a.xs_bytes + static_cast<size_t>(opc::kGemvWarps) * (opc::kRingBytesPerWarp + opc::kBarBytesPerWarp) + slots_smem;
  if (smem > static_cast<size_t>(dc.max_smem_optin))
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemv_noalloc: needs %zu bytes of shared memory, device allows %d", smem,
                dc.max_smem_optin);
  const int64_t grid = std::min<int64_t>(gemv_grid(p, dc.sm_count), kStaticMaxCtas);
  return launch_gemv_nt<1>(a, xs, grid, smem, s, dev);
}

int opc_dequant(const opc_layer* L, void* w, int64_t ldw, void* stream_v) {
  if (!L || !plan_ok(&L->plan)) return fail(OPC_ERR_INVALID, "opc_dequant: invalid layer plan");
  const opc_layer_plan& p = L->plan;
  if (!w || ldw < p.K) return fail(OPC_ERR_INVALID, "opc_dequant: bad output (ldw=%lld, K=%d)", static_cast<long long>(ldw), p.K);
  if (!aligned(L->units, 16)) return fail(OPC_ERR_INVALID, "opc_dequant: units not 16-byte aligned");
  if (p.sub_vector_size == 8) {
    const opc::Vq8Geom V = vq8_geom_of(p);
    const int64_t n = static_cast<int64_t>(p.M) * p.K;
    opc::vq8_dequant_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, static_cast<cudaStream_t>(stream_v)>>>(
        V, static_cast<const uint32_t*>(L->units), static_cast<const uint32_t*>(L->codebooks),
        static_cast<const uint16_t*>(L->tile_mask),
        reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(L->units) + p.packed_units * opc::kVq8UnitBytes),
        L->outlier_rows, static_cast<__half*>(w), ldw);
    OPC_CUDA(cudaGetLastError(), "launch vq8_dequant_kernel");
    return OPC_OK;
  }
  const opc::LayerGeom G = geom_of(p);
  const int warps = 8;
  opc::dequant_kernel<<<static_cast<unsigned>(ceil_div(p.total_units, warps)), warps * 32, 0,
                        static_cast<cudaStream_t>(stream_v)>>>(
      G, static_cast<const uint8_t*>(L->units), ounits_h(L), static_cast<const uint2*>(L->codebooks),
      static_cast<const uint16_t*>(L->tile_mask), L->outlier_rows, static_cast<uint16_t*>(w), ldw);
  OPC_CUDA(cudaGetLastError(), "launch dequant_kernel");
  return OPC_OK;
}

}  // extern "C"

namespace {

// The prefill GEMM for opc_gemm (no workspace) and for batches opc_gemv routes to it (its
// workspace past the GEMV's own part: `ws`, `ws_bytes`, which allow a K split).
int gemm_run(const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t n_tok, void* ws,
             size_t ws_bytes, void* stream_v) {
  if (!L || !plan_ok(&L->plan)) return fail(OPC_ERR_INVALID, "opc_gemm: invalid layer plan");
  const opc_layer_plan& p = L->plan;
  const bool svs8 = p.sub_vector_size == 8;
  if (!L->units || !L->codebooks || !L->tile_mask || !L->outlier_rows)
    return fail(OPC_ERR_INVALID, "opc_gemm: layer buffers not allocated");
  if (n_tok < 1) return fail(OPC_ERR_INVALID, "opc_gemm: n_tok %d < 1", n_tok);
  if (!x || !y) return fail(OPC_ERR_INVALID, "opc_gemm: x or y is NULL");
  if (ldx < p.K || ldy < p.M)
    return fail(OPC_ERR_INVALID, "opc_gemm: ldx=%lld < K=%d or ldy=%lld < M=%d", static_cast<long long>(ldx), p.K,
                static_cast<long long>(ldy), p.M);
  if (!aligned(x, 16) || ldx % 8 != 0)
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemm: x must be 16-byte aligned with ldx a multiple of 8 (TMA)");
  if (!aligned(y, 2)) return fail(OPC_ERR_INVALID, "opc_gemm: y not 2-byte aligned");
  if (!aligned(L->units, 16) || !aligned(L->codebooks, svs8 ? 16 : 8))
    return fail(OPC_ERR_INVALID, "opc_gemm: layer buffers misaligned");
  if (static_cast<int64_t>(n_tok) > (int64_t(65535) * 128))
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemm: n_tok %d too large", n_tok);
  auto encode = tensor_map_encoder();
  if (!encode) return fail(OPC_ERR_CUDA, "opc_gemm: cuTensorMapEncodeTiled unavailable");
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  GemmPlan gp = gemm_plan(p, n_tok, dc.sm_count, ws != nullptr);
  if (gp.ksplit > 1 && (ws_bytes < gp.split_bytes || !aligned(ws, 256))) gp = gemm_plan(p, n_tok, dc.sm_count, false);
  const int tn = gp.tn;
  const int64_t m_tiles = ceil_div(p.M_pad, opc::kGmM);
  if (opc::gm_smem_bytes(tn, gp.sub) > static_cast<size_t>(dc.max_smem_optin))
    return fail(OPC_ERR_UNSUPPORTED, "opc_gemm: needs %zu bytes of shared memory", opc::gm_smem_bytes(tn, gp.sub));

  CUtensorMap tx;
  const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(p.K), static_cast<cuuint64_t>(n_tok)};
  const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ldx) * 2};
  const cuuint32_t box[2] = {opc::kGmK, static_cast<cuuint32_t>(tn)};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult cr = encode(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), gdim, gstride, box, estride,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(OPC_ERR_CUDA, "opc_gemm: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(cr));
  // packed units as [MT][KT * unit bytes / 8] 8-byte elements: one box = one k block of 8 row tiles
  // (512-byte units of 128 columns; sub_vector_size 8: 128-byte units of 256 columns)
  CUtensorMap tu;
  {
    const int ub = svs8 ? opc::kVq8UnitBytes : opc::kUnitBytes;
    const cuuint64_t udim[2] = {static_cast<cuuint64_t>(p.k_units) * (ub / 8), static_cast<cuuint64_t>(p.row_tiles)};
    const cuuint64_t ustride[1] = {static_cast<cuuint64_t>(p.k_units) * ub};
    const cuuint32_t ubox[2] = {static_cast<cuuint32_t>(ub / 8), 8};
    const CUresult cu = encode(&tu, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(L->units), udim, ustride, ubox,
                               estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cu != CUDA_SUCCESS)
      return fail(OPC_ERR_CUDA, "opc_gemm: cuTensorMapEncodeTiled (units) failed (%d)", static_cast<int>(cu));
  }

  // the row-major outlier rows [slots][K_pad] fp16: a dense tile's A stage is one swizzled box
  const __half* dense = svs8 ? reinterpret_cast<const __half*>(static_cast<const uint8_t*>(L->units) +
                                                               p.packed_units * opc::kVq8UnitBytes)
                             : dense_outliers(L);
  CUtensorMap td;
  {
    const int64_t slots = std::max<int64_t>(p.outlier_tiles, 1) * opc::kTileRows;
    const cuuint64_t ddim[2] = {static_cast<cuuint64_t>(p.K_pad), static_cast<cuuint64_t>(slots)};
    const cuuint64_t dstride[1] = {static_cast<cuuint64_t>(p.K_pad) * 2};
    const cuuint32_t dbox[2] = {opc::kGmK, opc::kGmM};
    if (!aligned(dense, 16)) return fail(OPC_ERR_INVALID, "opc_gemm: outlier rows not 16-byte aligned");
    const CUresult cd = encode(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(dense), ddim, dstride, dbox,
                               estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cd != CUDA_SUCCESS)
      return fail(OPC_ERR_CUDA, "opc_gemm: cuTensorMapEncodeTiled (outlier rows) failed (%d)", static_cast<int>(cd));
  }

  opc::GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.units = static_cast<const uint8_t*>(L->units);
  a.cb = static_cast<const uint2*>(L->codebooks);
  a.cb8 = static_cast<const uint4*>(L->codebooks);
  a.svs8 = svs8 ? 1 : 0;
  a.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
  a.dense = dense;
  a.orow = L->outlier_rows;
  a.y = static_cast<__half*>(y);
  a.ldy = ldy;
  a.M = p.M;
  a.K_pad = p.K_pad;
  a.MT = p.row_tiles;
  a.KT = p.k_units;
  a.n_tok = n_tok;
  a.n_slots = p.outlier_tiles * opc::kTileRows;
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  a.m_tiles = static_cast<int32_t>(m_tiles);
  a.n_tiles = static_cast<int32_t>(ceil_div(n_tok, tn));
  const int64_t tiles = gp.tiles;
  if (tiles * gp.ksplit >= (int64_t(1) << 31)) return fail(OPC_ERR_UNSUPPORTED, "opc_gemm: too many tiles");
  a.tiles = static_cast<int32_t>(tiles);
  a.ksplit = gp.ksplit;
  a.nk_slice = gp.ksplit > 1 ? gp.nk_slice : p.K_pad / (opc::kGmK * gp.sub);
  if (gp.ksplit > 1) {
    a.cnt = static_cast<int32_t*>(ws);  // zero between calls: the last arrival of each count resets it
    a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + align_up(static_cast<size_t>(tiles) * 4 * sizeof(int32_t), 256));
  }
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(tiles * gp.ksplit, dc.sm_count));
  switch (tn) {
    case 256: return launch_gemm_t<256, 1>(tx, tu, td, a, grid, s, dev);
    case 128: return launch_gemm_t<128, 1>(tx, tu, td, a, grid, s, dev);
    case 64: return launch_gemm_t<64, 2>(tx, tu, td, a, grid, s, dev);
    case 32: return launch_gemm_t<32, 2>(tx, tu, td, a, grid, s, dev);
    default: return launch_gemm_t<16, 2>(tx, tu, td, a, grid, s, dev);
  }
}

}  // namespace

extern "C" {

int opc_gemm(const opc_layer* L, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t n_tok, void* stream_v) {
  return gemm_run(L, x, ldx, y, ldy, n_tok, nullptr, 0, stream_v);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode chain (persistent cooperative kernel), on one GPU or row-sharded over a node's GPUs.
// ---------------------------------------------------------------------------------------------
struct opc_chain {
  int device = 0;
  int32_t n_layers = 0, batch = 1, stages = 2, xs_bytes = 0, grid = 0, xc = 8;
  int32_t rank = 0, world = 1;
  size_t smem = 0;
  void* dev_mem = nullptr;              // [layers | onc | parts | epoch | acc (| flags | words)]
  opc::ChainLayer* d_layers = nullptr;
  const int4* d_parts = nullptr;        // [layers][grid][kChainSharePieces] warp-share records
  unsigned int* d_sync = nullptr;       // this rank's flags [world][grid]
  unsigned int* sync_peer[opc::kMaxRanks] = {};
  unsigned int* d_epoch = nullptr;      // [2]
  unsigned long long* trace = nullptr;  // optional per-phase timestamps (caller-owned)
  int32_t l2_prefetch = 0;
  // dataflow form (opc::chain2_kernel)
  int32_t form = OPC_CHAIN_FORM_BARRIER;
  int32_t nb0 = 0, nb1 = 0, s_total = 0;
  const opc::Chain2Layer* d_layers2 = nullptr;
  unsigned long long* d_s_all = nullptr;  // [2][s_total]
  std::vector<void*> owned;             // codebook and outlier forms of sub_vector_size-8 layers
  bool vq8 = false;                     // runs the kernel instance with those views
};

namespace {

// One rank of a chain as this process sees it (pointers valid in this process).
struct ChainRank {
  std::vector<int32_t> M;   // rows of its shard, per step
  std::vector<char*> y;     // row 0 of its fp16 copy of each step's full output
  std::vector<char*> yw;    // row 0 of its exchange words of each step's full output
  unsigned int* sync = nullptr;  // its flag array [world][grid]
};

int64_t chain_ldyw(int64_t ldy) { return (ldy + 7) / 8 * 8; }
size_t chain_words_bytes(int64_t ldy, int batch) {
  return align_up(static_cast<size_t>(batch) * chain_ldyw(ldy) * sizeof(uint32_t), 256);
}
size_t chain_sync_bytes(int world, int grid) {
  return align_up(static_cast<size_t>(world) * grid * sizeof(unsigned int), 256);
}

// Half-open byte ranges of a [rows x ld] fp16 matrix with `batch` rows of `cols` elements.
bool fp16_ranges_overlap(const void* a, int64_t lda, int64_t na, const void* b, int64_t ldb, int64_t nb, int batch) {
  const char* a0 = static_cast<const char*>(a);
  const char* b0 = static_cast<const char*>(b);
  const char* a1 = a0 + 2 * ((batch - 1) * lda + na);
  const char* b1 = b0 + 2 * ((batch - 1) * ldb + nb);
  return a0 < b1 && b0 < a1;
}

// One rank's steps against the kernel's limits; m_full[j] = rows of step j's full output.
struct Vq8View;
int check_chain_steps(const char* fn, const opc_chain_step* steps, int32_t n, int32_t batch, const DeviceCache& dc,
                      const std::vector<int32_t>& m_full, const std::vector<const Vq8View*>* views8 = nullptr) {
  if (n > opc::kChainMaxLayers) return fail(OPC_ERR_UNSUPPORTED, "%s: %d steps (at most %d)", fn, n, opc::kChainMaxLayers);
  for (int j = 0; j < n; ++j) {
    const opc_chain_step& st = steps[j];
    const bool view = views8 && (*views8)[j];  // an svs-8 layer's chain view (its plan was checked as svs 8)
    if (!st.layer || (!view && !plan_ok(&st.layer->plan)))
      return fail(OPC_ERR_INVALID, "%s: step %d: invalid layer", fn, j);
    if (st.layer->plan.sub_vector_size != 1)
      return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: sub_vector_size %d (the chain runs svs = 1)", fn, j,
                  st.layer->plan.sub_vector_size);
    const opc_layer* L = st.layer;
    const opc_layer_plan& p = L->plan;
    if (!L->units || !L->codebooks || !L->tile_mask || !L->outlier_rows || !aligned(L->units, 16))
      return fail(OPC_ERR_INVALID, "%s: step %d: layer buffers missing or misaligned", fn, j);
    if (!st.x || !st.y || st.ldx < p.K || st.ldy < m_full[j] || !aligned(st.x, 2) || !aligned(st.y, 2))
      return fail(OPC_ERR_INVALID, "%s: step %d: bad x/y (ldx=%lld K=%d ldy=%lld rows=%d)", fn, j,
                  static_cast<long long>(st.ldx), p.K, static_cast<long long>(st.ldy), m_full[j]);
    if (j > 0) {
      const opc_chain_step& pv = steps[j - 1];
      if (st.x != pv.y || st.ldx != pv.ldy || p.K > m_full[j - 1])
        return fail(OPC_ERR_UNSUPPORTED,
                    "%s: step %d: x must be the previous step's y (same pointer and leading dimension, K <= its "
                    "rows)", fn, j);
    }
    if (p.row_tiles / dc.sm_count + 2 > opc::kChainSplitSlots)
      return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: %d row tiles exceed %d per SM", fn, j, p.row_tiles,
                  opc::kChainSplitSlots - 2);
    if (static_cast<int64_t>(batch) * p.K_pad > 64 * opc::kQConsumerThreads)
      return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: batch*K_pad = %lld > %d", fn, j,
                  static_cast<long long>(batch) * p.K_pad, 64 * opc::kQConsumerThreads);
    // the kernel's warp ranges use 32-bit products of a share's size and the warp count
    if (p.total_units * (opc::kQConsumers + 1) >= (int64_t(1) << 31))
      return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: layer too large", fn, j);
  }
  // fp16 outputs: step 0's may not overlap the input; two steps' outputs are the same buffer
  // (then only the later one is written) or disjoint
  if (fp16_ranges_overlap(steps[0].x, steps[0].ldx, steps[0].layer->plan.K, steps[0].y, steps[0].ldy, m_full[0], batch))
    return fail(OPC_ERR_UNSUPPORTED, "%s: step 0 writes over its own input", fn);
  for (int i = 0; i < n; ++i)
    for (int j = i + 1; j < n; ++j) {
      if (!fp16_ranges_overlap(steps[i].y, steps[i].ldy, m_full[i], steps[j].y, steps[j].ldy, m_full[j], batch)) continue;
      if (steps[i].y != steps[j].y || steps[i].ldy != steps[j].ldy)
        return fail(OPC_ERR_UNSUPPORTED, "%s: outputs of steps %d and %d overlap without being the same buffer", fn, i, j);
    }
  return OPC_OK;
}

// Each CTA's share of a layer for the chain kernel (opc::chain_part): packed row tiles whole,
// outlier units evenly over all CTAs.  Measured: filling the least-loaded CTAs with the outlier
// units instead made the step 12% slower -- the outlier rows, completed by their last
// contributor, then finish late and every next layer waits for them.
std::vector<opc::ChainPart> chain_parts(const opc::ChainLayer& c, int G, int nw = opc::kQConsumers) {
  std::vector<opc::ChainPart> parts(G);
  for (int cta = 0; cta < G; ++cta) parts[cta] = opc::chain_part(c, cta, G, nw);
  return parts;
}

// Unit ranges of a CTA's consumer warps (out of nw, the other warps of the CTA being the producer
// and, in the dataflow form, the staging warp).  Packed warps split the packed share in proportion
// to their speed: the warps of an SM sub-partition (warp index mod 4) share its issue slots, and a
// sub-partition's packed warps run as fast as if each other busy warp on it (an outlier warp, the
// producer) were 0.4 of a packed warp (measured on the Llama-3.1-8B decode step: warps of a
// sub-partition with three packed warps and one other finish 1.18x faster per unit than those of a
// sub-partition with four packed warps).  Outlier warps split their share evenly.
void chain_warp_ranges(const opc::ChainPart& p, int nw, int32_t* u0, int32_t* u1) {
  constexpr int kCtaWarps = opc::kQConsumers + 1;  // consumer warps plus the producer (and staging) warps
  double busy[4] = {0, 0, 0, 0};
  for (int w = 0; w < kCtaWarps; ++w) busy[w % 4] += w < p.wp ? 1.0 : 0.4;
  double cum[opc::kQConsumers + 1];
  cum[0] = 0.0;
  for (int w = 0; w < p.wp; ++w) cum[w + 1] = cum[w] + 1.0 / busy[w % 4];
  const int32_t np = p.pu1 - p.pu0;
  for (int w = 0; w < nw; ++w) {
    if (w < p.wp) {
      u0[w] = p.pu0 + static_cast<int32_t>(std::lround(np * cum[w] / cum[p.wp]));
      u1[w] = p.pu0 + static_cast<int32_t>(std::lround(np * cum[w + 1] / cum[p.wp]));
    } else {
      opc::chain_warp_range(p, w, &u0[w], &u1[w], nw);
    }
  }
}

// Warps contributing to each outlier tile of a layer, for the kernel's completion counts.
std::vector<int32_t> outlier_contributors(const opc::ChainLayer& c, const std::vector<opc::ChainPart>& parts,
                                          int nw = opc::kQConsumers) {
  std::vector<int32_t> n(std::max(c.OT, 0), 0);
  for (const opc::ChainPart& p : parts) {
    for (int w = p.wp; w < nw; ++w) {
      int32_t u0 = 0, u1 = 0;
      opc::chain_warp_range(p, w, &u0, &u1, nw);
      if (u0 >= u1) continue;
      const int32_t t0 = (u0 - c.Up) / c.KO, t1 = (u1 - 1 - c.Up) / c.KO;
      for (int32_t t = t0; t <= t1; ++t) ++n[t];
    }
  }
  return n;
}

// Builds a chain from every rank's view (ranks[rank] is this process's own).  With own_scratch
// (one GPU) the flags and exchange words are allocated here and ranks[rank]'s pointers set.
// What the chain needs of a sub_vector_size-8 layer besides its own index units (streamed as is,
// four 128-byte units per 512-byte chain unit): the integer vector codebooks and row metadata
// (opc_layer.cuh, vq8_chain_vectors_kernel), and its outlier rows as the integer outlier units of
// the svs-1 kernels, taken from an svs-1 layer holding just those rows.  `L` describes the
// geometry the chain streams (units per row tile = K / 1024); its buffers are the svs-8 layer's
// except the ones below.  Device buffers owned by the chain.
struct Vq8View {
  opc_layer L{};
  uint4* cbq = nullptr;       // [M_pad] {0, 0, e, 0}
  uint4* cbv = nullptr;       // [M_pad][4] {hi[8], lo[8]} per vector
  const uint8_t* ounits = nullptr;
  int32_t* orow = nullptr;    // [slots] output row of each outlier slot, then [slots] exponents
  std::vector<void*> owned;
  void release() {
    for (void* p : owned) cudaFree(p);
    owned.clear();
  }
};

int make_vq8_view(const char* fn, int j, const opc_layer* L8, Vq8View* v) {
  const opc_layer_plan& p8 = L8->plan;
  if (p8.K % 1024 || p8.K_pad != p8.K)
    return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: sub_vector_size 8 on the chain needs K a multiple of 1024 (K=%d)",
                fn, j, p8.K);
  const int slots = n_slots_of(p8);
  std::vector<int32_t> orow(slots);
  OPC_CUDA(cudaMemcpy(orow.data(), L8->outlier_rows, slots * sizeof(int32_t), cudaMemcpyDeviceToHost),
           "vq8 view: outlier rows");
  int n = 0;  // valid slots come first (slots follow the sorted row ids)
  while (n < slots && orow[n] >= 0) ++n;
  for (int s = n; s < slots; ++s)
    if (orow[s] >= 0) return fail(OPC_ERR_INVALID, "%s: step %d: outlier slots not in order", fn, j);
  auto alloc = [&](void** ptr, size_t bytes) -> int {
    OPC_CUDA(cudaMalloc(ptr, std::max<size_t>(bytes, 16)), "vq8 view: cudaMalloc");
    v->owned.push_back(*ptr);
    return OPC_OK;
  };
  void *cbq = nullptr, *cbv = nullptr, *orw = nullptr;
  int rc;
  if ((rc = alloc(&cbq, static_cast<size_t>(p8.M_pad) * sizeof(uint4))) ||
      (rc = alloc(&cbv, static_cast<size_t>(p8.M_pad) * 4 * sizeof(uint4))) ||
      (rc = alloc(&orw, static_cast<size_t>(2 * slots) * sizeof(int32_t))))
    return rc;
  v->cbq = static_cast<uint4*>(cbq);
  v->cbv = static_cast<uint4*>(cbv);
  v->orow = static_cast<int32_t*>(orw);
  opc::vq8_chain_vectors_kernel<<<static_cast<unsigned>(ceil_div(p8.M_pad, 128)), 128>>>(
      p8.M, p8.M_pad, static_cast<const uint4*>(L8->codebooks), static_cast<const uint16_t*>(L8->tile_mask), v->cbv,
      v->cbq);
  OPC_CUDA(cudaGetLastError(), "vq8 view: vectors");
  OPC_CUDA(cudaMemcpy(v->orow, L8->outlier_rows, slots * sizeof(int32_t), cudaMemcpyDeviceToDevice), "vq8 view: rows");
  // outlier rows [n][K] fp16 (row-major, first in the svs-8 layer's copy since K_pad == K) as an
  // svs-1 layer whose rows are all outliers: its outlier units and slot exponents are the chain's
  if (n > 0) {
    opc_layer mini{};
    std::vector<int64_t> ids(n);
    for (int s = 0; s < n; ++s) ids[s] = s;
    if ((rc = opc_plan_layer(n, p8.K, n, 1, &mini.plan)) != OPC_OK) return rc;
    if (n_slots_of(mini.plan) != slots) return fail(OPC_ERR_INVALID, "%s: step %d: outlier slot count", fn, j);
    if ((rc = alloc(&mini.units, mini.plan.units_bytes)) || (rc = alloc(&mini.codebooks, mini.plan.codebook_bytes)) ||
        (rc = alloc(&mini.tile_mask, mini.plan.tile_mask_bytes)) ||
        (rc = alloc(reinterpret_cast<void**>(&mini.outlier_rows), mini.plan.outlier_rows_bytes)))
      return rc;
    void* tmp = nullptr;
    const size_t zb = static_cast<size_t>(n) * 4 * 2 + static_cast<size_t>(n) * p8.K;
    OPC_CUDA(cudaMalloc(&tmp, zb), "vq8 view: temporaries");
    cudaError_t e = cudaMemset(tmp, 0, zb);
    const uint8_t* rows8 = static_cast<const uint8_t*>(L8->units) + p8.packed_units * opc::kVq8UnitBytes;
    if (e == cudaSuccess)
      rc = opc_repack_layer(&mini, tmp, static_cast<uint8_t*>(tmp) + static_cast<size_t>(n) * 8, rows8, ids.data(), n,
                            nullptr);
    if (e == cudaSuccess && rc == OPC_OK)  // the exponents of the slots
      e = cudaMemcpy(v->orow + slots, mini.outlier_rows + slots, slots * sizeof(int32_t), cudaMemcpyDeviceToDevice);
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(e, "vq8 view: outlier units");
    if (rc != OPC_OK) return rc;
    v->ounits = ounits_q(&mini);
  } else {
    OPC_CUDA(cudaMemset(v->orow + slots, 0, slots * sizeof(int32_t)), "vq8 view: exponents");
    v->ounits = static_cast<const uint8_t*>(L8->units);  // never read (no outlier units)
  }
  OPC_CUDA(cudaDeviceSynchronize(), "vq8 view");
  // the geometry the chain streams: K/1024 chain units per row tile, the outlier units above
  opc_layer_plan q = p8;
  q.sub_vector_size = 1;
  q.k_units = p8.K / 1024;
  q.outlier_k_units = p8.K / 16;
  q.packed_units = static_cast<int64_t>(p8.row_tiles) * q.k_units;
  q.total_units = q.packed_units + static_cast<int64_t>(p8.outlier_tiles) * q.outlier_k_units;
  v->L.plan = q;
  v->L.units = L8->units;
  v->L.codebooks = v->cbq;
  v->L.tile_mask = L8->tile_mask;
  v->L.outlier_rows = v->orow;
  return OPC_OK;
}

int chain_build(const char* fn, const opc_chain_step* steps, int32_t n, int32_t batch, int32_t rank, int32_t world,
                std::vector<ChainRank>& ranks, bool own_scratch, opc_chain** out,
                const std::vector<const Vq8View*>* views8 = nullptr) {
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  std::vector<int32_t> m_full(n, 0), row_off(n, 0);
  for (int j = 0; j < n; ++j)
    for (int p = 0; p < world; ++p) {
      if (p < rank) row_off[j] += ranks[p].M[j];
      m_full[j] += ranks[p].M[j];
    }
  rc = check_chain_steps(fn, steps, n, batch, dc, m_full, views8);
  if (rc != OPC_OK) return rc;

  auto view8 = [&](int j) -> const Vq8View* { return views8 ? (*views8)[j] : nullptr; };
  int32_t kt_max = 1;  // 128-column blocks of the staged x
  int64_t bk_max = 0;
  for (int j = 0; j < n; ++j) {
    kt_max = std::max(kt_max, view8(j) ? steps[j].layer->plan.K / 128 : steps[j].layer->plan.k_units);
    bk_max = std::max<int64_t>(bk_max, static_cast<int64_t>(batch) * steps[j].layer->plan.K_pad);
  }
  const int xs = static_cast<int>(align_up(static_cast<size_t>(3 * batch) * opc::xsq_col_bytes(kt_max) +
                                          opc::kQZeroBytes + opc::kQOnesBytes, 128));
  const bool vq8 = views8 != nullptr;  // a chain with sub_vector_size-8 layers (one GPU)
  auto smem_for = [&](int stages) {
    return static_cast<size_t>(xs) + static_cast<size_t>(opc::kQConsumers) * stages * (opc::kQChunkBytes + 16) +
           sizeof(opc::ChainShared) + (vq8 ? opc::kChainVq8SliceBytes : 0);
  };
  int stages = opc::kQMaxStages;
  while (stages >= 2 && smem_for(stages) > static_cast<size_t>(dc.max_smem_optin)) --stages;
  if (stages < 2) return fail(OPC_ERR_UNSUPPORTED, "%s: staged x too large for shared memory", fn);
  const size_t smem = smem_for(stages);
  const int xc = bk_max <= 4 * 8 * opc::kQConsumerThreads ? 4 : 8;
  const bool multi = world > 1;
  if (vq8 && multi) return fail(OPC_ERR_UNSUPPORTED, "%s: sub_vector_size 8 runs on the one-GPU chain", fn);
  auto kern = xc == 4 ? (multi ? opc::chain_kernel<4, true> : vq8 ? opc::chain_kernel<4, false, true> : opc::chain_kernel<4, false>)
                      : (multi ? opc::chain_kernel<8, true> : vq8 ? opc::chain_kernel<8, false, true> : opc::chain_kernel<8, false>);
  OPC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
           "cudaFuncSetAttribute(max dynamic smem, chain)");
  int per_sm = 0;
  OPC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, opc::kQThreads, smem),
           "cudaOccupancyMaxActiveBlocksPerMultiprocessor(chain)");
  if (per_sm < 1) return fail(OPC_ERR_UNSUPPORTED, "%s: chain kernel does not fit on an SM", fn);
  const int G = dc.sm_count;

  // device memory: [layers | onc | parts | epoch] (copied) then [acc (| flags | words)] (zeroed)
  std::vector<opc::ChainLayer> hl(n);
  std::vector<std::vector<int32_t>> onc(n);
  const size_t layers_bytes = align_up(sizeof(opc::ChainLayer) * n, 256);
  size_t off = layers_bytes;
  std::vector<size_t> onc_off(n), acc_off(n), yw_off(n);
  std::vector<int32_t> parts(opc::kChainShareInts * static_cast<size_t>(G) * n, 0);  // [n][G] warp-share records
  for (int j = 0; j < n; ++j) {
    const opc_layer_plan& p = steps[j].layer->plan;
    opc::ChainLayer& c = hl[j];
    memset(&c, 0, sizeof(c));
    c.Up = static_cast<int32_t>(p.packed_units);
    c.U = static_cast<int32_t>(p.total_units);
    c.MT = p.row_tiles;
    c.KT = p.k_units;
    c.OT = p.outlier_tiles;
    c.KO = p.outlier_k_units;
    const std::vector<opc::ChainPart> cparts = chain_parts(c, G);
    onc[j] = outlier_contributors(c, cparts);
    for (int32_t v : onc[j])
      if (v > opc::kMaxContributors)
        return fail(OPC_ERR_UNSUPPORTED, "%s: step %d: %d warps share an outlier tile (at most %d)", fn, j, v,
                    opc::kMaxContributors);
    onc_off[j] = off;
    off += align_up(std::max<size_t>(onc[j].size(), 1) * sizeof(int32_t), 256);
    // each CTA's warp shares, so the kernel does no partition arithmetic (and no division):
    // per warp its unit range and first segment, plus the packed warps and first packed tile
    for (int cta = 0; cta < G; ++cta) {
      const opc::ChainPart& pt = cparts[cta];
      int32_t* e = parts.data() + opc::kChainShareInts * (static_cast<size_t>(j) * G + cta);
      int32_t wu0[opc::kQConsumers], wu1[opc::kQConsumers];
      chain_warp_ranges(pt, opc::kQConsumers, wu0, wu1);
      for (int w = 0; w < opc::kQConsumers; ++w) {
        const int32_t u0 = wu0[w], u1 = wu1[w];
        e[opc::kShU0 + w] = u0;
        e[opc::kShU1 + w] = u1;
        e[opc::kShSeg0 + w] = u0 >= u1 ? 0 : (u0 < c.Up ? u0 / c.KT : c.MT + (u0 - c.Up) / c.KO);
      }
      e[opc::kShWp] = pt.wp;
      e[opc::kShTile0] = c.KT > 0 ? pt.pu0 / c.KT : 0;
    }
  }
  const size_t parts_off = off;
  off += align_up(parts.size() * sizeof(int32_t), 256);
  const size_t epoch_off = off;
  off += 256;
  const size_t image_bytes = off;
  for (int j = 0; j < n; ++j) {
    const opc_layer_plan& p = steps[j].layer->plan;
    acc_off[j] = off;
    off += align_up(static_cast<size_t>(n_slots_of(p)) * opc::kQMaxBatch * sizeof(unsigned long long), 256);
  }
  size_t sync_off = 0;
  if (own_scratch) {
    sync_off = off;
    off += chain_sync_bytes(world, G);
    for (int j = 0; j < n; ++j) {
      yw_off[j] = off;
      off += chain_words_bytes(steps[j].ldy, batch);
    }
  }
  void* mem = nullptr;
  OPC_CUDA(cudaMalloc(&mem, off), "cudaMalloc(chain)");
  char* base = static_cast<char*>(mem);
  ChainRank& me = ranks[rank];
  if (own_scratch) {
    me.sync = reinterpret_cast<unsigned int*>(base + sync_off);
    for (int j = 0; j < n; ++j) me.yw[j] = base + yw_off[j];
  }

  std::vector<unsigned char> img(image_bytes, 0);
  for (int j = 0; j < n; ++j) {
    const opc_chain_step& st = steps[j];
    const opc_layer* L = st.layer;
    const opc_layer_plan& p = L->plan;
    opc::ChainLayer& c = hl[j];
    c.units = static_cast<const uint8_t*>(L->units);
    c.ounits = ounits_q(L);
    c.cbq = codebooks_q(L);
    if (const Vq8View* v = view8(j)) {  // a sub_vector_size-8 layer: its own units, these codebooks
      c.cbq = v->cbq;
      c.cbv = v->cbv;
      c.ounits = v->ounits;
      c.vq8 = 1;
      c.cb_stride = p.K / 128;  // 128-column blocks of the staged x (p.k_units counts 1024-column units)
    }
    c.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
    c.orow = L->outlier_rows;
    c.oexp = L->outlier_rows + n_slots_of(p);
    c.x = static_cast<const __half*>(st.x);
    c.xw = j > 0 ? reinterpret_cast<const uint32_t*>(me.yw[j - 1]) : nullptr;
    c.acc = reinterpret_cast<unsigned long long*>(base + acc_off[j]);
    c.onc = reinterpret_cast<const int32_t*>(base + onc_off[j]);
    for (int q = 0; q < world; ++q) {
      c.y_peer[q] = reinterpret_cast<__half*>(ranks[q].y[j]) + row_off[j];
      c.yw_peer[q] = reinterpret_cast<uint32_t*>(ranks[q].yw[j]) + row_off[j];
    }
    c.ldx = st.ldx;
    c.ldy = st.ldy;
    c.ldxw = j > 0 ? chain_ldyw(steps[j - 1].ldy) : 0;
    c.ldyw = chain_ldyw(st.ldy);
    c.M = p.M;
    c.K = p.K;
    c.K_pad = p.K_pad;
    c.x_vec16 = (p.K % 8 == 0) && (st.ldx % 8 == 0) && aligned(st.x, 16);
    c.row_off = row_off[j];
    c.m_full = m_full[j];
    // a later step writing the same fp16 buffer makes this step's fp16 stores dead
    c.write_y = 1;
    for (int k = j + 1; k < n; ++k)
      if (steps[k].y == st.y && steps[k].ldy == st.ldy && m_full[k] >= m_full[j]) c.write_y = 0;
    c.y_alias_x0 = j > 0 && (fp16_ranges_overlap(steps[0].x, steps[0].ldx, steps[0].layer->plan.K, st.y, st.ldy,
                                                 m_full[j], batch) ||
                             (world > 1 && j == n - 1));
    memcpy(img.data() + j * sizeof(opc::ChainLayer), &c, sizeof(c));
    if (!onc[j].empty()) memcpy(img.data() + onc_off[j], onc[j].data(), onc[j].size() * sizeof(int32_t));

  }
  memcpy(img.data() + parts_off, parts.data(), parts.size() * sizeof(int32_t));
  cudaError_t e = cudaMemcpy(base, img.data(), image_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(base + image_bytes, 0, off - image_bytes);
  if (e == cudaSuccess && !own_scratch) e = cudaMemset(me.sync, 0, chain_sync_bytes(world, G));
  if (e == cudaSuccess && !own_scratch)
    for (int j = 0; j < n && e == cudaSuccess; ++j) e = cudaMemset(me.yw[j], 0, chain_words_bytes(steps[j].ldy, batch));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(mem);
    return cuda_fail(e, "chain setup copy");
  }
  opc_chain* ch = new opc_chain();
  ch->device = dev;
  ch->n_layers = n;
  ch->batch = batch;
  ch->stages = stages;
  ch->xs_bytes = xs;
  ch->smem = smem;
  ch->grid = G;
  ch->xc = xc;
  ch->rank = rank;
  ch->world = world;
  ch->dev_mem = mem;
  ch->d_layers = reinterpret_cast<opc::ChainLayer*>(base);
  ch->d_parts = reinterpret_cast<const int4*>(base + parts_off);
  ch->d_sync = me.sync;
  for (int q = 0; q < world; ++q) ch->sync_peer[q] = ranks[q].sync;
  ch->d_epoch = reinterpret_cast<unsigned int*>(base + epoch_off);
  ch->vq8 = vq8;
  *out = ch;
  return OPC_OK;
}

// Largest |centroid| and largest |outlier value| of a layer (split fp16 codebooks and the
// row-major outlier copy; outlier and padding rows are zero in the codebooks).  One float as bits:
// non-negative floats order like their bit patterns, so an integer atomicMax finds the maximum.
__global__ void layer_absmax_kernel(int32_t m_pad, const uint2* __restrict__ cb, int64_t n_dense,
                                    const uint16_t* __restrict__ dense, unsigned int* __restrict__ out) {
  float m = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < m_pad; i += stride) {
    const uint2 c = cb[i];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t h = ((c.x >> (8 * e)) & 0xffu) | (((c.y >> (8 * e)) & 0xffu) << 8);
      m = fmaxf(m, fabsf(__half2float(__ushort_as_half(static_cast<unsigned short>(h)))));
    }
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_dense; i += stride)
    m = fmaxf(m, fabsf(__half2float(__ushort_as_half(dense[i]))));
  const uint32_t b = __reduce_max_sync(0xffffffffu, m == m ? __float_as_uint(m) : 0x7f800000u);
  if ((threadIdx.x & 31) == 0) atomicMax(out, b);
}

// Upper bound of every dequantized row's 2-norm, as the integer kernel sees the row (centroids
// rounded to 15 bits of the row's largest): sqrt(K) * max|w| * (1 + 2^-12), rounded up to float.
int layer_row_norm_bound(const opc_layer* L, unsigned int* d_tmp, float* out) {
  const opc_layer_plan& p = L->plan;
  OPC_CUDA(cudaMemset(d_tmp, 0, sizeof(unsigned int)), "cudaMemset(absmax)");
  const int64_t n_dense = static_cast<int64_t>(n_slots_of(p)) * p.K_pad;
  layer_absmax_kernel<<<148, 256>>>(p.M_pad, static_cast<const uint2*>(L->codebooks), n_dense,
                                    reinterpret_cast<const uint16_t*>(dense_outliers(L)), d_tmp);
  OPC_CUDA(cudaGetLastError(), "launch layer_absmax_kernel");
  unsigned int bits = 0;
  OPC_CUDA(cudaMemcpy(&bits, d_tmp, sizeof(bits), cudaMemcpyDeviceToHost), "cudaMemcpy(absmax)");
  float amax = 0.f;
  memcpy(&amax, &bits, sizeof(amax));
  if (!(amax <= 65504.f)) return fail(OPC_ERR_INVALID, "chain: a layer holds non-finite weights");
  const double b = std::sqrt(static_cast<double>(p.K)) * static_cast<double>(amax) * (1.0 + 1.0 / 4096.0);
  float f = static_cast<float>(b);
  if (static_cast<double>(f) < b) f = std::nextafter(f, INFINITY);
  *out = f;
  return OPC_OK;
}

// The dataflow form (opc::chain2_kernel): batch 1, one GPU.  Besides the weights' descriptors and
// warp shares (computed as for the barrier form), every layer j >= 1 gets its input's digit
// buffer (KT_j blocks of 512 bytes, initialised to the digits of 0 so that padding columns read
// as 0), its block row counters, and its block sums in the [2][s_total] array.
int chain2_build(const char* fn, const opc_chain_step* steps, int32_t n, opc_chain** out) {
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  std::vector<int32_t> m_full(n);
  for (int j = 0; j < n; ++j) m_full[j] = steps[j].layer->plan.M;
  rc = check_chain_steps(fn, steps, n, 1, dc, m_full);
  if (rc != OPC_OK) return rc;
  int32_t nb[2] = {1, 1};
  for (int j = 0; j < n; ++j) nb[j & 1] = std::max(nb[j & 1], steps[j].layer->plan.k_units);
  if (nb[0] > opc::kC2MaxBlocks || nb[1] > opc::kC2MaxBlocks)
    return fail(OPC_ERR_UNSUPPORTED, "%s: K above %d columns", fn, opc::kC2MaxBlocks * opc::kPackedCols);
  const int nbmax = std::max(nb[0], nb[1]);
  auto smem_for = [&](int stages) {
    return static_cast<size_t>(nb[0] + nb[1]) * opc::kC2BlockBytes + 256 +
           static_cast<size_t>(opc::kC2Consumers) * stages * (opc::kQChunkBytes + 16) + 2 * nbmax * 8 + 48 + 16 +
           sizeof(opc::Chain2Shared);
  };
  int stages = opc::kQMaxStages;
  while (stages >= 2 && smem_for(stages) > static_cast<size_t>(dc.max_smem_optin)) --stages;
  if (stages < 2) return fail(OPC_ERR_UNSUPPORTED, "%s: staged x too large for shared memory", fn);
  const size_t smem = smem_for(stages);
  OPC_CUDA(cudaFuncSetAttribute(opc::chain2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
           "cudaFuncSetAttribute(max dynamic smem, chain2)");
  int per_sm = 0;
  OPC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, opc::chain2_kernel, opc::kC2Threads, smem),
           "cudaOccupancyMaxActiveBlocksPerMultiprocessor(chain2)");
  if (per_sm < 1) return fail(OPC_ERR_UNSUPPORTED, "%s: dataflow chain kernel does not fit on an SM", fn);
  const int G = dc.sm_count;

  // copied image: [layers | onc | parts | epoch]; zeroed: [acc | ocnt per layer | sync | s_all |
  // counters per layer]; digit buffers per layer (set to the digits of 0)
  std::vector<opc::Chain2Layer> hl(n);
  std::vector<std::vector<int32_t>> onc(n);
  size_t off = align_up(sizeof(opc::Chain2Layer) * n, 256);
  std::vector<size_t> onc_off(n), acc_off(n), ocnt_off(n), cnt_off(n, 0), xd_off(n, 0), s_off(n, 0);
  std::vector<int32_t> parts(opc::kChainShareInts * static_cast<size_t>(G) * n, 0);
  for (int j = 0; j < n; ++j) {
    const opc_layer_plan& p = steps[j].layer->plan;
    opc::ChainLayer c;
    memset(&c, 0, sizeof(c));
    c.Up = static_cast<int32_t>(p.packed_units);
    c.U = static_cast<int32_t>(p.total_units);
    c.MT = p.row_tiles;
    c.KT = p.k_units;
    c.OT = p.outlier_tiles;
    c.KO = p.outlier_k_units;
    const std::vector<opc::ChainPart> cparts = chain_parts(c, G, opc::kC2Consumers);
    onc[j] = outlier_contributors(c, cparts, opc::kC2Consumers);
    onc_off[j] = off;
    off += align_up(std::max<size_t>(onc[j].size(), 1) * sizeof(int32_t), 256);
    for (int cta = 0; cta < G; ++cta) {
      const opc::ChainPart& pt = cparts[cta];
      int32_t* e = parts.data() + opc::kChainShareInts * (static_cast<size_t>(j) * G + cta);
      for (int w = 0; w < opc::kC2Consumers; ++w) {
        int32_t u0 = 0, u1 = 0;
        opc::chain_warp_range(pt, w, &u0, &u1, opc::kC2Consumers);
        e[opc::kShU0 + w] = u0;
        e[opc::kShU1 + w] = u1;
        e[opc::kShSeg0 + w] = u0 >= u1 ? 0 : (u0 < c.Up ? u0 / c.KT : c.MT + (u0 - c.Up) / c.KO);
      }
      e[opc::kShWp] = pt.wp;
      e[opc::kShTile0] = c.KT > 0 ? pt.pu0 / c.KT : 0;
    }
  }
  const size_t parts_off = off;
  off += align_up(parts.size() * sizeof(int32_t), 256);
  const size_t epoch_off = off;
  off += 256;
  const size_t image_bytes = off;
  for (int j = 0; j < n; ++j) {
    const opc_layer_plan& p = steps[j].layer->plan;
    acc_off[j] = off;
    off += align_up(static_cast<size_t>(n_slots_of(p)) * sizeof(unsigned long long), 256);
    ocnt_off[j] = off;
    off += align_up(static_cast<size_t>(std::max(p.outlier_tiles, 1)) * sizeof(int32_t), 256);
  }
  const size_t sync_off = off;
  off += chain_sync_bytes(1, G);
  int32_t s_total = 0;
  for (int j = 1; j < n; ++j) {
    s_off[j] = static_cast<size_t>(s_total);
    s_total += steps[j].layer->plan.k_units;
  }
  const size_t s_all_off = off;
  off += align_up(static_cast<size_t>(2) * std::max(s_total, 1) * sizeof(unsigned long long), 256);
  for (int j = 1; j < n; ++j) {
    cnt_off[j] = off;
    off += align_up(static_cast<size_t>(steps[j].layer->plan.k_units) * sizeof(uint32_t), 256);
  }
  const size_t zero_end = off;
  for (int j = 1; j < n; ++j) {
    xd_off[j] = off;
    off += align_up(static_cast<size_t>(steps[j].layer->plan.k_units) * opc::kC2BlockBytes, 256);
  }
  void* mem = nullptr;
  OPC_CUDA(cudaMalloc(&mem, off), "cudaMalloc(chain2)");
  char* base = static_cast<char*>(mem);
  auto undo = [&](int code) {
    cudaFree(mem);
    return code;
  };
  std::vector<float> wb(n, 0.f);
  unsigned int* d_tmp = reinterpret_cast<unsigned int*>(base + epoch_off + 128);  // scratch word, reset below
  for (int j = 0; j < n; ++j) {
    rc = layer_row_norm_bound(steps[j].layer, d_tmp, &wb[j]);
    if (rc != OPC_OK) return undo(rc);
  }
  std::vector<unsigned char> img(image_bytes, 0);
  for (int j = 0; j < n; ++j) {
    const opc_chain_step& st = steps[j];
    const opc_layer* L = st.layer;
    const opc_layer_plan& p = L->plan;
    opc::Chain2Layer& c = hl[j];
    memset(&c, 0, sizeof(c));
    c.units = static_cast<const uint8_t*>(L->units);
    c.ounits = ounits_q(L);
    c.cbq = codebooks_q(L);
    c.tile_mask = static_cast<const uint16_t*>(L->tile_mask);
    c.orow = L->outlier_rows;
    c.oexp = L->outlier_rows + n_slots_of(p);
    c.acc = reinterpret_cast<unsigned long long*>(base + acc_off[j]);
    c.ocnt = reinterpret_cast<int32_t*>(base + ocnt_off[j]);
    c.onc = reinterpret_cast<const int32_t*>(base + onc_off[j]);
    c.x = static_cast<const __half*>(st.x);
    if (j > 0) {
      c.xd = reinterpret_cast<const uint8_t*>(base + xd_off[j]);
      c.xcnt = reinterpret_cast<const uint32_t*>(base + cnt_off[j]);
      c.xS = reinterpret_cast<const unsigned long long*>(base + s_all_off) + s_off[j];
    }
    c.y = static_cast<__half*>(st.y);
    if (j + 1 < n) {
      c.yd = reinterpret_cast<uint8_t*>(base + xd_off[j + 1]);
      c.ycnt = reinterpret_cast<uint32_t*>(base + cnt_off[j + 1]);
      c.yS = reinterpret_cast<unsigned long long*>(base + s_all_off) + s_off[j + 1];
      c.y_rows = steps[j + 1].layer->plan.K;
      c.KT_next = steps[j + 1].layer->plan.k_units;
    }
    c.ldx = st.ldx;
    c.ldy = st.ldy;
    c.Up = static_cast<int32_t>(p.packed_units);
    c.U = static_cast<int32_t>(p.total_units);
    c.M = p.M;
    c.K = p.K;
    c.K_pad = p.K_pad;
    c.MT = p.row_tiles;
    c.KT = p.k_units;
    c.OT = p.outlier_tiles;
    c.KO = p.outlier_k_units;
    c.x_vec16 = (p.K % 8 == 0) && (st.ldx % 8 == 0) && aligned(st.x, 16);
    c.write_y = 1;
    for (int k = j + 1; k < n; ++k)
      if (steps[k].y == st.y && steps[k].ldy == st.ldy && m_full[k] >= m_full[j]) c.write_y = 0;
    c.y_alias_x0 = j > 0 && fp16_ranges_overlap(steps[0].x, steps[0].ldx, steps[0].layer->plan.K, st.y, st.ldy, m_full[j], 1);
    c.wbound = wb[j];
    memcpy(img.data() + j * sizeof(opc::Chain2Layer), &c, sizeof(c));
    if (!onc[j].empty()) memcpy(img.data() + onc_off[j], onc[j].data(), onc[j].size() * sizeof(int32_t));
  }
  memcpy(img.data() + parts_off, parts.data(), parts.size() * sizeof(int32_t));
  cudaError_t e = cudaMemcpy(base, img.data(), image_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(base + image_bytes, 0, zero_end - image_bytes);
  // digit buffers: the digits of 0 (m + 2^30 = 0x40000000: 0x40 in plane 0, 0 elsewhere)
  if (e == cudaSuccess && off > zero_end) e = cudaMemset(base + zero_end, 0, off - zero_end);
  for (int j = 1; j < n && e == cudaSuccess; ++j)
    e = cudaMemset2D(base + xd_off[j], opc::kC2BlockBytes, 0x40, 128, steps[j].layer->plan.k_units);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return undo(cuda_fail(e, "chain2 setup copy"));
  opc_chain* ch = new opc_chain();
  ch->device = dev;
  ch->n_layers = n;
  ch->batch = 1;
  ch->stages = stages;
  ch->smem = smem;
  ch->grid = G;
  ch->rank = 0;
  ch->world = 1;
  ch->dev_mem = mem;
  ch->form = OPC_CHAIN_FORM_DATAFLOW;
  ch->nb0 = nb[0];
  ch->nb1 = nb[1];
  ch->s_total = s_total;
  ch->d_layers2 = reinterpret_cast<const opc::Chain2Layer*>(base);
  ch->d_parts = reinterpret_cast<const int4*>(base + parts_off);
  ch->d_sync = reinterpret_cast<unsigned int*>(base + sync_off);
  ch->d_epoch = reinterpret_cast<unsigned int*>(base + epoch_off);
  ch->d_s_all = reinterpret_cast<unsigned long long*>(base + s_all_off);
  *out = ch;
  return OPC_OK;
}

// Exchanged description of one rank's shards (opc_chain_tp_info).
constexpr uint32_t kTpInfoMagic = 0x4f504354u;  // "OPCT"
constexpr uint32_t kTpInfoVersion = 2;
struct TpInfoHeader {
  uint32_t magic, version;
  int32_t n_steps, grid, batch, world;
  uint64_t region_bytes, scratch_offset;
};
struct TpInfoStep {
  int32_t M, K;
  int64_t ldy;
  uint64_t y_offset, yw_offset;
};

}  // namespace

extern "C" {

int opc_chain_create(const opc_chain_step* steps, int32_t n_steps, int32_t batch, opc_chain** out) {
  return opc_chain_create_ex(steps, n_steps, batch, OPC_CHAIN_FORM_AUTO, out);
}

int opc_chain_create_ex(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t form, opc_chain** out) {
  if (!out) return fail(OPC_ERR_INVALID, "opc_chain_create: out is NULL");
  if (form != OPC_CHAIN_FORM_AUTO && form != OPC_CHAIN_FORM_BARRIER && form != OPC_CHAIN_FORM_DATAFLOW)
    return fail(OPC_ERR_INVALID, "opc_chain_create: unknown form %d", form);
  if (form == OPC_CHAIN_FORM_DATAFLOW && batch != 1)
    return fail(OPC_ERR_UNSUPPORTED, "opc_chain_create: the dataflow form runs batch 1 (got %d)", batch);
  // AUTO picks the barrier form: on the Llama-3.1-8B decode step it measured 843 tok/s against
  // 574 for the dataflow form, whose per-layer hand-off (release, acquire, bulk copy) is slower
  // than the barrier form's polling of tagged words.
  if (form == OPC_CHAIN_FORM_DATAFLOW && steps && n_steps >= 1) {
    *out = nullptr;
    bool plans_ok = true;
    for (int j = 0; j < n_steps; ++j) plans_ok = plans_ok && steps[j].layer && plan_ok(&steps[j].layer->plan);
    if (!plans_ok) return fail(OPC_ERR_INVALID, "opc_chain_create: invalid layer");
    const int rc = chain2_build("opc_chain_create", steps, n_steps, out);
    if (rc == OPC_OK || form == OPC_CHAIN_FORM_DATAFLOW || rc != OPC_ERR_UNSUPPORTED) return rc;
    // AUTO: outside the dataflow form's limits, the barrier form may still run it
  }
  *out = nullptr;
  if (!steps || n_steps < 1) return fail(OPC_ERR_INVALID, "opc_chain_create: no steps");
  if (batch < 1 || batch > opc::kQMaxBatch)
    return fail(OPC_ERR_UNSUPPORTED, "opc_chain_create: batch %d (the chain runs batch 1..%d)", batch, opc::kQMaxBatch);
  std::vector<ChainRank> ranks(1);
  ChainRank& me = ranks[0];
  me.M.resize(n_steps);
  me.y.resize(n_steps);
  me.yw.resize(n_steps, nullptr);
  for (int j = 0; j < n_steps; ++j) {
    if (!steps[j].layer || !plan_ok(&steps[j].layer->plan))
      return fail(OPC_ERR_INVALID, "opc_chain_create: step %d: invalid layer", j);
    me.M[j] = steps[j].layer->plan.M;
    me.y[j] = static_cast<char*>(steps[j].y);
  }
  // sub_vector_size-8 steps: their codebook and outlier forms for the chain (built here, owned by it)
  std::vector<opc_chain_step> st(steps, steps + n_steps);
  std::vector<Vq8View> views(n_steps);
  std::vector<const Vq8View*> views8(n_steps, nullptr);
  bool any8 = false;
  for (int j = 0; j < n_steps; ++j) {
    if (steps[j].layer->plan.sub_vector_size != 8) continue;
    any8 = true;
    const int rc = make_vq8_view("opc_chain_create", j, steps[j].layer, &views[j]);
    if (rc != OPC_OK) {
      for (auto& v : views) v.release();
      return rc;
    }
    st[j].layer = &views[j].L;
    views8[j] = &views[j];
  }
  const int rc = chain_build("opc_chain_create", st.data(), n_steps, batch, 0, 1, ranks, true, out,
                             any8 ? &views8 : nullptr);
  if (rc != OPC_OK) {
    for (auto& v : views) v.release();
    return rc;
  }
  for (auto& v : views) (*out)->owned.insert((*out)->owned.end(), v.owned.begin(), v.owned.end());
  return OPC_OK;
}

int opc_chain_tp_scratch_bytes(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t world,
                               size_t* bytes) {
  if (!bytes) return fail(OPC_ERR_INVALID, "opc_chain_tp_scratch_bytes: bytes is NULL");
  *bytes = 0;
  if (!steps || n_steps < 1) return fail(OPC_ERR_INVALID, "opc_chain_tp_scratch_bytes: no steps");
  if (batch < 1 || batch > opc::kQMaxBatch)
    return fail(OPC_ERR_UNSUPPORTED, "opc_chain_tp_scratch_bytes: batch %d", batch);
  if (world < 1 || world > opc::kMaxRanks)
    return fail(OPC_ERR_UNSUPPORTED, "opc_chain_tp_scratch_bytes: world %d (1..%d)", world, opc::kMaxRanks);
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  const int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  size_t b = chain_sync_bytes(world, dc.sm_count);
  for (int j = 0; j < n_steps; ++j) {
    if (steps[j].ldy < 1) return fail(OPC_ERR_INVALID, "opc_chain_tp_scratch_bytes: step %d: ldy not set", j);
    b += chain_words_bytes(steps[j].ldy, batch);
  }
  *bytes = b;
  return OPC_OK;
}

int opc_chain_tp_info(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t world, const void* region,
                      size_t region_bytes, size_t scratch_offset, void* info, size_t* info_bytes) {
  if (!info_bytes) return fail(OPC_ERR_INVALID, "opc_chain_tp_info: info_bytes is NULL");
  if (!steps || n_steps < 1 || !region) return fail(OPC_ERR_INVALID, "opc_chain_tp_info: no steps or region");
  const size_t need = sizeof(TpInfoHeader) + sizeof(TpInfoStep) * n_steps;
  if (!info) {
    *info_bytes = need;
    return OPC_OK;
  }
  if (*info_bytes < need) return fail(OPC_ERR_INVALID, "opc_chain_tp_info: %zu bytes given, %zu needed", *info_bytes, need);
  size_t scratch = 0;
  int rc = opc_chain_tp_scratch_bytes(steps, n_steps, batch, world, &scratch);
  if (rc != OPC_OK) return rc;
  if (scratch_offset % 256 || scratch_offset + scratch > region_bytes || reinterpret_cast<uintptr_t>(region) % 256)
    return fail(OPC_ERR_INVALID, "opc_chain_tp_info: scratch [%zu, +%zu) not 256-aligned inside the %zu-byte region",
                scratch_offset, scratch, region_bytes);
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  unsigned char* o = static_cast<unsigned char*>(info);
  TpInfoHeader h;
  memset(&h, 0, sizeof(h));
  h.magic = kTpInfoMagic;
  h.version = kTpInfoVersion;
  h.n_steps = n_steps;
  h.grid = dc.sm_count;
  h.batch = batch;
  h.world = world;
  h.region_bytes = region_bytes;
  h.scratch_offset = scratch_offset;
  memcpy(o, &h, sizeof(h));
  size_t yw = scratch_offset + chain_sync_bytes(world, dc.sm_count);
  const char* rb = static_cast<const char*>(region);
  for (int j = 0; j < n_steps; ++j) {
    if (!steps[j].layer || !plan_ok(&steps[j].layer->plan))
      return fail(OPC_ERR_INVALID, "opc_chain_tp_info: step %d: invalid layer", j);
    const char* y = static_cast<const char*>(steps[j].y);
    if (!y || y < rb || y >= rb + region_bytes)
      return fail(OPC_ERR_INVALID, "opc_chain_tp_info: step %d: y is not inside the region", j);
    TpInfoStep s;
    memset(&s, 0, sizeof(s));
    s.M = steps[j].layer->plan.M;
    s.K = steps[j].layer->plan.K;
    s.ldy = steps[j].ldy;
    s.y_offset = static_cast<uint64_t>(y - rb);
    s.yw_offset = yw;
    yw += chain_words_bytes(steps[j].ldy, batch);
    memcpy(o + sizeof(TpInfoHeader) + j * sizeof(TpInfoStep), &s, sizeof(s));
  }
  *info_bytes = need;
  return OPC_OK;
}

int opc_chain_create_tp(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t rank, int32_t world,
                        void* const* regions, const void* const* infos, opc_chain** out) {
  const char* fn = "opc_chain_create_tp";
  if (!out) return fail(OPC_ERR_INVALID, "%s: out is NULL", fn);
  *out = nullptr;
  if (!steps || n_steps < 1 || !regions || !infos) return fail(OPC_ERR_INVALID, "%s: missing arguments", fn);
  if (batch < 1 || batch > opc::kQMaxBatch) return fail(OPC_ERR_UNSUPPORTED, "%s: batch %d", fn, batch);
  if (world < 1 || world > opc::kMaxRanks || rank < 0 || rank >= world)
    return fail(OPC_ERR_UNSUPPORTED, "%s: rank %d of world %d (1..%d ranks)", fn, rank, world, opc::kMaxRanks);
  for (int j = 0; j < n_steps; ++j)
    if (!steps[j].layer || !plan_ok(&steps[j].layer->plan)) return fail(OPC_ERR_INVALID, "%s: step %d: invalid layer", fn, j);
  std::vector<ChainRank> ranks(world);
  std::vector<std::vector<TpInfoStep>> st(world, std::vector<TpInfoStep>(n_steps));
  std::vector<TpInfoHeader> hd(world);
  for (int p = 0; p < world; ++p) {
    const unsigned char* b = static_cast<const unsigned char*>(infos[p]);
    if (!b || !regions[p]) return fail(OPC_ERR_INVALID, "%s: rank %d: no info or region", fn, p);
    TpInfoHeader& h = hd[p];
    memcpy(&h, b, sizeof(h));
    if (h.magic != kTpInfoMagic || h.version != kTpInfoVersion)
      return fail(OPC_ERR_INVALID, "%s: rank %d: not a chain info of this library version", fn, p);
    if (h.n_steps != n_steps || h.batch != batch || h.world != world)
      return fail(OPC_ERR_INVALID, "%s: rank %d: %d steps, batch %d, world %d (here %d, %d, %d)", fn, p, h.n_steps,
                  h.batch, h.world, n_steps, batch, world);
    if (h.grid != hd[0].grid) return fail(OPC_ERR_UNSUPPORTED, "%s: ranks run %d and %d CTAs", fn, hd[0].grid, h.grid);
    for (int j = 0; j < n_steps; ++j) memcpy(&st[p][j], b + sizeof(TpInfoHeader) + j * sizeof(TpInfoStep), sizeof(TpInfoStep));
  }
  for (int p = 0; p < world; ++p) {
    ChainRank& r = ranks[p];
    r.M.resize(n_steps);
    r.y.resize(n_steps);
    r.yw.resize(n_steps);
    char* region = static_cast<char*>(regions[p]);
    const TpInfoHeader& h = hd[p];
    if (h.scratch_offset + chain_sync_bytes(world, h.grid) > h.region_bytes)
      return fail(OPC_ERR_INVALID, "%s: rank %d: flags outside its region", fn, p);
    r.sync = reinterpret_cast<unsigned int*>(region + h.scratch_offset);
    for (int j = 0; j < n_steps; ++j) {
      const TpInfoStep& s = st[p][j];
      int64_t rows = 0;
      for (int q = 0; q < world; ++q) rows += st[q][j].M;
      if (s.K != steps[j].layer->plan.K || s.M < 1 || s.ldy != st[0][j].ldy || s.ldy < rows)
        return fail(OPC_ERR_INVALID, "%s: rank %d step %d: K %d, rows %d, ld %lld (here K %d; full rows %lld)", fn, p, j,
                    s.K, s.M, static_cast<long long>(s.ldy), steps[j].layer->plan.K, static_cast<long long>(rows));
      const uint64_t y_end = s.y_offset + 2 * static_cast<uint64_t>((batch - 1) * s.ldy + rows);
      const uint64_t w_end = s.yw_offset + chain_words_bytes(s.ldy, batch);
      if (s.y_offset % 2 || s.yw_offset % 256 || y_end > h.region_bytes || w_end > h.region_bytes)
        return fail(OPC_ERR_INVALID, "%s: rank %d step %d: outputs exceed its region", fn, p, j);
      r.M[j] = s.M;
      r.y[j] = region + s.y_offset;
      r.yw[j] = region + s.yw_offset;
    }
  }
  ChainRank& me = ranks[rank];
  for (int j = 0; j < n_steps; ++j)
    if (steps[j].layer->plan.M != me.M[j] || static_cast<char*>(steps[j].y) != me.y[j] || steps[j].ldy != st[rank][j].ldy)
      return fail(OPC_ERR_INVALID, "%s: step %d: does not match this rank's info", fn, j);
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  DeviceCache dc;
  const int rc = device_cache(dev, &dc);
  if (rc != OPC_OK) return rc;
  if (dc.sm_count != hd[0].grid)
    return fail(OPC_ERR_UNSUPPORTED, "%s: this GPU has %d SMs, the ranks %d", fn, dc.sm_count, hd[0].grid);
  return chain_build(fn, steps, n_steps, batch, rank, world, ranks, false, out);
}

int opc_chain_launch(opc_chain* ch, void* stream_v) {
  if (!ch) return fail(OPC_ERR_INVALID, "opc_chain_launch: chain is NULL");
  int dev = 0;
  OPC_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != ch->device) return fail(OPC_ERR_INVALID, "opc_chain_launch: chain lives on device %d, current is %d", ch->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  if (ch->form == OPC_CHAIN_FORM_DATAFLOW) {
    opc::Chain2Args a2;
    memset(&a2, 0, sizeof(a2));
    a2.layers = ch->d_layers2;
    a2.parts = ch->d_parts;
    a2.sync = ch->d_sync;
    a2.epoch = ch->d_epoch;
    a2.s_all = ch->d_s_all;
    a2.trace = ch->trace;
    a2.n_layers = ch->n_layers;
    a2.stages = ch->stages;
    a2.s_total = ch->s_total;
    a2.nb0 = ch->nb0;
    a2.nb1 = ch->nb1;
    a2.negz = opc::kNegZero2;
    cudaLaunchConfig_t cfg2 = {};
    cfg2.gridDim = dim3(static_cast<unsigned>(ch->grid));
    cfg2.blockDim = dim3(opc::kC2Threads);
    cfg2.dynamicSmemBytes = ch->smem;
    cfg2.stream = s;
    cudaLaunchAttribute attr2[1];
    attr2[0].id = cudaLaunchAttributeCooperative;
    attr2[0].val.cooperative = 1;
    cfg2.attrs = attr2;
    cfg2.numAttrs = 1;
    OPC_CUDA(cudaLaunchKernelEx(&cfg2, opc::chain2_kernel, a2), "launch chain2_kernel");
    return OPC_OK;
  }
  opc::ChainArgs a;
  memset(&a, 0, sizeof(a));
  a.layers = ch->d_layers;
  a.parts = ch->d_parts;
  a.sync = ch->d_sync;
  for (int p = 0; p < ch->world; ++p) a.sync_peer[p] = ch->sync_peer[p];
  a.epoch = ch->d_epoch;
  a.trace = ch->trace;
  a.n_layers = ch->n_layers;
  a.batch = ch->batch;
  a.stages = ch->stages;
  a.xs_bytes = ch->xs_bytes;
  a.negz = opc::kNegZero2;
  a.l2_prefetch = ch->l2_prefetch;
  a.rank = ch->rank;
  a.world = ch->world;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ch->grid));
  cfg.blockDim = dim3(opc::kQThreads);
  cfg.dynamicSmemBytes = ch->smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool multi = a.world > 1;
  if (ch->xc == 4) {
    if (multi) OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<4, true>, a), "launch chain_kernel");
    else if (ch->vq8) OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<4, false, true>, a), "launch chain_kernel");
    else OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<4, false>, a), "launch chain_kernel");
  } else {
    if (multi) OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<8, true>, a), "launch chain_kernel");
    else if (ch->vq8) OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<8, false, true>, a), "launch chain_kernel");
    else OPC_CUDA(cudaLaunchKernelEx(&cfg, opc::chain_kernel<8, false>, a), "launch chain_kernel");
  }
  return OPC_OK;
}

size_t opc_chain_trace_bytes(const opc_chain* ch) {
  if (!ch) return 0;
  return static_cast<size_t>(ch->n_layers) * ch->grid * opc::kChainTracePhases * sizeof(unsigned long long);
}

int32_t opc_chain_grid(const opc_chain* ch) { return ch ? ch->grid : 0; }

int32_t opc_chain_form(const opc_chain* ch) { return ch ? ch->form : 0; }


int opc_chain_set_trace(opc_chain* ch, void* trace) {
  if (!ch) return fail(OPC_ERR_INVALID, "opc_chain_set_trace: chain is NULL");
  if (trace && !aligned(trace, 8)) return fail(OPC_ERR_INVALID, "opc_chain_set_trace: buffer not 8-byte aligned");
  ch->trace = static_cast<unsigned long long*>(trace);
  return OPC_OK;
}

int opc_chain_set_option(opc_chain* ch, int32_t option, int32_t value) {
  if (!ch) return fail(OPC_ERR_INVALID, "opc_chain_set_option: chain is NULL");
  switch (option) {
    case OPC_CHAIN_L2_PREFETCH: ch->l2_prefetch = value ? 1 : 0; return OPC_OK;
    default: return fail(OPC_ERR_INVALID, "opc_chain_set_option: unknown option %d", option);
  }
}

int opc_chain_destroy(opc_chain* ch) {
  if (!ch) return OPC_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ch->device);
  cudaError_t e = cudaFree(ch->dev_mem);
  for (void* p : ch->owned) {
    const cudaError_t e2 = cudaFree(p);
    if (e == cudaSuccess) e = e2;
  }
  cudaSetDevice(prev);
  delete ch;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(chain)");
  return OPC_OK;
}

// ---------------------------------------------------------------------------------------------
// Peer-visible memory through CUDA IPC (one process per GPU).
// ---------------------------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == OPC_PEER_HANDLE_BYTES, "IPC handle size");

int opc_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(OPC_ERR_INVALID, "opc_peer_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  OPC_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(peer region)");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "opc_peer_alloc");
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return OPC_OK;
}

int opc_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(OPC_ERR_INVALID, "opc_peer_open: bad arguments");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  OPC_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return OPC_OK;
}

int opc_peer_close(void* ptr) {
  if (!ptr) return OPC_OK;
  OPC_CUDA(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return OPC_OK;
}

int opc_peer_free(void* ptr) {
  if (!ptr) return OPC_OK;
  OPC_CUDA(cudaFree(ptr), "cudaFree(peer region)");
  return OPC_OK;
}

int opc_set_gemm_crossover(int32_t batch) {
  if (batch < 0 || batch > kMaxBatch)
    return fail(OPC_ERR_INVALID, "opc_set_gemm_crossover: batch %d outside [0, %d]", batch, kMaxBatch);
  g_gemm_crossover.store(batch, std::memory_order_relaxed);
  return OPC_OK;
}

int32_t opc_gemm_crossover(void) { return g_gemm_crossover.load(std::memory_order_relaxed); }

// XXH64 (xxHash, 64-bit variant, as published with its specification): four 64-bit lanes over
// 32-byte stripes, then the tail in 8-, 4- and 1-byte steps, then the avalanche.  Host code.
namespace {
constexpr uint64_t kXxP1 = 0x9E3779B185EBCA87ull, kXxP2 = 0xC2B2AE3D27D4EB4Full, kXxP3 = 0x165667B19E3779F9ull,
                   kXxP4 = 0x85EBCA77C2B2AE63ull, kXxP5 = 0x27D4EB2F165667C5ull;
inline uint64_t xx_rotl(uint64_t v, int r) { return (v << r) | (v >> (64 - r)); }
inline uint64_t xx_read64(const unsigned char* p) {
  uint64_t v;
  memcpy(&v, p, 8);  // little-endian host
  return v;
}
inline uint32_t xx_read32(const unsigned char* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}
inline uint64_t xx_round(uint64_t acc, uint64_t in) { return xx_rotl(acc + in * kXxP2, 31) * kXxP1; }
inline uint64_t xx_merge(uint64_t acc, uint64_t v) { return (acc ^ xx_round(0, v)) * kXxP1 + kXxP4; }
}  // namespace

uint64_t opc_xxh64(const void* data, size_t len, uint64_t seed) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  const unsigned char* end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + kXxP1 + kXxP2, v2 = seed + kXxP2, v3 = seed, v4 = seed - kXxP1;
    for (; end - p >= 32; p += 32) {
      v1 = xx_round(v1, xx_read64(p));
      v2 = xx_round(v2, xx_read64(p + 8));
      v3 = xx_round(v3, xx_read64(p + 16));
      v4 = xx_round(v4, xx_read64(p + 24));
    }
    h = xx_rotl(v1, 1) + xx_rotl(v2, 7) + xx_rotl(v3, 12) + xx_rotl(v4, 18);
    h = xx_merge(h, v1);
    h = xx_merge(h, v2);
    h = xx_merge(h, v3);
    h = xx_merge(h, v4);
  } else {
    h = seed + kXxP5;
  }
  h += static_cast<uint64_t>(len);
  for (; end - p >= 8; p += 8) h = xx_rotl(h ^ xx_round(0, xx_read64(p)), 27) * kXxP1 + kXxP4;
  if (end - p >= 4) {
    h = xx_rotl(h ^ (static_cast<uint64_t>(xx_read32(p)) * kXxP1), 23) * kXxP2 + kXxP3;
    p += 4;
  }
  for (; p < end; ++p) h = xx_rotl(h ^ (static_cast<uint64_t>(*p) * kXxP5), 11) * kXxP1;
  h ^= h >> 33;
  h *= kXxP2;
  h ^= h >> 29;
  h *= kXxP3;
  h ^= h >> 32;
  return h;
}

int opc_take_device_error(int32_t device, int32_t* code) {
  if (!code) return fail(OPC_ERR_INVALID, "opc_take_device_error: code is NULL");
  int prev = 0;
  OPC_CUDA(cudaGetDevice(&prev), "cudaGetDevice");
  OPC_CUDA(cudaSetDevice(device), "cudaSetDevice");
  int v = 0, zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, opc::g_opc_device_error, sizeof(int));
  if (e == cudaSuccess && v != 0) e = cudaMemcpyToSymbol(opc::g_opc_device_error, &zero, sizeof(int));  // (already 0 otherwise)
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "opc_take_device_error");
  *code = v;
  return OPC_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Element-wise (COO) outliers (opc_coo.cuh)
// ------------------------------------------------------------------------------------------------
extern "C" {

int opc_coo_build(int32_t M, int32_t K, int32_t svs, const void* codebooks_f16, const uint8_t* indices_u8,
                  const int64_t* coo, const void* values_f16, int64_t nnz, int32_t* row_ptr, int32_t* cols,
                  void* values_out_f16, float* delta, int64_t* nnz_out) {
  if (M <= 0 || K <= 0 || (svs != 1 && svs != 8) || K % svs)
    return fail(OPC_ERR_INVALID, "opc_coo_build: M=%d K=%d sub_vector_size=%d", M, K, svs);
  if (nnz < 0 || (nnz > 0 && (!coo || !values_f16)) || !codebooks_f16 || !indices_u8 || !row_ptr || !nnz_out)
    return fail(OPC_ERR_INVALID, "opc_coo_build: NULL argument");
  if (nnz > INT32_MAX) return fail(OPC_ERR_INVALID, "opc_coo_build: %lld entries exceed int32 offsets", static_cast<long long>(nnz));
  const __half* cb = static_cast<const __half*>(codebooks_f16);
  const __half* val = static_cast<const __half*>(values_f16);
  // position -> last entry (a repeated position keeps its last value)
  std::vector<std::pair<int64_t, int64_t>> key(static_cast<size_t>(nnz));
  for (int64_t j = 0; j < nnz; ++j) {
    const int64_t r = coo[2 * j], c = coo[2 * j + 1];
    if (r < 0 || r >= M || c < 0 || c >= K)
      return fail(OPC_ERR_INVALID, "opc_coo_build: entry %lld at (%lld, %lld) outside %d x %d", static_cast<long long>(j),
                  static_cast<long long>(r), static_cast<long long>(c), M, K);
    key[static_cast<size_t>(j)] = {r * K + c, j};
  }
  std::stable_sort(key.begin(), key.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  std::vector<int64_t> keep;
  keep.reserve(key.size());
  for (size_t i = 0; i < key.size(); ++i)
    if (i + 1 == key.size() || key[i + 1].first != key[i].first) keep.push_back(key[i].second);
  const int64_t n = static_cast<int64_t>(keep.size());
  *nnz_out = n;
  if (!cols && !values_out_f16 && !delta) {  // size query: row_ptr only
  } else if (!cols || !values_out_f16 || !delta) {
    return fail(OPC_ERR_INVALID, "opc_coo_build: cols, values and delta must all be given");
  }
  std::fill(row_ptr, row_ptr + M + 1, 0);
  for (int64_t j : keep) ++row_ptr[coo[2 * j] + 1];
  for (int32_t r = 0; r < M; ++r) row_ptr[r + 1] += row_ptr[r];
  if (!cols) return OPC_OK;
  __half* vout = static_cast<__half*>(values_out_f16);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t j = keep[static_cast<size_t>(i)];
    const int64_t r = coo[2 * j], c = coo[2 * j + 1];
    const int idx = indices_u8[r * (K / svs) + c / svs];
    if (idx > 3) return fail(OPC_ERR_INVALID, "opc_coo_build: codebook index %d at (%lld, %lld)", idx, static_cast<long long>(r), static_cast<long long>(c));
    const float q = __half2float(cb[(r * 4 + idx) * svs + c % svs]);
    cols[i] = static_cast<int32_t>(c);
    vout[i] = val[j];
    delta[i] = __half2float(val[j]) - q;
  }
  return OPC_OK;
}

int opc_coo_gemv(int32_t M, const int32_t* row_ptr, const int32_t* cols, const float* delta, const void* x, int64_t ldx,
                 void* y, int64_t ldy, int32_t batch, void* stream) {
  if (M <= 0 || !row_ptr || !cols || !delta || !x || !y || batch < 1 || ldy < M)
    return fail(OPC_ERR_INVALID, "opc_coo_gemv: invalid arguments (M=%d, batch=%d)", M, batch);
  const unsigned grid =
      static_cast<unsigned>(std::min<int64_t>(ceil_div(static_cast<int64_t>(M) * batch, opc::kCooWarps * 32), 148 * 16));
  opc::coo_gemv_kernel<<<grid, opc::kCooWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      M, row_ptr, cols, delta, static_cast<const __half*>(x), ldx, static_cast<__half*>(y), ldy, batch);
  OPC_CUDA(cudaGetLastError(), "opc_coo_gemv launch");
  return OPC_OK;
}

int opc_coo_scatter(int32_t M, const int32_t* row_ptr, const int32_t* cols, const void* values_f16, void* w, int64_t ldw,
                    void* stream) {
  if (M <= 0 || !row_ptr || !cols || !values_f16 || !w) return fail(OPC_ERR_INVALID, "opc_coo_scatter: invalid arguments");
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(M, 8), 148 * 8));
  opc::coo_scatter_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      M, row_ptr, cols, static_cast<const __half*>(values_f16), static_cast<__half*>(w), ldw);
  OPC_CUDA(cudaGetLastError(), "opc_coo_scatter launch");
  return OPC_OK;
}

}  // extern "C"
