/*
 * opc_b200.h -- C ABI of the B200 (sm_100a) fused 2-bit codebook dequant-matmul library.
 *
 * This is the drop-in boundary for opacc1ty's fused dequant path.  Every entry point takes
 * plain pointers and sizes; CUDA streams are passed as `void*` (a cudaStream_t, NULL = legacy
 * default stream).  Unless stated otherwise all data pointers are DEVICE pointers.  Calls are
 * stream-ordered and asynchronous; no entry point on the hot path (opc_gemv) allocates memory or
 * synchronises the host.
 *
 * Error convention: every `int` entry point returns OPC_OK (0) on success and a negative
 * OPC_ERR_* code on failure; opc_last_error() then returns a human-readable message for the
 * calling thread.  This replaces the reference's Python exceptions raised by
 * MetalKernelManager (opacc1ty/utils/metal_utils.py:111,171,183,307) and the C runtime's
 * `-1` + engine->error string (runtime/src/bf2_format.c:151-225).
 *
 * Layer data starts out in the reference's .bf2 layout (opacc1ty/format/bf2.py:121-134):
 *   codebooks      [M][4][svs] fp16
 *   indices        [M][K/svs]  uint8, values 0..3 (one byte per index, not packed)
 *   outlier values [n][K]      fp16, whole output rows
 *   outlier ids    [n]         integer row ids
 * opc_repack_layer converts it once, at load time, into the device layout the kernels stream
 * (see opc_layer_plan below).  sub_vector_size 1 (2 bits/weight, 4 fp16 centroids per output
 * row) runs on every path; sub_vector_size 8 (true VQ: an index selects one of 4 fp16 vectors of
 * 8 per row, the reference quantizer's default) runs opc_gemv / opc_gemv_noalloc (any batch),
 * opc_gemm and opc_dequant, with K a multiple of 8, and the one-GPU decode chain with K a
 * multiple of 1024; other sizes return OPC_ERR_UNSUPPORTED.
 */
#ifndef OPC_B200_H
#define OPC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OPC_ABI_VERSION 1

enum {
  OPC_OK = 0,
  OPC_ERR_INVALID = -1,     /* bad argument: shape, pointer, alignment, out-of-range id */
  OPC_ERR_UNSUPPORTED = -2, /* valid request this build does not implement (e.g. svs 4) */
  OPC_ERR_CUDA = -3,        /* a CUDA runtime call failed; message has the CUDA error */
  OPC_ERR_WORKSPACE = -4,   /* workspace missing or smaller than opc_gemv_workspace_bytes() */
  OPC_ERR_DEVICE = -5       /* a kernel reported an error through the device error word */
};

/* Geometry of one repacked layer.  Filled by opc_plan_layer(); the caller allocates the four
 * device buffers with the byte sizes given here.
 *
 * sub_vector_size 8: k_units = K_pad/256 (K_pad = K rounded up to 256); units = packed_units
 * 128-byte index units (row tile t x 256-column block b = unit t*k_units + b; 16 bytes per row
 * pair g, byte s of word w holding the 2-bit vector indices of rows g and g+8 for the two
 * 8-column groups of k16 step 4w+s), then the outlier rows row-major [outlier_tiles*16][K_pad]
 * fp16; codebooks [row_tiles][32 lanes][8] 32-bit words (lane 4g+q: halves 2q, 2q+1 of vectors
 * 0..3 of row g, then of row g+8; outlier rows zero); tile_mask and outlier_rows as below.
 *
 * sub_vector_size 1 device layout ("units" are 512-byte blocks streamed by the GEMV):
 *   units[0 .. packed_units)      packed 2-bit indices: row tile t (16 rows) x k block b (128
 *                                 columns) is unit t*k_units + b.  Inside a unit, lane l of a
 *                                 warp owns bytes [16l, 16l+16): four 32-bit words whose 2-bit
 *                                 fields are laid out so that a masked word is directly a PRMT
 *                                 selector of four int8 weights, and one IMAD turns a field pair
 *                                 into a selector of two fp16 weights (mma.sync A fragments).
 *   then (total_units - packed_units) outlier units for the integer kernel (batch 1..2): 16 rows x
 *                                 16 columns, each value as two int8 parts of a per-row integer
 *                                 form, in mma.sync A-fragment order;
 *   then as many outlier units for the fp16 kernel (16x16 fp16 blocks in A-fragment order);
 *   then the outlier rows row-major, [outlier_tiles*16][K_pad] fp16 (prefill GEMM).
 *   units_bytes = (packed_units + 2 * outlier units) * 512 + max(outlier_tiles,1)*16*K_pad*2.
 *   codebooks   [M_pad] x 8 bytes: for each row the low bytes of its 4 fp16 centroids, then
 *               the high bytes; then [M_pad] x 16 bytes: the centroids as integers
 *               c * 2^e (|.| <= 2^14) in two int8 parts (4 high, 4 low) and the int32 e.
 *               Outlier rows and padding rows are zero.
 *   tile_mask   [row_tiles] uint16: bit i set when row 16t+i is an outlier row.
 *   outlier_rows[outlier_tiles*16] int32: output row of each outlier slot, -1 for padding; then
 *               as many int32 exponents of the slots' integer rows.
 */
typedef struct opc_layer_plan {
  int32_t M, K, n_outliers, sub_vector_size;
  int32_t M_pad, K_pad;                 /* M rounded up to 16, K rounded up to 128 */
  int32_t row_tiles, k_units;           /* M_pad/16, K_pad/128 */
  int32_t outlier_tiles, outlier_k_units; /* ceil(n_outliers/16), K_pad/16 */
  int64_t packed_units, total_units;
  int64_t units_bytes, codebook_bytes, tile_mask_bytes, outlier_rows_bytes;
} opc_layer_plan;

/* A repacked layer: the plan plus the caller-owned device buffers it describes. */
typedef struct opc_layer {
  opc_layer_plan plan;
  void* units;
  void* codebooks;
  void* tile_mask;
  int32_t* outlier_rows;
} opc_layer;

typedef struct opc_device_props {
  char name[256];
  int32_t device, sm_count, cc_major, cc_minor;
  int64_t total_mem_bytes;
  int32_t max_smem_per_block_optin, max_threads_per_block, l2_bytes, warp_size;
} opc_device_props;

/* Library version string ("opc_b200 <semver> abi <n>"); replaces bf_version()
 * (runtime/include/opacc1ty.h:205). */
const char* opc_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* opc_last_error(void);

/* Properties of CUDA device `device`; mirrors get_metal_device_info() / GPUInfo
 * (opacc1ty/utils/metal_utils.py:24-76).  Returns OPC_ERR_CUDA when no device is present. */
int opc_device_info(int32_t device, opc_device_props* out);

/* Compute the device geometry for an M x K layer with n_outliers outlier rows.
 * Replaces the size arithmetic of BF2Reader._build_index (opacc1ty/format/bf2.py:204-213). */
int opc_plan_layer(int32_t M, int32_t K, int32_t n_outliers, int32_t sub_vector_size,
                   opc_layer_plan* plan);

/* Repack one .bf2 layer into `layer`'s device buffers (load time, not the hot path).
 *   codebooks_f16   device [M][4][svs] fp16
 *   indices_u8      device [M][K/svs] uint8; an index > 3 is rejected (OPC_ERR_INVALID), as
 *                   the reference's codebook lookup would raise
 *   outlier_f16     device [n_rows][K] fp16 (may be NULL when n_rows == 0)
 *   outlier_ids     HOST   [n_rows] int64 row ids.  Ids outside [0, M) are rejected.  A
 *                   repeated id keeps its LAST row, matching the sequential replacement of
 *                   dequantize_layer (opacc1ty/export/converter.py:59-63).
 * Outlier rows get an all-zero codebook, so "add the outlier dot product in the epilogue"
 * (kernels/dequant_gemv.metal:118-131) and "replace the row" (converter.py:63) coincide.
 * `layer->plan.n_outliers` must equal opc_count_distinct_ids(outlier_ids, n_rows).
 * Synchronises `stream`. */
int opc_repack_layer(const opc_layer* layer, const void* codebooks_f16, const uint8_t* indices_u8,
                     const void* outlier_f16, const int64_t* outlier_ids, int32_t n_rows,
                     void* stream);

/* Number of distinct ids in a host id list (the n_outliers to plan with). */
int32_t opc_count_distinct_ids(const int64_t* ids, int32_t n);

/* Workspace bytes opc_gemv needs for `layer` on `device` (a scratch area for partial sums,
 * then one counter per 16-row tile).  The workspace must be zero-filled once before first use
 * (opc_workspace_init); every opc_gemv leaves its counters at zero again.  One workspace may
 * serve any number of layers and batch sizes whose calls are ordered on one stream (size it for
 * the layer with the most rows); calls that can overlap on the GPU need separate workspaces. */
size_t opc_gemv_workspace_bytes(const opc_layer_plan* plan, int32_t batch, int32_t device);

/* Zero `bytes` of workspace on `stream`. */
int opc_workspace_init(void* workspace, size_t bytes, void* stream);

/* Fused dequant-GEMV / small-batch GEMM:  y[b][r] = sum_k x[b][k] * W_hat[r][k]
 * for b < batch (1..64), r < M, with W_hat = codebook lookup + outlier-row replacement.
 *   x  device fp16, row b at x + b*ldx (ldx >= K, in elements)
 *   y  device fp16, row b at y + b*ldy (ldy >= M)
 * Batches above opc_gemm_crossover() (default 8, up to 64) with x 16-byte aligned and
 * ldx % 8 == 0 run the prefill GEMM (opc_gemm), splitting K in the workspace where that helps.
 * Batch 1..2 (when the staged x fits in shared memory): x is staged per CTA as integers
 * round(x * 2^e_x), below 2^22 in magnitude (e_x from max |x|), the centroids are the 15-bit
 * integer codebooks above; the dot
 * products accumulate exactly in integers (mma.sync int8, int64 combination) and are scaled and
 * rounded once to fp16.  Larger batches: fp16 x fp16 products accumulated in fp32
 * (mma.sync m16n8k16), rounded once to fp16.
 * Replaces MetalKernelManager.dequant_gemv (opacc1ty/utils/metal_utils.py:202-288) and
 * metal_forward_layer (runtime/src/metal_backend.m:224-331).  Launched with programmatic
 * dependent launch: the weight stream of this call starts while the previous opc_gemv on the
 * stream is still finishing.  Results are deterministic (fixed summation order). */
int opc_gemv(const opc_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy,
             int32_t batch, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free opc_gemv, for callers that cannot allocate device memory: plugin hosts
 * that hand a plugin only its preallocated input and output buffers, or serving processes
 * whose whole device memory belongs to their own pool.  No counterpart in the reference.
 * Same computation and arguments as opc_gemv, but the scratch comes from a 448 KiB array
 * compiled into this library (every GPU that loads the library keeps it until exit) rather than
 * a workspace, and the call allocates and frees nothing.  sub_vector_size 1 layers always run
 * the fp16 GEMV kernel here: results equal opc_gemv's bit for bit at batch 3..8 (where opc_gemv
 * runs the same kernel) and agree within the GEMV tolerance at batch 1..2 (where opc_gemv runs
 * the integer kernel).  sub_vector_size 8 layers run the same kernel as opc_gemv and use no
 * scratch.  Limits: batch 1..8 and, for sub_vector_size 1, at most 16384 tiles (row tiles of
 * 16 rows plus outlier tiles), i.e. M <= 262144; larger requests return OPC_ERR_INVALID with the
 * reason.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  Every call shares the one array, so calls that may overlap on the GPU (different
 * streams, or different host threads on one device) race and must be serialised by the
 * caller; each call clears the counters it needs before its kernel runs. */
int opc_gemv_noalloc(const opc_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy,
                     int32_t batch, void* stream);

/* Prefill GEMM on the 5th-generation tensor cores:  y[t][r] = sum_k x[t][k] * W_hat[r][k]
 * for t < n_tok tokens.  Replaces the reference's dequant_gemm_2bit pipeline
 * (kernels/dequant_gemm.metal:34-149, loaded by metal_utils.py:188-196).
 *   x  device fp16 [n_tok][ldx], 16-byte aligned, ldx a multiple of 8 (read with TMA)
 *   y  device fp16 [n_tok][ldy] (ldy >= M)
 * One persistent kernel (one CTA per SM): weight tiles of 128 rows are decoded from the packed
 * indices (sub_vector_size 1: through the row's fp16 codebook; 8: one codebook vector per 8
 * columns) into shared memory and multiplied with x tiles of 16..256 tokens (the size chosen
 * from n_tok and the SM count) by tcgen05.mma (fp16 x fp16 -> fp32 in tensor memory, two
 * accumulators so that a tile's epilogue overlaps the next tile's MMAs), rounded once to fp16;
 * outlier rows are computed as extra tiles from the row-major outlier copy.  Deterministic.  No
 * workspace.  Other x layouts return OPC_ERR_UNSUPPORTED (use opc_gemv, batch <= 64). */
int opc_gemm(const opc_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy, int32_t n_tok,
             void* stream);

/* Decode chain: a sequence of dependent GEMVs run by ONE persistent cooperative kernel (one CTA
 * per SM; a producer warp streams every step's weights ahead across step boundaries; no grid
 * barrier between steps: every output element is also published as a tagged 32-bit word that
 * the next step's readers poll).  Replaces per-step dispatch of MetalKernelManager.dequant_gemv for
 * a forward pass (runtime/src/inference.c:117-233 calls one layer at a time).  Each step is the
 * batch 1..2 integer GEMV of opc_gemv; results equal opc_gemv's bit for bit.
 *   steps[0].x      the chain input (device fp16, ldx)
 *   steps[j].x      for j >= 1 must be steps[j-1].y with the same leading dimension (a prefix:
 *                   steps[j].layer K <= steps[j-1].layer M)
 *   steps[j].y      fp16 outputs of two steps are either disjoint or the same buffer (same
 *                   pointer and leading dimension: only the later step's values are stored);
 *                   step 0's output may not overlap the chain input, later ones may
 * Requires batch 1..2, batch * K_pad <= 30720 for every step and fewer than 65535 steps.
 * A sub_vector_size-8 step (K a multiple of 1024; one GPU, barrier form) streams the layer's own
 * index units; the chain builds and owns the integer forms of its codebook vectors (one exponent
 * per row) and of its outlier rows.  Its dot products are exact like svs 1's (not bit-equal to
 * opc_gemv's svs-8 kernel, which accumulates in fp32).
 * opc_chain_create copies the step list to the device and allocates the chain's scratch (freed
 * by opc_chain_destroy); opc_chain_launch launches on `stream` (one kernel, nothing to clear;
 * capturable into a CUDA graph).  One chain must not run on two streams at once.  A launch
 * whose bounded wait gives up (2 s) records device error 3 and poisons the chain: every later
 * launch records error 4 and does nothing; destroy and recreate it. */
typedef struct opc_chain opc_chain;
typedef struct opc_chain_step {
  const opc_layer* layer;
  const void* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
} opc_chain_step;
int opc_chain_create(const opc_chain_step* steps, int32_t n_steps, int32_t batch, opc_chain** out);
/* The same with an explicit form of the decode-step kernel:
 *   OPC_CHAIN_FORM_BARRIER   the step-by-step form above: each step's x is staged per CTA from the
 *                            previous step's fp16 outputs with its exponent from max|x| (as
 *                            opc_gemv does), so results equal opc_gemv's bit for bit; batch 1..2.
 *   OPC_CHAIN_FORM_DATAFLOW  batch 1, one GPU, K <= 32768 (and the barrier form's other limits):
 *                            steps exchange their outputs as fixed-point digits whose scale is
 *                            fixed in advance from a norm bound (|y_r| <= ||W row r||_2 ||x||_2;
 *                            30-bit integers below 2^29 in magnitude, at least as fine as the
 *                            barrier form's 22 bits for every x whose norm is within 2^7 of its
 *                            largest element times sqrt(K)), written by the warp that finishes each
 *                            row and copied into every CTA per 128-column block as soon as that block
 *                            is complete.  No barrier of any kind between steps.  Every step's fp16
 *                            output is rounded once from an exact integer dot product, so results
 *                            are deterministic; they agree with opc_gemv within the GEMV tolerance
 *                            rather than bit for bit (the inputs' fixed-point scale differs).  A
 *                            non-finite step output records device error 5.
 *   OPC_CHAIN_FORM_AUTO      (opc_chain_create) the barrier form (measured faster on the Llama-3.1-8B
 *                            decode step: 843 against 574 tok/s).
 * The dataflow form replaces nothing in the reference beyond what opc_chain_create replaces. */
enum { OPC_CHAIN_FORM_AUTO = 0, OPC_CHAIN_FORM_BARRIER = 1, OPC_CHAIN_FORM_DATAFLOW = 2 };
int opc_chain_create_ex(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t form, opc_chain** out);
/* The form a chain was built with (OPC_CHAIN_FORM_BARRIER or OPC_CHAIN_FORM_DATAFLOW). */
int32_t opc_chain_form(const opc_chain* chain);
int opc_chain_launch(opc_chain* chain, void* stream);
int opc_chain_destroy(opc_chain* chain);
/* Tracing: with a device buffer of opc_chain_trace_bytes() set, every launch records per step
 * and per CTA %globaltimer stamps (ns).  Barrier form, taken by the CTA's first consumer
 * thread: step start, setup done, first poll of its x words done, x complete, max barrier passed,
 * digits stored, x staged, its own units done.  Dataflow form: [0] the staging warp begins the
 * step, [1] it holds every block of x, [2] consumer warp 0 begins the step, [3] warp 0's units
 * done, [4] / [5] the staging warp's first / last block arrival, [6] warp 0 starts waiting for
 * its first chunk's x blocks (0 if it did not wait), [7] it has them.  Barrier form also: [8 + w]
 * consumer warp w finished its units and row writes of the step.  Layout [step][cta][24] uint64
 * (unused slots stay as the caller left them); NULL turns tracing off.  opc_chain_grid() is the
 * number of CTAs (one per SM). */
size_t opc_chain_trace_bytes(const opc_chain* chain);
/* Options: OPC_CHAIN_L2_PREFETCH (default 0): stream the weights with an L2 evict-first policy
 * (measured no faster on the Llama-3.1-8B decode step, kept as an option). */
enum { OPC_CHAIN_L2_PREFETCH = 1 };
int opc_chain_set_option(opc_chain* chain, int32_t option, int32_t value);
int32_t opc_chain_grid(const opc_chain* chain);
int opc_chain_set_trace(opc_chain* chain, void* trace);

/* Row-sharded decode chain over `world` GPUs of one node (one process per GPU), replacing the
 * per-layer GEMV + all-gather of tensor parallelism with ONE kernel per rank: each rank computes
 * its contiguous shard of every step's output rows from the full x and stores each finished row
 * (fp16 and tagged exchange word, system-scope stores) straight into every rank's copies over
 * NVLink; readers poll their local copy, so no barrier separates the steps.  One cross-rank flag
 * barrier ends each launch.  No all-gather, no NCCL call, no TMA multicast.  Results equal the
 * one-GPU chain over the unsharded layers, opc_gemv and the NCCL form bit for bit (the dot
 * products are exact integers; every rank stages the same x).
 *
 * Peer-visible memory ("region"): opc_peer_alloc allocates device memory on the current GPU and
 * exports an OPC_PEER_HANDLE_BYTES handle; other ranks map it with opc_peer_open.  Each rank's
 * region holds its copy of every step's full fp16 output and the chain's scratch (flags and
 * exchange words: opc_chain_tp_scratch_bytes, at a 256-aligned offset; call it with every
 * step's layer and ldy set).
 *
 * Steps, per rank: layer = this rank's row shard of the step's matrix (ranks in row order: rank
 * p's shard starts after the rows of ranks < p); y = row 0 of this rank's copy of the full output
 * (inside its region, ldy >= the full row count and the same on every rank); x as for
 * opc_chain_create (step 0 any device buffer holding the same values on every rank; step j a
 * prefix of step j-1's full output).  Step 0's input may overlap the LAST step's output only.
 * Setup: every rank calls opc_chain_tp_info (info = NULL first for the size), the infos are
 * exchanged (any transport; the ranks' infos in rank order), every rank calls
 * opc_chain_create_tp with all regions mapped in its process (regions[rank] = its own), and ALL
 * ranks must have returned from opc_chain_create_tp before ANY rank launches (a host barrier).
 * Then every rank calls opc_chain_launch once per decode step, in the same order.  A rank's
 * outputs are complete when its launch has finished.  All ranks need the same SM count. */
#define OPC_PEER_HANDLE_BYTES 64
#define OPC_MAX_RANKS 8
int opc_peer_alloc(size_t bytes, void** ptr, void* handle);
int opc_peer_open(const void* handle, void** ptr);
int opc_peer_close(void* ptr);
int opc_peer_free(void* ptr);
int opc_chain_tp_scratch_bytes(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t world,
                               size_t* bytes);
int opc_chain_tp_info(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t world, const void* region,
                      size_t region_bytes, size_t scratch_offset, void* info, size_t* info_bytes);
int opc_chain_create_tp(const opc_chain_step* steps, int32_t n_steps, int32_t batch, int32_t rank, int32_t world,
                        void* const* regions, const void* const* infos, opc_chain** out);

/* Write the dequantized matrix W_hat [M][K] fp16 (row r at w + r*ldw) from the repacked
 * layer.  Bit-exact restatement of dequantize_layer (opacc1ty/export/converter.py:26-67),
 * decoded with the same device routine the GEMV uses. */
int opc_dequant(const opc_layer* layer, void* w, int64_t ldw, void* stream);

/* GEMV -> GEMM crossover: opc_gemv runs batches above `batch` (default 8) on the prefill GEMM
 * when x is TMA-readable, and smaller batches on the GEMV kernels.  The GEMM then uses opc_gemv's
 * workspace (opc_gemv_workspace_bytes counts it for batches above 8) to split K for layers with
 * fewer 128-row tiles than SMs.  0 sends every TMA-readable call to the GEMM, 64 none.  Process-wide; takes effect for later calls.  The reference has a
 * single GEMV dispatch (opacc1ty/utils/metal_utils.py:202-288) and no such switch; the setting
 * exists so the crossover can be measured (both kernels timed at every batch) and tuned. */
int opc_set_gemm_crossover(int32_t batch);
int32_t opc_gemm_crossover(void);

/* Element-wise (COO) outliers: single weights kept exactly in fp16 beside the codebook form (the
 * "sparse_outlier" layer type the reference's format reserves, format/header.py:57-60, and its
 * quantizer never produces).  W_hat = codebook lookup, then W_hat[r][c] = v per entry (a repeated
 * position keeps its last value).  The codebook part is an ordinary layer without outlier rows
 * (opc_plan_layer with n_outliers 0, opc_repack_layer); the entries become a row-compressed list:
 *
 * opc_coo_build (HOST pointers, load time): codebooks [M][4][svs] fp16 and indices [M][K/svs]
 * uint8 (the layer's .bf2 arrays), coo [nnz][2] int64 (row, col), values [nnz] fp16 ->
 * row_ptr [M+1] int32, then for the *nnz_out unique positions in (row, col) order cols int32,
 * values fp16 and delta = value - codebook value at the position, fp32.  With cols, values_out
 * and delta all NULL it only fills row_ptr and *nnz_out (a size query). */
int opc_coo_build(int32_t M, int32_t K, int32_t sub_vector_size, const void* codebooks_f16, const uint8_t* indices_u8,
                  const int64_t* coo, const void* values_f16, int64_t nnz, int32_t* row_ptr, int32_t* cols,
                  void* values_out_f16, float* delta, int64_t* nnz_out);
/* Epilogue after opc_gemv / opc_gemm of the codebook part (same stream; device pointers):
 * y[b][r] = fp16(y[b][r] + sum_j delta_j * x[b][col_j]) for b < batch, the sum in fp32 in a fixed
 * order.  x must hold every column the entries name.  One extra fp16 rounding (<= 2^-11 of |y|). */
int opc_coo_gemv(int32_t M, const int32_t* row_ptr, const int32_t* cols, const float* delta, const void* x, int64_t ldx,
                 void* y, int64_t ldy, int32_t batch, void* stream);
/* After opc_dequant: w[r][col_j] = value_j (device pointers); the result is bit-exact. */
int opc_coo_scatter(int32_t M, const int32_t* row_ptr, const int32_t* cols, const void* values_f16, void* w, int64_t ldw,
                    void* stream);

/* XXH64 (seed `seed`) of a HOST buffer: the checksum that the .bf2 layout places after the last
 * layer (opacc1ty/format/header.py:26; the reference documents it but never writes it).  Files
 * written with it set bit 0 of the file header's flags.  A format helper, not a kernel. */
uint64_t opc_xxh64(const void* data, size_t len, uint64_t seed);

/* Read and clear the device error word of `device` (synchronises the device).  Kernels with
 * bounded waits record a nonzero code there instead of hanging; 0 = no error. */
int opc_take_device_error(int32_t device, int32_t* code);

#ifdef __cplusplus
}
#endif

#endif /* OPC_B200_H */
