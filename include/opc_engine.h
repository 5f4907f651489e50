/*
 * opc_engine.h -- C engine API over the B200 fused dequant library: load a .bf2 model and run a
 * Llama-style decoder on it (prefill, decode steps with a KV cache, sampling).
 *
 * Same functions, types and argument meaning as the reference's C runtime header
 * (runtime/include/opacc1ty.h:33-212), so a program written against it links against this
 * library instead.  The reference implements the calls as stubs (runtime/src/inference.c:183-245
 * returns fixed pseudo-random logits; bf2_format.c:131-314 reads no model numbers); here they
 * run the model:
 *
 *   bf_engine_create    parses the .bf2 file (file header, model JSON, every layer; int32 or
 *                       int64 outlier ids; the XXH64 trailer when the flags announce it), copies
 *                       each quantized layer to the GPU and repacks it (opc_repack_layer),
 *                       dequantizes the token embedding into an fp16 table (opc_dequant), keeps
 *                       fp16 pass-through tensors (the RMSNorm weights) on the device and
 *                       allocates the KV cache.
 *   forward / prefill / forward_step
 *                       per block: RMSNorm, q/k/v projections (opc_gemv: the integer GEMV for
 *                       one token, the fp16 GEMV or the tcgen05 GEMM up to 64 tokens; opc_gemm
 *                       for longer prompt chunks), rotary embedding, K/V appended to the cache,
 *                       causal grouped-query attention, o projection + residual, RMSNorm,
 *                       gate/up projections, SiLU(gate) * up, down projection + residual; then
 *                       the final RMSNorm and the lm_head GEMV (the embedding when the file has
 *                       no lm_head).  Prompts run in chunks of up to 512 tokens.  Residual stream
 *                       fp32, GEMV inputs and outputs fp16.
 *   generate            byte-level stub tokenizer as in the reference (each prompt byte is a
 *                       token id, tokens < 256 print as that byte), prefill, then decode steps
 *                       with greedy / temperature / top-k / top-p sampling.
 *
 * Tensor names follow Hugging Face Llama checkpoints (model.embed_tokens.weight,
 * model.layers.N.self_attn.{q,k,v,o}_proj.weight, model.layers.N.mlp.{gate,up,down}_proj.weight,
 * model.layers.N.{input,post_attention}_layernorm.weight, model.norm.weight, lm_head.weight).
 * A missing RMSNorm weight counts as all ones.  Model numbers come from the file's model JSON
 * (hidden_size, num_hidden_layers, num_attention_heads, num_kv_heads or num_key_value_heads,
 * intermediate_size, vocab_size, rope_theta, rms_norm_eps, max_position_embeddings); those it
 * lacks are taken from the layer shapes (hidden and vocab from the embedding, kv heads from
 * k_proj, intermediate from gate_proj) or default (rope_theta 10000, eps 1e-5, head_dim 128
 * when num_attention_heads is absent).
 *
 * Errors: as in the reference (bf2_format.c:151-225), bf_engine_create returns a handle even when
 * loading fails; bf_engine_get_error() is then non-NULL and every compute call returns -1.
 * NULL is returned only for a NULL path or a failed host allocation.  Compute calls return 0 /
 * -1 (and record the message); they run on the engine's own CUDA stream and return when the
 * logits are on the host.  An engine is used by one thread at a time.
 */
#ifndef OPC_ENGINE_H
#define OPC_ENGINE_H

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct BFEngine BFEngine;
typedef struct BFModelConfig BFModelConfig;

/* Model configuration (runtime/include/opacc1ty.h:40-51). */
struct BFModelConfig {
  char architecture[64];
  uint32_t vocab_size;
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_hidden_layers;
  uint32_t num_attention_heads;
  uint32_t num_kv_heads;
  uint32_t max_position_embeddings;
  float rope_theta;
  uint32_t head_dim;
};

/* Sampling parameters (opacc1ty.h:53-62): temperature <= 0 is greedy; top_p 0 and top_k 0
 * disable those filters; repetition_penalty 1 disables it (applied to the tokens generated so
 * far: positive logits divided, negative multiplied); seed 0 draws a seed from the clock. */
typedef struct {
  float temperature;
  float top_p;
  int32_t top_k;
  float repetition_penalty;
  uint32_t seed;
} BFSamplingParams;

/* temperature 1, top_p 0, top_k 0, repetition_penalty 1, seed 0 (opacc1ty.h:64-67). */
extern const BFSamplingParams BF_DEFAULT_SAMPLING;

typedef struct {
  uint64_t total_tokens_generated;
  double total_time_seconds;
  double tokens_per_second;
  size_t peak_memory_bytes;   /* device bytes the engine holds (weights, tables, KV cache, scratch) */
  uint32_t n_kernel_dispatches;
} BFStats;

/* Load `path` on CUDA device 0 with a KV cache of min(max_position_embeddings, 4096) positions
 * (4096 when the JSON has none).  opacc1ty.h:69-78. */
BFEngine* bf_engine_create(const char* path);
/* Same, on `device` with `max_context` cache positions (0: the default above). */
BFEngine* bf_engine_create_ex(const char* path, int32_t device, uint32_t max_context);
void bf_engine_destroy(BFEngine* engine);
const BFModelConfig* bf_engine_get_config(const BFEngine* engine);
/* Message of the engine's last error, NULL if none (opacc1ty.h:90-93). */
const char* bf_engine_get_error(const BFEngine* engine);
uint32_t bf_engine_vocab_size(const BFEngine* engine);

/* Tokenize `prompt` (one token per byte), prefill, generate up to max_new_tokens (stopping after
 * token 0) and write each token's text to `output` (NULL: no output).  Starts from an empty
 * cache.  Returns the number of tokens generated, -1 on error.  opacc1ty.h:95-116. */
int32_t bf_engine_generate(BFEngine* engine, const char* prompt, uint32_t max_new_tokens,
                           const BFSamplingParams* params, FILE* output);
/* Token-level generate: prompt token ids in, generated ids out (out_tokens holds
 * max_new_tokens).  Same loop and stopping rule as bf_engine_generate. */
int32_t bf_engine_generate_tokens(BFEngine* engine, const int32_t* prompt, uint32_t prompt_len,
                                  uint32_t max_new_tokens, const BFSamplingParams* params, int32_t* out_tokens);

/* Reset the cache, run all seq_len tokens and write the last position's logits
 * (vocab_size floats; vocab_size must equal the model's).  opacc1ty.h:118-136. */
int bf_engine_forward(BFEngine* engine, const int32_t* tokens, uint32_t seq_len, float* logits_out,
                      uint32_t vocab_size);
/* Append seq_len tokens to the cache without computing logits.  opacc1ty.h:138-152. */
int bf_engine_prefill(BFEngine* engine, const int32_t* tokens, uint32_t seq_len);
/* Append one token and write the next token's logits.  opacc1ty.h:154-171. */
int bf_engine_forward_step(BFEngine* engine, int32_t token, float* logits_out, uint32_t vocab_size);
void bf_engine_reset_kv_cache(BFEngine* engine);
/* Bytes of the KV cache (allocated at create).  opacc1ty.h:178-181. */
size_t bf_engine_kv_cache_size(const BFEngine* engine);
/* Tokens currently in the cache. */
uint32_t bf_engine_position(const BFEngine* engine);

void bf_engine_get_stats(const BFEngine* engine, BFStats* stats);
void bf_engine_reset_stats(BFEngine* engine);

/* Runtime version string.  opacc1ty.h:200-203. */
const char* bf_version(void);
/* 0: this build has no Metal backend (opacc1ty.h:205-210). */
int bf_has_metal_gpu(void);
/* 1 when a CUDA device of compute capability 10.0 (B200) is present. */
int bf_has_cuda_gpu(void);

#ifdef __cplusplus
}
#endif

#endif /* OPC_ENGINE_H */
