/*
 * opc_oracle.c -- CPU oracle for the fused 2-bit codebook dequant-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the reference algorithm the CUDA
 * library must reproduce.  It is linked only by tests/, by __graft_entry__.smoke() and by the
 * CPU-baseline legs of bench.py, always as the checker or the timed CPU baseline, never as part
 * of the product path.
 *
 * Reference semantics followed (paths relative to the opacc1ty project):
 *   oracle_dequant     opacc1ty/export/converter.py:26-67  (dequantize_layer)
 *                        W[r][g*svs + s] = cb[r][idx[r][g]][s]   (converter.py:48-53)
 *                        columns trimmed to in_features          (converter.py:56)
 *                        W[oi[i]] = ov[i] for i in order         (converter.py:59-63)
 *   oracle_gemv_f64    y = x . W^T recomputed in double (exact products of fp16 values)
 *   oracle_gemv_cpu    the reference's CPU path for one layer -- dequantize the row, then an
 *                        fp32 dot product (converter.py:26-67 + torch.matmul in fp32) -- fused
 *                        per row and spread over pthreads: the CPU baseline.
 * Parity is pinned by tests/golden/ fixtures generated from the reference's own Python code.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* IEEE-754 binary16 <-> binary32, written from the format definition. */
static inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: value = man * 2^-24 */
      float v = (float)man * 5.9604644775390625e-08f;
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Round-to-nearest-even float -> binary16. */
static inline uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                    /* below 2^-14: subnormal / zero */
    float a;
    memcpy(&a, &ax, 4);
    const float scaled = a * 16777216.0f; /* a / 2^-24 */
    uint32_t m = (uint32_t)scaled;
    const float frac = scaled - (float)m;
    if (frac > 0.5f || (frac == 0.5f && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  const uint32_t exp = ((ax >> 23) - 112u) << 10;
  const uint32_t man = (ax >> 13) & 0x3ffu;
  const uint32_t rest = ax & 0x1fffu;
  uint32_t h = exp | man;
  if (rest > 0x1000u || (rest == 0x1000u && (man & 1u))) h++;
  return (uint16_t)(sign | h);
}

float oracle_half_to_float(uint16_t h) { return h2f(h); }
uint16_t oracle_float_to_half(float f) { return f2h(f); }

/*
 * dequantize_layer restated.  cb: [M][4][svs] fp16 bits; idx: [M][n_groups] uint8;
 * ov: [n_out][K] fp16 bits; oi: [n_out] row ids (Python indexing: -M <= id < M);
 * W: [M][Kc] fp16 bits with Kc = min(n_groups*svs, K).
 * Returns 0, -1 for an index value > 3, -2 for an outlier id outside [-M, M), -3 when
 * outliers are present and Kc != K (the reference's row assignment would fail to broadcast).
 */
int oracle_dequant(int32_t M, int32_t K, int32_t svs, int32_t n_groups, const uint16_t* cb, const uint8_t* idx,
                   int32_t n_out, const uint16_t* ov, const int64_t* oi, uint16_t* W) {
  const int64_t full = (int64_t)n_groups * svs;
  const int32_t Kc = (int32_t)(full < K ? full : K);
  for (int32_t r = 0; r < M; ++r) {
    for (int32_t g = 0; g < n_groups; ++g) {
      const uint8_t c = idx[(int64_t)r * n_groups + g];
      if (c > 3) return -1;
      for (int32_t s = 0; s < svs; ++s) {
        const int64_t col = (int64_t)g * svs + s;
        if (col < Kc) W[(int64_t)r * Kc + col] = cb[((int64_t)r * 4 + c) * svs + s];
      }
    }
  }
  if (n_out > 0 && Kc != K) return -3;
  for (int32_t i = 0; i < n_out; ++i) {
    int64_t row = oi[i];
    if (row < -(int64_t)M || row >= M) return -2;
    if (row < 0) row += M;
    memcpy(W + row * Kc, ov + (int64_t)i * K, (size_t)Kc * 2);
  }
  return 0;
}

/* y64[b][r] = sum_k x[b][k] * W[r][k] in double.  W: [M][ldw] fp16, x: [batch][ldx] fp16. */
void oracle_gemv_f64(int32_t M, int32_t K, const uint16_t* W, int64_t ldw, int32_t batch, const uint16_t* x,
                     int64_t ldx, double* y, int64_t ldy) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)K);
  for (int32_t b = 0; b < batch; ++b) {
    for (int32_t k = 0; k < K; ++k) xd[k] = (double)h2f(x[(int64_t)b * ldx + k]);
    for (int32_t r = 0; r < M; ++r) {
      const uint16_t* w = W + (int64_t)r * ldw;
      double s = 0.0;
      for (int32_t k = 0; k < K; ++k) s += xd[k] * (double)h2f(w[k]);
      y[(int64_t)b * ldy + r] = s;
    }
  }
  free(xd);
}

/* ---------------------------------------------------------------------------------------
 * CPU baseline: the reference path (dequantize, then fp32 matmul) for svs == 1, fused per row
 * so it runs in cache, rows split across threads.  Outlier rows use their fp16 values
 * (row replacement).  slot[r] = index into ov of row r's outlier values, or -1.
 * ------------------------------------------------------------------------------------- */
typedef struct {
  int32_t M, K, batch, r0, r1;
  const uint16_t* cb;
  const uint8_t* idx;
  const uint16_t* ov;
  const int32_t* slot;
  const float* xf; /* [batch][K] */
  uint16_t* y;     /* [batch][M] fp16 */
} cpu_job;

static void* cpu_worker(void* arg) {
  cpu_job* j = (cpu_job*)arg;
  float* wrow = (float*)malloc(sizeof(float) * (size_t)j->K);
  for (int32_t r = j->r0; r < j->r1; ++r) {
    const int32_t s = j->slot ? j->slot[r] : -1;
    if (s >= 0) {
      const uint16_t* o = j->ov + (int64_t)s * j->K;
      for (int32_t k = 0; k < j->K; ++k) wrow[k] = h2f(o[k]);
    } else {
      float c[4];
      for (int e = 0; e < 4; ++e) c[e] = h2f(j->cb[(int64_t)r * 4 + e]);
      const uint8_t* ix = j->idx + (int64_t)r * j->K;
      for (int32_t k = 0; k < j->K; ++k) wrow[k] = c[ix[k] & 3];
    }
    for (int32_t b = 0; b < j->batch; ++b) {
      const float* xb = j->xf + (int64_t)b * j->K;
      float acc = 0.f;
      for (int32_t k = 0; k < j->K; ++k) acc += wrow[k] * xb[k];
      j->y[(int64_t)b * j->M + r] = f2h(acc);
    }
  }
  free(wrow);
  return NULL;
}

/* Returns 0 on success.  threads <= 0 means 1. */
int oracle_gemv_cpu(int32_t M, int32_t K, const uint16_t* cb, const uint8_t* idx, const uint16_t* ov,
                    const int32_t* slot, int32_t batch, const uint16_t* x, uint16_t* y, int32_t threads) {
  if (threads <= 0) threads = 1;
  if (threads > 256) threads = 256;
  float* xf = (float*)malloc(sizeof(float) * (size_t)batch * K);
  if (!xf) return -1;
  for (int64_t i = 0; i < (int64_t)batch * K; ++i) xf[i] = h2f(x[i]);
  pthread_t tid[256];
  cpu_job jobs[256];
  const int32_t per = (M + threads - 1) / threads;
  int32_t started = 0;
  for (int32_t t = 0; t < threads; ++t) {
    const int32_t r0 = t * per;
    const int32_t r1 = (r0 + per < M) ? r0 + per : M;
    if (r0 >= r1) break;
    jobs[t] = (cpu_job){M, K, batch, r0, r1, cb, idx, ov, slot, xf, y};
    pthread_create(&tid[t], NULL, cpu_worker, &jobs[t]);
    ++started;
  }
  for (int32_t t = 0; t < started; ++t) pthread_join(tid[t], NULL);
  free(xf);
  return 0;
}
