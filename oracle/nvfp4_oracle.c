/*
 * CPU oracle for the routed-expert NVFP4 MoE path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the CUDA path is compared
 * against; nothing in the product links or calls it. Only tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline leg of bench.py load it.
 *
 * It restates, in plain C, the arithmetic of the reference implementation's
 * expert path (SRSWTI/shooting-brake):
 *
 *   - element decode  e2m1: src/phase7/cpu_expert_capi.cpp:52-60,
 *                          src/QuixiCore-XPU/kernels/moe/nvfp4_moe/variants/
 *                          xpu_sycl/nvfp4_dequant.hpp:35-40
 *   - block scale     e4m3: src/phase7/cpu_expert_capi.cpp:70-92
 *   - row dequant     W[n][k] = e2m1(nib) * fp32(e4m3(sf[n][k/16]) * g),
 *                     low nibble = even k: cpu_expert_capi.cpp:301-346
 *   - GEMV, 4 fp32 accumulators combined (a0+a1)+(a2+a3):
 *                     cpu_expert_capi.cpp:364-420
 *   - SwiGLU  h = silu(g) * u, silu(x) = x / (1 + exp(-x)):
 *                     cpu_expert_capi.cpp:94, 521-543
 *   - routing: ids < 0 or >= E dropped; per expert the routes stay in
 *     (token, k) ascending order; out = sum_k w[t,k] * y[t,k]:
 *                     cpu_expert_capi.cpp:553-628; the skip rule for
 *                     invalid ids also nvfp4_moe.sycl.cpp:139-141
 *   - multiply_router_weight flag: nvfp4_moe.sycl.cpp:178
 *
 * w13 is [E, 2I, K/2] with gate rows [0, I) and up rows [I, 2I) sharing one
 * per-expert global scale (src/phase1/extract_experts.py:254-264), w2 is
 * [E, K, I/2]; scales are linear e4m3 bytes [E, rows, cols/16].
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, so every fp32 operation
 * rounds exactly once in the order written).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float f32_from_bits(uint32_t b) {
  float f;
  memcpy(&f, &b, sizeof f);
  return f;
}

static float bf16_to_f32(uint16_t v) { return f32_from_bits((uint32_t)v << 16); }

/* e2m1 magnitude ladder {0, .5, 1, 1.5, 2, 3, 4, 6}; bit 3 is the sign. */
float sbo_e2m1(uint32_t nib) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float m = mag[nib & 7u];
  return (nib & 8u) ? -m : m;
}

/* float8_e4m3fn: bias 7, subnormals 2^-6 * man/8, exponent 15 with mantissa 7
 * is NaN (no infinities). */
float sbo_e4m3(uint32_t v) {
  const uint32_t sign = v & 0x80u;
  const uint32_t exp = (v >> 3) & 0x0Fu;
  const uint32_t man = v & 0x07u;
  float f;
  if (exp == 0u) {
    f = ldexpf((float)man, -9);
  } else if (exp == 15u && man == 7u) {
    f = NAN;
  } else {
    f = ldexpf(1.0f + (float)man / 8.0f, (int)exp - 7);
  }
  return sign ? -f : f;
}

/* W = e2m1 * fp32(e4m3 * g), rows x cols, row-major. */
void sbo_nvfp4_dequant(const uint8_t* q, const uint8_t* sf, float g, float* out,
                       size_t rows, size_t cols) {
  const size_t kb = cols / 16;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t b = 0; b < kb; ++b) {
      const float bs = sbo_e4m3(sf[r * kb + b]) * g;
      for (size_t j = 0; j < 8; ++j) {
        const uint8_t byte = q[r * (cols / 2) + b * 8 + j];
        out[r * cols + b * 16 + 2 * j] = sbo_e2m1(byte & 0x0Fu) * bs;
        out[r * cols + b * 16 + 2 * j + 1] = sbo_e2m1(byte >> 4) * bs;
      }
    }
  }
}

/* Stable counting sort of routes by expert.
 *   counts[E], offsets[E+1] (exclusive scan, offsets[E] = valid routes),
 *   sorted[valid] = route index r = token*top_k + k, in (expert, r) order,
 *   slot_of[M*top_k] = position of route r in sorted, or -1 when dropped.
 * Returns the number of ids outside [-1, E) (they are dropped, like -1). */
int64_t sbo_route_plan(const int32_t* ids, size_t M, size_t top_k, size_t E,
                       int32_t* counts, int32_t* offsets, int32_t* sorted,
                       int32_t* slot_of) {
  const size_t R = M * top_k;
  int64_t bad = 0;
  for (size_t e = 0; e < E; ++e) counts[e] = 0;
  for (size_t r = 0; r < R; ++r) {
    const int32_t e = ids[r];
    if (e < 0 || (size_t)e >= E) {
      if (e < -1 || (e >= 0 && (size_t)e >= E)) ++bad;
      continue;
    }
    ++counts[e];
  }
  offsets[0] = 0;
  for (size_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t* cursor = (int32_t*)malloc(E * sizeof(int32_t));
  for (size_t e = 0; e < E; ++e) cursor[e] = offsets[e];
  for (size_t r = 0; r < R; ++r) {
    const int32_t e = ids[r];
    if (e < 0 || (size_t)e >= E) {
      slot_of[r] = -1;
      continue;
    }
    const int32_t s = cursor[e]++;
    sorted[s] = (int32_t)r;
    slot_of[r] = s;
  }
  free(cursor);
  return bad;
}

/* Dot of one decoded fp32 weight row with one fp32 input row, in the
 * reference's 4-accumulator order. */
static float dot4(const float* w, const float* x, size_t K) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  size_t k = 0;
  for (; k + 4 <= K; k += 4) {
    a0 += x[k + 0] * w[k + 0];
    a1 += x[k + 1] * w[k + 1];
    a2 += x[k + 2] * w[k + 2];
    a3 += x[k + 3] * w[k + 3];
  }
  for (; k < K; ++k) a0 += x[k] * w[k];
  return (a0 + a1) + (a2 + a3);
}

static void decode_row(const uint8_t* q, const uint8_t* sf, float g, float* w,
                       size_t cols) {
  const size_t kb = cols / 16;
  for (size_t b = 0; b < kb; ++b) {
    const float bs = sbo_e4m3(sf[b]) * g;
    for (size_t j = 0; j < 8; ++j) {
      const uint8_t byte = q[b * 8 + j];
      w[b * 16 + 2 * j] = sbo_e2m1(byte & 0x0Fu) * bs;
      w[b * 16 + 2 * j + 1] = sbo_e2m1(byte >> 4) * bs;
    }
  }
}

static float silu(float x) { return x / (1.0f + expf(-x)); }

/* One routed expert applied to one token: y[K] = W2 (silu(W1 x) * (W3 x)). */
static void expert_ffn(const float* x, const uint8_t* w13, const uint8_t* s13,
                       float g13, const uint8_t* w2, const uint8_t* s2,
                       float g2, size_t K, size_t I, float* wrow, float* h,
                       float* y) {
  for (size_t i = 0; i < I; ++i) {
    decode_row(w13 + i * (K / 2), s13 + i * (K / 16), g13, wrow, K);
    const float gv = dot4(wrow, x, K);
    decode_row(w13 + (I + i) * (K / 2), s13 + (I + i) * (K / 16), g13, wrow, K);
    const float uv = dot4(wrow, x, K);
    h[i] = silu(gv) * uv;
  }
  for (size_t n = 0; n < K; ++n) {
    decode_row(w2 + n * (I / 2), s2 + n * (I / 16), g2, wrow, I);
    y[n] = dot4(wrow, h, I);
  }
}

typedef struct {
  const uint16_t* hidden;
  const int32_t* ids;
  const float* weights;
  const uint8_t *w13, *s13, *w2, *s2;
  const float *g13, *g2;
  size_t E, top_k, K, I;
  int multiply_router_weight;
  const int32_t* tokens;
  size_t n_tokens;
  float* out;
  size_t begin, end;
} moe_job;

static void* moe_worker(void* arg) {
  moe_job* j = (moe_job*)arg;
  const size_t K = j->K, I = j->I;
  const size_t kmax = K > I ? K : I;
  float* x = (float*)malloc(K * sizeof(float));
  float* wrow = (float*)malloc(kmax * sizeof(float));
  float* h = (float*)malloc(I * sizeof(float));
  float* y = (float*)malloc(K * sizeof(float));
  for (size_t ti = j->begin; ti < j->end; ++ti) {
    const size_t t = (size_t)j->tokens[ti];
    float* o = j->out + ti * K;
    for (size_t n = 0; n < K; ++n) o[n] = 0.0f;
    for (size_t k = 0; k < K; ++k) x[k] = bf16_to_f32(j->hidden[t * K + k]);
    /* The reference scatters expert by expert in ascending id, so a token's
     * contributions are summed in (expert, k) order. */
    size_t order[64];
    size_t n_ord = 0;
    for (size_t kk = 0; kk < j->top_k && n_ord < 64; ++kk) {
      size_t p = n_ord++;
      while (p > 0 && j->ids[t * j->top_k + order[p - 1]] > j->ids[t * j->top_k + kk]) {
        order[p] = order[p - 1];
        --p;
      }
      order[p] = kk;
    }
    for (size_t oi = 0; oi < n_ord; ++oi) {
      const size_t kk = order[oi];
      const int32_t e = j->ids[t * j->top_k + kk];
      if (e < 0 || (size_t)e >= j->E) continue;
      const size_t ue = (size_t)e;
      expert_ffn(x, j->w13 + ue * 2 * I * (K / 2), j->s13 + ue * 2 * I * (K / 16),
                 j->g13[ue], j->w2 + ue * K * (I / 2), j->s2 + ue * K * (I / 16),
                 j->g2[ue], K, I, wrow, h, y);
      const float w = j->multiply_router_weight ? j->weights[t * j->top_k + kk] : 1.0f;
      for (size_t n = 0; n < K; ++n) o[n] += w * y[n];
    }
  }
  free(x);
  free(wrow);
  free(h);
  free(y);
  return NULL;
}

/* Routed-expert MoE for a list of tokens. out is [n_tokens, K] fp32, row i
 * holding token tokens[i]. Each token's result depends only on its own routes,
 * so a sampled token list checks a full-size batch exactly. */
int sbo_moe_forward_tokens(const uint16_t* hidden, const int32_t* ids,
                           const float* weights, const uint8_t* w13,
                           const uint8_t* s13, const float* g13,
                           const uint8_t* w2, const uint8_t* s2,
                           const float* g2, size_t E, size_t top_k, size_t K,
                           size_t I, int multiply_router_weight,
                           const int32_t* tokens, size_t n_tokens, float* out,
                           int n_threads) {
  if (K % 16 || I % 16) return -1;
  if (top_k > 64) return -2;
  if (n_threads < 1) n_threads = 1;
  if ((size_t)n_threads > n_tokens) n_threads = n_tokens ? (int)n_tokens : 1;
  moe_job* jobs = (moe_job*)calloc((size_t)n_threads, sizeof(moe_job));
  pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
  const size_t per = (n_tokens + (size_t)n_threads - 1) / (size_t)n_threads;
  for (int i = 0; i < n_threads; ++i) {
    moe_job* j = &jobs[i];
    j->hidden = hidden; j->ids = ids; j->weights = weights;
    j->w13 = w13; j->s13 = s13; j->w2 = w2; j->s2 = s2; j->g13 = g13; j->g2 = g2;
    j->E = E; j->top_k = top_k; j->K = K; j->I = I;
    j->multiply_router_weight = multiply_router_weight;
    j->tokens = tokens; j->n_tokens = n_tokens; j->out = out;
    j->begin = (size_t)i * per;
    j->end = j->begin + per > n_tokens ? n_tokens : j->begin + per;
    if (j->begin > j->end) j->begin = j->end;
    pthread_create(&th[i], NULL, moe_worker, j);
  }
  for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
  free(jobs);
  free(th);
  return 0;
}
