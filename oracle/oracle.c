/*
 * CPU oracle for the Llama decode step -- TEST INFRASTRUCTURE ONLY.
 * See oracle.h for what is restated, from which reference file:line, and who
 * may call it. Build: oracle/Makefile (gcc, -ffp-contract=off so every fp32
 * operation the sampler restates is a single IEEE rounding, as on the GPU).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* bf16                                                                      */
/* ------------------------------------------------------------------------ */

float orc_bf16_to_float(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t orc_float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  }
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

static inline float rb(float f) { return orc_bf16_to_float(orc_float_to_bf16(f)); }

void orc_round_bf16_inplace(float* x, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = rb(x[i]);
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* Config-level                                                              */
/* ------------------------------------------------------------------------ */

/* src/config.cpp:223-259: theta^(-2i/d) in double, rounded to float, then the
 * llama3 three-band rescaling evaluated in double from that float. */
void orc_rope_inv_freq(const orc_config* c, float* out) {
  const int pairs = c->head_dim / 2;
  for (int i = 0; i < pairs; ++i) {
    const double exponent = (double)(2 * i) / c->head_dim;
    out[i] = (float)(1.0 / pow((double)c->theta, exponent));
  }
  if (!c->rope_scaling) return;
  const double old_context = c->rope_orig_ctx;
  const double low_wavelen = old_context / c->rope_low;
  const double high_wavelen = old_context / c->rope_high;
  const double two_pi = 2.0 * M_PI;
  for (int i = 0; i < pairs; ++i) {
    const double freq = out[i];
    const double wavelen = two_pi / freq;
    double scaled;
    if (wavelen < high_wavelen) {
      scaled = freq;
    } else if (wavelen > low_wavelen) {
      scaled = freq / c->rope_factor;
    } else {
      const double smooth = (old_context / wavelen - c->rope_low) /
                            (c->rope_high - c->rope_low);
      scaled = (1.0 - smooth) * (freq / c->rope_factor) + smooth * freq;
    }
    out[i] = (float)scaled;
  }
}

/* src/model.cu:91-102: every projection, both norms per layer, the final norm
 * and the output head; one embedding row is not counted. */
size_t orc_weight_bytes_per_token(const orc_config* c) {
  const size_t h = (size_t)c->hidden, q = (size_t)c->heads * c->head_dim;
  const size_t kv = (size_t)c->kv_heads * c->head_dim, f = (size_t)c->ffn;
  size_t per = 0;
  for (int l = 0; l < c->layers; ++l) {
    per += h * 2 + q * h + kv * h * 2 + h * q + f * h * 3;
  }
  per += h + (size_t)c->vocab * h;
  return per * 2;
}

/* ------------------------------------------------------------------------ */
/* Kernel maths                                                              */
/* ------------------------------------------------------------------------ */

/* y[r] = sum_k W[r][k] x[k] in fp32 (cuBLAS gemm_nt with fp32 compute,
 * src/model.cu:38-45, is the operation being restated): sixteen interleaved
 * fp32 partial sums, added in double at the end. */
static void gemv_f(float* y, const uint16_t* w, const float* x, int rows,
                   int cols) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint16_t* row = w + (size_t)r * cols;
    /* 16 fp32 partial sums (columns k mod 16), combined in double. */
    float part[16] = {0};
    int k = 0;
    for (; k + 16 <= cols; k += 16) {
      for (int j = 0; j < 16; ++j) {
        uint32_t u = (uint32_t)row[k + j] << 16;
        float wf;
        memcpy(&wf, &u, 4);
        part[j] = fmaf(wf, x[k + j], part[j]);
      }
    }
    for (; k < cols; ++k) {
      uint32_t u = (uint32_t)row[k] << 16;
      float wf;
      memcpy(&wf, &u, 4);
      part[k & 15] = fmaf(wf, x[k], part[k & 15]);
    }
    double acc = 0.0;
    for (int j = 0; j < 16; ++j) acc += part[j];
    y[r] = (float)acc;
  }
}

/* The same product summed in the opposite order, one fp32 accumulator
 * (ORC_MODE_BF16_REORDERED): a second, equally valid evaluation order, to
 * measure how far two implementations of the bf16-storage algorithm drift
 * apart from summation order alone. */
static void gemv_f_reordered(float* y, const uint16_t* w, const float* x,
                             int rows, int cols) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint16_t* row = w + (size_t)r * cols;
    float acc = 0.f;
    for (int k = cols - 1; k >= 0; --k) {
      uint32_t u = (uint32_t)row[k] << 16;
      float wf;
      memcpy(&wf, &u, 4);
      acc = fmaf(wf, x[k], acc);
    }
    y[r] = acc;
  }
}

void orc_gemv(float* y, const uint16_t* w, const uint16_t* x, int rows,
              int cols) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)cols);
  for (int k = 0; k < cols; ++k) xf[k] = orc_bf16_to_float(x[k]);
  gemv_f(y, w, xf, rows, cols);
  free(xf);
}

/* src/kernels/rmsnorm.cu:21-63: scale = rsqrt(mean(x^2) + eps) with an fp32
 * sum of squares; out = x * scale * w evaluated left to right in fp32. The sum
 * of squares is taken over `sq_src` (the unrounded residual sum in the fused
 * kernel, src/kernels/rmsnorm.cu:84-96) and the scaling over `x`. */
static void rmsnorm_f(float* out, const float* x, const float* sq_src,
                      const uint16_t* w, int dim, float eps, int round_out) {
  double sum = 0.0;
  for (int i = 0; i < dim; ++i) sum += (double)sq_src[i] * sq_src[i];
  const float scale = (float)(1.0 / sqrt(sum / dim + (double)eps));
  for (int i = 0; i < dim; ++i) {
    float v = (x[i] * scale) * orc_bf16_to_float(w[i]);
    out[i] = round_out ? rb(v) : v;
  }
}

void orc_rmsnorm(float* out, const uint16_t* x, const uint16_t* weight,
                 int tokens, int dim, float eps, int round_out) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)dim);
  for (int t = 0; t < tokens; ++t) {
    for (int i = 0; i < dim; ++i) xf[i] = orc_bf16_to_float(x[(size_t)t * dim + i]);
    rmsnorm_f(out + (size_t)t * dim, xf, xf, weight, dim, eps, round_out);
  }
  free(xf);
}

/* src/kernels/rmsnorm.cu:68-119: x += delta (stored bf16), sum of squares over
 * the unrounded sums, scaling over the stored (rounded) x. */
void orc_add_residual_rmsnorm(float* out, uint16_t* x, const uint16_t* delta,
                              const uint16_t* weight, int tokens, int dim,
                              float eps) {
  float* sum = (float*)malloc(sizeof(float) * (size_t)dim);
  float* xr = (float*)malloc(sizeof(float) * (size_t)dim);
  for (int t = 0; t < tokens; ++t) {
    for (int i = 0; i < dim; ++i) {
      const size_t k = (size_t)t * dim + i;
      sum[i] = orc_bf16_to_float(x[k]) + orc_bf16_to_float(delta[k]);
      x[k] = orc_float_to_bf16(sum[i]);
      xr[i] = orc_bf16_to_float(x[k]);
    }
    rmsnorm_f(out + (size_t)t * dim, xr, sum, weight, dim, eps, 1);
  }
  free(sum);
  free(xr);
}

/* src/kernels/elementwise.cu:64-68: silu(v) = v / (1 + exp(-v)). */
static float silu_f(float v) { return (float)((double)v / (1.0 + exp(-(double)v))); }

void orc_swiglu(float* out, const uint16_t* gate, const uint16_t* up,
                long count) {
  for (long i = 0; i < count; ++i) {
    out[i] = silu_f(orc_bf16_to_float(gate[i])) * orc_bf16_to_float(up[i]);
  }
}

/* src/kernels/rope.cu:9-11, 33-56: element i pairs with i + d/2; the angle is
 * the fp32 product float(position) * inv_freq[i]. */
static void rope_head(float* out, const float* in, const float* inv_freq,
                      int position, int head_dim) {
  const int half = head_dim / 2;
  for (int i = 0; i < half; ++i) {
    const float angle = (float)position * inv_freq[i];
    const double s = sin((double)angle), co = cos((double)angle);
    const double lo = in[i], hi = in[i + half];
    out[i] = (float)(lo * co - hi * s);
    out[i + half] = (float)(hi * co + lo * s);
  }
}

void orc_rope_rows(float* out, const uint16_t* in, const float* inv_freq,
                   int tokens, int start_position, int heads, int head_dim,
                   int src_row_stride, int head_major) {
  float* src = (float*)malloc(sizeof(float) * (size_t)head_dim);
  for (int t = 0; t < tokens; ++t) {
    for (int h = 0; h < heads; ++h) {
      for (int i = 0; i < head_dim; ++i) {
        src[i] = orc_bf16_to_float(in[(size_t)t * src_row_stride + (size_t)h * head_dim + i]);
      }
      float* dst = head_major ? out + ((size_t)h * tokens + t) * head_dim
                              : out + ((size_t)t * heads + h) * head_dim;
      rope_head(dst, src, inv_freq, start_position + t, head_dim);
    }
  }
  free(src);
}

/* Nested-loop GQA decode attention (tests/test_kernels.cu:341-381; the kernel
 * is src/kernels/attention.cu:110-299). keys/values are [pos][kv_heads][d]. */
void orc_attention(float* out, const uint16_t* q, const uint16_t* keys,
                   const uint16_t* values, int num_heads, int num_kv_heads,
                   int head_dim, int positions, float scale) {
  const int group = num_heads / num_kv_heads;
  double* sc = (double*)malloc(sizeof(double) * (size_t)(positions > 0 ? positions : 1));
  for (int h = 0; h < num_heads; ++h) {
    const int kv = h / group;
    double mx = -INFINITY;
    for (int p = 0; p < positions; ++p) {
      double dot = 0.0;
      for (int d = 0; d < head_dim; ++d) {
        dot += (double)orc_bf16_to_float(q[(size_t)h * head_dim + d]) *
               orc_bf16_to_float(keys[((size_t)p * num_kv_heads + kv) * head_dim + d]);
      }
      sc[p] = dot * scale;
      if (sc[p] > mx) mx = sc[p];
    }
    double sum = 0.0;
    for (int p = 0; p < positions; ++p) {
      sc[p] = exp(sc[p] - mx);
      sum += sc[p];
    }
    for (int d = 0; d < head_dim; ++d) {
      double acc = 0.0;
      for (int p = 0; p < positions; ++p) {
        acc += sc[p] * orc_bf16_to_float(values[((size_t)p * num_kv_heads + kv) * head_dim + d]);
      }
      out[(size_t)h * head_dim + d] = (float)(acc / sum);
    }
  }
  free(sc);
}

/* ------------------------------------------------------------------------ */
/* The decode step: Model::decode -> run_layers(1, position)                 */
/* (src/model.cu:347-368, 370-484)                                           */
/* ------------------------------------------------------------------------ */

struct orc_state {
  orc_config c;
  int max_seq;
  float* k; /* [layers][kv_heads][max_seq][head_dim], the contiguous layout of
               src/kv_cache.cu:104-119 */
  float* v;
  float* inv_freq;
};

orc_state* orc_state_new(const orc_config* c, int max_seq) {
  orc_state* s = (orc_state*)calloc(1, sizeof(orc_state));
  s->c = *c;
  s->max_seq = max_seq;
  const size_t n = (size_t)c->layers * c->kv_heads * (size_t)max_seq * c->head_dim;
  s->k = (float*)calloc(n, sizeof(float));
  s->v = (float*)calloc(n, sizeof(float));
  s->inv_freq = (float*)malloc(sizeof(float) * (size_t)(c->head_dim / 2));
  orc_rope_inv_freq(c, s->inv_freq);
  return s;
}

void orc_state_free(orc_state* s) {
  if (!s) return;
  free(s->k);
  free(s->v);
  free(s->inv_freq);
  free(s);
}

void orc_state_reset(orc_state* s) {
  const orc_config* c = &s->c;
  const size_t n = (size_t)c->layers * c->kv_heads * (size_t)s->max_seq * c->head_dim;
  memset(s->k, 0, n * sizeof(float));
  memset(s->v, 0, n * sizeof(float));
}

int orc_decode(const orc_config* c, const orc_weights* w, orc_state* s,
               int token, int position, int mode, float* logits, float* taps) {
  if (token < 0 || token >= c->vocab || position < 0 || position >= s->max_seq) return 1;
  const int bf = (mode == ORC_MODE_BF16 || mode == ORC_MODE_BF16_REORDERED);
  const int kvbf = bf || mode == ORC_MODE_FP32_KV_BF16; /* the cache stores bf16 */
  void (*gemv)(float*, const uint16_t*, const float*, int, int) =
      mode == ORC_MODE_BF16_REORDERED ? gemv_f_reordered : gemv_f;
  const int H = c->hidden, F = c->ffn, d = c->head_dim;
  const int qd = c->heads * d, kvd = c->kv_heads * d, group = c->heads / c->kv_heads;
  const int seq = position + 1;
  const float scale = 1.0f / sqrtf((float)d);

  float* x = (float*)malloc(sizeof(float) * H);      /* residual stream */
  float* xsum = (float*)malloc(sizeof(float) * H);   /* unrounded residual sum */
  float* normed = (float*)malloc(sizeof(float) * H);
  float* qkv = (float*)malloc(sizeof(float) * (qd + 2 * kvd));
  float* qr = (float*)malloc(sizeof(float) * qd);
  float* attn = (float*)malloc(sizeof(float) * qd);
  float* proj = (float*)malloc(sizeof(float) * H);
  float* gu = (float*)malloc(sizeof(float) * 2 * F);
  float* act = (float*)malloc(sizeof(float) * F);
  double* sc = (double*)malloc(sizeof(double) * seq);

  /* Embedding row (src/kernels/elementwise.cu:25-41): exact copy. */
  for (int i = 0; i < H; ++i) x[i] = orc_bf16_to_float(w->embed[(size_t)token * H + i]);
  memcpy(xsum, x, sizeof(float) * H);
  if (taps) memcpy(taps, x, sizeof(float) * H);

  for (int l = 0; l < c->layers; ++l) {
    /* input norm: unfused for layer 0, otherwise fused into the previous
       layer's MLP residual join (src/model.cu:384-388, 449-458) */
    rmsnorm_f(normed, x, xsum, w->input_norm[l], H, c->eps, bf);

    gemv(qkv, w->qkv[l], normed, qd + 2 * kvd, H);
    if (bf) orc_round_bf16_inplace(qkv, (size_t)(qd + 2 * kvd));

    /* RoPE on Q (head-major out, bf16) and K, plus the cache write
       (src/kernels/rope.cu:33-87). V is copied unrotated. */
    for (int h = 0; h < c->heads; ++h) {
      rope_head(qr + (size_t)h * d, qkv + (size_t)h * d, s->inv_freq, position, d);
    }
    if (bf) orc_round_bf16_inplace(qr, (size_t)qd);
    float kr[256];
    for (int h = 0; h < c->kv_heads; ++h) {
      rope_head(kr, qkv + qd + (size_t)h * d, s->inv_freq, position, d);
      const size_t base = (((size_t)l * c->kv_heads + h) * s->max_seq + position) * d;
      for (int i = 0; i < d; ++i) {
        s->k[base + i] = kvbf ? rb(kr[i]) : kr[i];
        const float v = qkv[qd + kvd + (size_t)h * d + i];
        s->v[base + i] = kvbf ? rb(v) : v;
      }
    }

    /* GQA decode attention over positions 0..position
       (src/kernels/attention.cu:110-299): q scaled once, fp32 softmax. */
    for (int h = 0; h < c->heads; ++h) {
      const int kv = h / group;
      const float* kb = s->k + (((size_t)l * c->kv_heads + kv) * s->max_seq) * d;
      const float* vb = s->v + (((size_t)l * c->kv_heads + kv) * s->max_seq) * d;
      float qs[256];
      for (int i = 0; i < d; ++i) qs[i] = qr[(size_t)h * d + i] * scale;
      double mx = -INFINITY;
      for (int p = 0; p < seq; ++p) {
        double dot = 0.0;
        for (int i = 0; i < d; ++i) dot += (double)qs[i] * kb[(size_t)p * d + i];
        sc[p] = dot;
        if (dot > mx) mx = dot;
      }
      double sum = 0.0;
      for (int p = 0; p < seq; ++p) {
        sc[p] = exp(sc[p] - mx);
        sum += sc[p];
      }
      for (int i = 0; i < d; ++i) {
        double acc = 0.0;
        for (int p = 0; p < seq; ++p) acc += sc[p] * vb[(size_t)p * d + i];
        attn[(size_t)h * d + i] = (float)(acc / sum);
      }
    }
    if (bf) orc_round_bf16_inplace(attn, (size_t)qd);

    /* o_proj, then the attention residual join fused with the post-attention
       norm (src/model.cu:418-428). */
    gemv(proj, w->o[l], attn, H, qd);
    if (bf) orc_round_bf16_inplace(proj, (size_t)H);
    for (int i = 0; i < H; ++i) {
      xsum[i] = x[i] + proj[i];
      x[i] = bf ? rb(xsum[i]) : xsum[i];
    }
    rmsnorm_f(normed, x, xsum, w->post_norm[l], H, c->eps, bf);

    /* gate/up as one [2F][H] GEMM, then SwiGLU on the two halves
       (src/model.cu:429-438). */
    gemv(gu, w->gate_up[l], normed, 2 * F, H);
    if (bf) orc_round_bf16_inplace(gu, (size_t)2 * F);
    for (int i = 0; i < F; ++i) {
      const float a = silu_f(gu[i]) * gu[F + i];
      act[i] = bf ? rb(a) : a;
    }

    /* down_proj and the MLP residual join (src/model.cu:439-458). */
    gemv(proj, w->down[l], act, H, F);
    if (bf) orc_round_bf16_inplace(proj, (size_t)H);
    for (int i = 0; i < H; ++i) {
      xsum[i] = x[i] + proj[i];
      x[i] = bf ? rb(xsum[i]) : xsum[i];
    }
    if (taps) memcpy(taps + (size_t)(l + 1) * H, x, sizeof(float) * H);
  }

  /* final norm fused into the last residual join, then the tied lm_head on
     the last row with fp32 logits (src/model.cu:449-483). */
  rmsnorm_f(normed, x, xsum, w->final_norm, H, c->eps, bf);
  if (taps) memcpy(taps + (size_t)(c->layers + 1) * H, normed, sizeof(float) * H);
  gemv(logits, w->lm_head, normed, c->vocab, H);

  free(x); free(xsum); free(normed); free(qkv); free(qr); free(attn);
  free(proj); free(gu); free(act); free(sc);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Chunked prefill: Model::prefill -> run_layers(n, start)                   */
/* (src/model.cu:308-345, 370-484, attention 509-560)                        */
/* ------------------------------------------------------------------------ */

#include <immintrin.h>

static inline float hsum8(__m256 v) {
  float t[8];
  _mm256_storeu_ps(t, v);
  double s = 0.0;
  for (int i = 0; i < 8; ++i) s += t[i];
  return (float)s;
}

/* Y[t * ldy + r] = sum_k W[r][k] X[t][k] for n rows of X (cols a multiple of
 * 8): the chunk's projection as one GEMM, gemm_nt of src/model.cu:38-45 with
 * fp32 accumulation. Weight rows are widened once per 8-row block; each
 * (2 tokens x 2 rows) tile keeps eight fp32 lanes per product and sums the
 * lanes in double. */
static void gemm_f(float* Y, int ldy, const uint16_t* W, const float* X, int n,
                   int rows, int cols) {
#pragma omp parallel
  {
    float* wf = (float*)aligned_alloc(32, sizeof(float) * 8 * (size_t)cols);
#pragma omp for schedule(dynamic, 1)
    for (int r0 = 0; r0 < rows; r0 += 8) {
      const int nr = rows - r0 < 8 ? rows - r0 : 8;
      for (int r = 0; r < nr; ++r) {
        const uint16_t* src = W + (size_t)(r0 + r) * cols;
        for (int k = 0; k < cols; ++k) wf[(size_t)r * cols + k] = orc_bf16_to_float(src[k]);
      }
      for (int t = 0; t < n; t += 2) {
        const int nt = n - t < 2 ? n - t : 2;
        const float* x0 = X + (size_t)t * cols;
        const float* x1 = X + (size_t)(t + nt - 1) * cols;
        for (int r = 0; r < nr; r += 2) {
          const int r1 = r + 1 < nr ? r + 1 : r;
          const float* w0 = wf + (size_t)r * cols;
          const float* w1 = wf + (size_t)r1 * cols;
          __m256 a00 = _mm256_setzero_ps(), a01 = a00, a10 = a00, a11 = a00;
          for (int k = 0; k < cols; k += 8) {
            const __m256 xv0 = _mm256_loadu_ps(x0 + k), xv1 = _mm256_loadu_ps(x1 + k);
            const __m256 wv0 = _mm256_load_ps(w0 + k), wv1 = _mm256_load_ps(w1 + k);
            a00 = _mm256_fmadd_ps(xv0, wv0, a00);
            a01 = _mm256_fmadd_ps(xv0, wv1, a01);
            a10 = _mm256_fmadd_ps(xv1, wv0, a10);
            a11 = _mm256_fmadd_ps(xv1, wv1, a11);
          }
          Y[(size_t)t * ldy + r0 + r] = hsum8(a00);
          if (r1 != r) Y[(size_t)t * ldy + r0 + r1] = hsum8(a01);
          if (nt == 2) {
            Y[(size_t)(t + 1) * ldy + r0 + r] = hsum8(a10);
            if (r1 != r) Y[(size_t)(t + 1) * ldy + r0 + r1] = hsum8(a11);
          }
        }
      }
    }
    free(wf);
  }
}

static inline float dot8n(const float* a, const float* b, int d) {
  __m256 acc = _mm256_setzero_ps();
  for (int i = 0; i < d; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
  return hsum8(acc);
}

int orc_prefill(const orc_config* c, const orc_weights* w, orc_state* s,
                const int32_t* tokens, int n, int start, int mode,
                float* last_logits) {
  if (n <= 0 || start < 0 || start + n > s->max_seq) return 1;
  if (mode != ORC_MODE_FP32 && mode != ORC_MODE_BF16 && mode != ORC_MODE_FP32_KV_BF16) return 2;
  for (int t = 0; t < n; ++t) {
    if (tokens[t] < 0 || tokens[t] >= c->vocab) return 1;
  }
  const int bf = mode == ORC_MODE_BF16;
  const int kvbf = bf || mode == ORC_MODE_FP32_KV_BF16;
  const int H = c->hidden, F = c->ffn, d = c->head_dim;
  const int qd = c->heads * d, kvd = c->kv_heads * d, group = c->heads / c->kv_heads;
  const int nqkv = qd + 2 * kvd;
  if (H % 8 || F % 8 || d % 8 || qd % 8) return 2;
  const float scale = 1.0f / sqrtf((float)d);
  const size_t N = (size_t)n;

  float* x = (float*)malloc(sizeof(float) * N * H);
  float* xsum = (float*)malloc(sizeof(float) * N * H);
  float* normed = (float*)malloc(sizeof(float) * N * (H > qd ? H : qd));
  float* qkv = (float*)malloc(sizeof(float) * N * nqkv);
  float* qr = (float*)malloc(sizeof(float) * N * qd);
  float* attn = (float*)malloc(sizeof(float) * N * qd);
  float* proj = (float*)malloc(sizeof(float) * N * H);
  float* gu = (float*)malloc(sizeof(float) * N * 2 * F);
  float* act = (float*)malloc(sizeof(float) * N * F);

  for (size_t t = 0; t < N; ++t) {
    for (int i = 0; i < H; ++i) x[t * H + i] = orc_bf16_to_float(w->embed[(size_t)tokens[t] * H + i]);
  }
  memcpy(xsum, x, sizeof(float) * N * H);

  for (int l = 0; l < c->layers; ++l) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; ++t) {
      rmsnorm_f(normed + (size_t)t * H, x + (size_t)t * H, xsum + (size_t)t * H, w->input_norm[l], H, c->eps, bf);
    }
    gemm_f(qkv, nqkv, w->qkv[l], normed, n, nqkv, H);
    if (bf) orc_round_bf16_inplace(qkv, N * nqkv);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; ++t) {
      const int pos = start + t;
      const float* row = qkv + (size_t)t * nqkv;
      for (int h = 0; h < c->heads; ++h) {
        rope_head(qr + (size_t)t * qd + (size_t)h * d, row + (size_t)h * d, s->inv_freq, pos, d);
      }
      float kr[256];
      for (int h = 0; h < c->kv_heads; ++h) {
        rope_head(kr, row + qd + (size_t)h * d, s->inv_freq, pos, d);
        const size_t base = (((size_t)l * c->kv_heads + h) * s->max_seq + pos) * d;
        for (int i = 0; i < d; ++i) {
          s->k[base + i] = kvbf ? rb(kr[i]) : kr[i];
          const float v = row[qd + kvd + (size_t)h * d + i];
          s->v[base + i] = kvbf ? rb(v) : v;
        }
      }
    }
    if (bf) orc_round_bf16_inplace(qr, N * qd);
    /* causal GQA attention of every chunk row over the cache up to its own
       position, q scaled once, fp32 softmax. In ORC_MODE_BF16 a chunk of more
       than one row stores the normalised probabilities as bf16 before they
       multiply V (causal_softmax_kernel, src/kernels/attention.cu:42-100,
       feeding the P.V GEMM of src/model.cu:545-551); a chunk of one row takes
       the decode attention, fp32 throughout (src/model.cu:412-413). */
    const int round_p = bf && n > 1;
#pragma omp parallel
    {
      float* sc = (float*)malloc(sizeof(float) * (size_t)(start + n));
      float qs[256], acc[256];
#pragma omp for schedule(dynamic, 4) collapse(2)
      for (int t = 0; t < n; ++t) {
        for (int h = 0; h < c->heads; ++h) {
          const int seq = start + t + 1, kv = h / group;
          const float* kb = s->k + (((size_t)l * c->kv_heads + kv) * s->max_seq) * d;
          const float* vb = s->v + (((size_t)l * c->kv_heads + kv) * s->max_seq) * d;
          for (int i = 0; i < d; ++i) qs[i] = qr[(size_t)t * qd + (size_t)h * d + i] * scale;
          float mx = -INFINITY;
          for (int p = 0; p < seq; ++p) {
            sc[p] = dot8n(qs, kb + (size_t)p * d, d);
            if (sc[p] > mx) mx = sc[p];
          }
          double sum = 0.0;
          for (int p = 0; p < seq; ++p) {
            sc[p] = (float)exp((double)sc[p] - mx);
            sum += sc[p];
          }
          const float inv_sum = (float)(1.0 / sum);
          if (round_p) {
            for (int p = 0; p < seq; ++p) sc[p] = rb(sc[p] * inv_sum);
          }
          for (int i = 0; i < d; ++i) acc[i] = 0.f;
          for (int p = 0; p < seq; ++p) {
            const __m256 pv = _mm256_set1_ps(sc[p]);
            for (int i = 0; i < d; i += 8) {
              _mm256_storeu_ps(acc + i, _mm256_fmadd_ps(pv, _mm256_loadu_ps(vb + (size_t)p * d + i),
                                                        _mm256_loadu_ps(acc + i)));
            }
          }
          for (int i = 0; i < d; ++i) {
            attn[(size_t)t * qd + (size_t)h * d + i] = round_p ? acc[i] : (float)(acc[i] / sum);
          }
        }
      }
      free(sc);
    }
    if (bf) orc_round_bf16_inplace(attn, N * qd);

    gemm_f(proj, H, w->o[l], attn, n, H, qd);
    if (bf) orc_round_bf16_inplace(proj, N * H);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; ++t) {
      float* xr = x + (size_t)t * H;
      float* sr = xsum + (size_t)t * H;
      for (int i = 0; i < H; ++i) {
        sr[i] = xr[i] + proj[(size_t)t * H + i];
        xr[i] = bf ? rb(sr[i]) : sr[i];
      }
      rmsnorm_f(normed + (size_t)t * H, xr, sr, w->post_norm[l], H, c->eps, bf);
    }

    gemm_f(gu, 2 * F, w->gate_up[l], normed, n, 2 * F, H);
    if (bf) orc_round_bf16_inplace(gu, N * 2 * F);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; ++t) {
      for (int i = 0; i < F; ++i) {
        const float a = silu_f(gu[(size_t)t * 2 * F + i]) * gu[(size_t)t * 2 * F + F + i];
        act[(size_t)t * F + i] = bf ? rb(a) : a;
      }
    }

    gemm_f(proj, H, w->down[l], act, n, H, F);
    if (bf) orc_round_bf16_inplace(proj, N * H);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; ++t) {
      float* xr = x + (size_t)t * H;
      float* sr = xsum + (size_t)t * H;
      for (int i = 0; i < H; ++i) {
        sr[i] = xr[i] + proj[(size_t)t * H + i];
        xr[i] = bf ? rb(sr[i]) : sr[i];
      }
    }
  }

  if (last_logits) {
    const size_t t = N - 1;
    rmsnorm_f(normed, x + t * H, xsum + t * H, w->final_norm, H, c->eps, bf);
    gemv_f(last_logits, w->lm_head, normed, c->vocab, H);
  }
  free(x); free(xsum); free(normed); free(qkv); free(qr); free(attn);
  free(proj); free(gu); free(act);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Sampling                                                                  */
/* ------------------------------------------------------------------------ */

/* Greedy: the largest logit, ties to the lowest index -- the packed
 * (order key, ~index) atomicMax of src/kernels/sampling.cu:42-67. */
int orc_argmax(const float* logits, int vocab) {
  int best = 0;
  for (int i = 1; i < vocab; ++i) {
    if (logits[i] > logits[best]) best = i;
  }
  return best;
}

/* exp(x) by Cody-Waite reduction (x = k ln2 + r, ln2 split into a float head
 * and tail) and the degree-7 Taylor polynomial of exp(r) on |r| <= ln2/2,
 * evaluated by Horner with fused multiply-adds, then scaled by 2^k in two
 * exact steps. Every operation is a single IEEE fp32 rounding, so the CUDA
 * sampler's copy of this function returns the same bits. */
float orc_det_expf(float x) {
  if (!(x > -88.0f)) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float kLog2e = 1.44269504088896341f;
  const float kLn2Hi = 0.693147182464599609375f;
  const float kLn2Lo = -1.904654299957768e-09f;
  const float k = rintf(x * kLog2e);
  float r = fmaf(-k, kLn2Hi, x);
  r = fmaf(-k, kLn2Lo, r);
  float p = 1.98412698412698413e-4f; /* 1/7! */
  p = fmaf(p, r, 1.38888888888888889e-3f); /* 1/6! */
  p = fmaf(p, r, 8.33333333333333333e-3f); /* 1/5! */
  p = fmaf(p, r, 4.16666666666666667e-2f); /* 1/4! */
  p = fmaf(p, r, 1.66666666666666667e-1f); /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = (int)k;
  const int k1 = ki / 2, k2 = ki - k1;
  uint32_t b1 = (uint32_t)(k1 + 127) << 23, b2 = (uint32_t)(k2 + 127) << 23;
  float s1, s2;
  memcpy(&s1, &b1, 4);
  memcpy(&s2, &b2, 4);
  return (p * s1) * s2;
}

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
 * easy as 1, 2, 3", SC'11): ten rounds of two 32x32->64 multiplies with the
 * Weyl key schedule. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2],
                       uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    const uint32_t n3 = (uint32_t)p0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* One uniform in [0, 1) for (seed, counter, stream): the top 24 bits of the
 * first Philox output word, times 2^-24 (exact). */
float orc_philox_uniform(uint64_t seed, uint64_t counter, uint32_t stream) {
  const uint32_t ctr[4] = {(uint32_t)counter, (uint32_t)(counter >> 32), stream, 0u};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t out[4];
  orc_philox4x32_10(ctr, key, out);
  return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

/* The CUDA sampler's fixed summation tree: 1024 strided per-thread sums in
 * index order, then an xor butterfly inside each warp of 32 and one more over
 * the 32 warp totals. */
float orc_tree_sum_1024(const float* e, int n) {
  float lane[1024];
  for (int t = 0; t < 1024; ++t) {
    float acc = 0.0f;
    for (int i = t; i < n; i += 1024) acc = acc + e[i];
    lane[t] = acc;
  }
  float warp[32];
  for (int w = 0; w < 32; ++w) {
    float v[32], nv[32];
    for (int l = 0; l < 32; ++l) v[l] = lane[w * 32 + l];
    for (int off = 16; off > 0; off >>= 1) {
      for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
      memcpy(v, nv, sizeof v);
    }
    warp[w] = v[0];
  }
  for (int off = 16; off > 0; off >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = warp[l] + warp[l ^ off];
    memcpy(warp, nv, sizeof nv);
  }
  return warp[0];
}

typedef struct {
  float s;
  int i;
} cand_t;

static int cand_cmp(const void* a, const void* b) {
  const cand_t* x = (const cand_t*)a;
  const cand_t* y = (const cand_t*)b;
  if (x->s > y->s) return -1;
  if (x->s < y->s) return 1;
  return (x->i > y->i) - (x->i < y->i);
}

/* Temperature / top-k / top-p sampling. Semantics of
 * src/kernels/sampling.cu:97-224 -- scaled s = (logit - max) / T, a full-vocab
 * exponential sum as the denominator, candidates walked in descending order,
 * cut at top_k or once the kept mass reaches top_p (the crossing token kept),
 * then a pick at uniform * kept_mass -- made exact and deterministic: the
 * candidates are the first min(top_k or vocab, 1024) tokens ordered by
 * (s desc, index asc), exp is orc_det_expf, and the denominator is
 * orc_tree_sum_1024. A temperature of zero (inv_temperature <= 0) is argmax. */
int orc_sample(const float* logits, int vocab, float inv_temperature,
               int top_k, float top_p, float uniform) {
  if (vocab <= 0) return -1;
  if (!(inv_temperature > 0.0f)) return orc_argmax(logits, vocab);
  float mx = logits[0];
  for (int i = 1; i < vocab; ++i) mx = logits[i] > mx ? logits[i] : mx;
  cand_t* c = (cand_t*)malloc(sizeof(cand_t) * (size_t)vocab);
  float* e = (float*)malloc(sizeof(float) * (size_t)vocab);
  for (int i = 0; i < vocab; ++i) {
    const float s = (logits[i] - mx) * inv_temperature;
    c[i].s = s;
    c[i].i = i;
    e[i] = orc_det_expf(s);
  }
  const float total = orc_tree_sum_1024(e, vocab);
  qsort(c, (size_t)vocab, sizeof(cand_t), cand_cmp);
  int m = top_k > 0 ? top_k : vocab;
  if (m > 1024) m = 1024;
  if (m > vocab) m = vocab;
  const float inv_total = 1.0f / total;
  int keep = 0;
  float kept = 0.0f;
  for (int j = 0; j < m; ++j) {
    const float p = e[c[j].i] * inv_total;
    kept = kept + p;
    ++keep;
    if (top_p < 1.0f && kept >= top_p) break;
  }
  const float target = uniform * kept;
  float running = 0.0f;
  int picked = c[0].i;
  for (int j = 0; j < keep; ++j) {
    const float p = e[c[j].i] * inv_total;
    running = running + p;
    picked = c[j].i;
    if (running >= target) break;
  }
  free(c);
  free(e);
  return picked;
}

/* ------------------------------------------------------------------------ */
/* Paged KV page allocator                                                    */
/* ------------------------------------------------------------------------ */

int orc_paged_reserve(int32_t* tables, int layers, int max_pages,
                      int page_size, int old_length, int new_length,
                      int pages_mapped, int pool_pages, const int32_t* order) {
  if (new_length <= old_length) return pages_mapped;
  const int have = (old_length + page_size - 1) / page_size;
  const int need = (new_length + page_size - 1) / page_size;
  if (need > max_pages) return -1;
  for (int l = 0; l < layers; ++l) {
    for (int p = have; p < need; ++p) {
      if (pages_mapped >= pool_pages) return -1;
      const int phys = order ? order[pages_mapped] : pages_mapped;
      tables[(size_t)l * max_pages + p] = phys;
      ++pages_mapped;
    }
  }
  return pages_mapped;
}

/* splitmix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number
 * generators", OOPSLA'14) driving a Fisher-Yates shuffle. */
static uint64_t splitmix64(uint64_t* state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void orc_page_permutation(int32_t* out, int n, uint64_t seed) {
  for (int i = 0; i < n; ++i) out[i] = i;
  uint64_t st = seed;
  for (int i = n - 1; i > 0; --i) {
    const int j = (int)(splitmix64(&st) % (uint64_t)(i + 1));
    const int32_t t = out[i];
    out[i] = out[j];
    out[j] = t;
  }
}
