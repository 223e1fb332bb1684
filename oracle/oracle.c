/*
 * oracle.c — CPU fp32 restatement of llm.cpp's GPT-2 training path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for libllmk's CUDA
 * kernels, never part of the product. Parity of this file against the
 * reference is pinned by tests/test_oracle_golden.py (the reference gtest
 * literals) and tests/test_oracle_vs_ref.py (the reference CPU sources
 * compiled into oracle/_ref/).
 *
 * Layout: row-major flat buffers, (B,T,C) activations, W as (OC, C) — the
 * byte layout of the reference's column-major Eigen (C, OC) weights.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ----------------------------------------------------------------- rng */
static uint64_t splitmix64(uint64_t* x) {
  uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

void orc_rng_seed(orc_rng* r, uint64_t seed, uint64_t stream) {
  uint64_t x = seed ^ (stream * 0xD1B54A32D192ED03ull);
  for (int i = 0; i < 4; ++i) r->s[i] = splitmix64(&x);
}
uint64_t orc_rng_next(orc_rng* r) {
  uint64_t* s = r->s;
  const uint64_t result = rotl(s[1] * 5, 7) * 9;
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl(s[3], 45);
  return result;
}
double orc_rng_uniform(orc_rng* r) { return (double)((orc_rng_next(r) >> 11) + 1) * (1.0 / 9007199254740992.0); }

void orc_fill_normal(float* out, size_t n, float stddev, uint64_t seed, uint64_t stream) {
  orc_rng r;
  orc_rng_seed(&r, seed, stream);
  const double two_pi = 6.283185307179586476925286766559;
  for (size_t i = 0; i < n; ++i) {
    double u1 = orc_rng_uniform(&r), u2 = orc_rng_uniform(&r);
    out[i] = (float)(sqrt(-2.0 * log(u1)) * cos(two_pi * u2) * (double)stddev);
  }
}
void orc_fill_tokens(int* out, size_t n, int vocab, uint64_t seed, uint64_t stream) {
  orc_rng r;
  orc_rng_seed(&r, seed, stream);
  for (size_t i = 0; i < n; ++i) out[i] = (int)(((orc_rng_next(&r) >> 32) * (uint64_t)vocab) >> 32);
}

/* -------------------------------------------------------------- matmul */
void orc_matmul_forward(float* out, const float* inp, const float* W, const float* bias, int BT, int C, int OC) {
  /* reference: outputs[b] = inputs[b] * weight, then += bias row-wise (matmul.cpp:23-35) */
#pragma omp parallel for schedule(static)
  for (int o = 0; o < OC; ++o) {
    const float* w = W + (size_t)o * C;
    const float b = bias ? bias[o] : 0.0f;
    for (int r = 0; r < BT; ++r) {
      const float* x = inp + (size_t)r * C;
      float s = 0.0f;
      for (int c = 0; c < C; ++c) s += x[c] * w[c];
      out[(size_t)r * OC + o] = s + b;
    }
  }
}

void orc_matmul_backward(float* dinp, float* dW, float* dbias, const float* dout, const float* inp, const float* W,
                         int BT, int C, int OC) {
  /* d_inputs += d_outputs * W^T  (matmul.cpp:67-68): row blocks reuse W rows */
  if (dinp) {
    const int RB = 16;
#pragma omp parallel for schedule(dynamic, 1)
    for (int r0 = 0; r0 < BT; r0 += RB) {
      const int r1 = r0 + RB < BT ? r0 + RB : BT;
      for (int o = 0; o < OC; ++o) {
        const float* w = W + (size_t)o * C;
        for (int r = r0; r < r1; ++r) {
          const float g = dout[(size_t)r * OC + o];
          float* d = dinp + (size_t)r * C;
          for (int c = 0; c < C; ++c) d[c] += g * w[c];
        }
      }
    }
  }
  /* d_weight += inputs^T * d_outputs (matmul.cpp:67), d_bias += colsum (matmul.cpp:51-55) */
#pragma omp parallel for schedule(static)
  for (int o = 0; o < OC; ++o) {
    float* dw = dW + (size_t)o * C;
    float bsum = 0.0f;
    for (int r = 0; r < BT; ++r) {
      const float g = dout[(size_t)r * OC + o];
      const float* x = inp + (size_t)r * C;
      bsum += g;
      for (int c = 0; c < C; ++c) dw[c] += g * x[c];
    }
    if (dbias) dbias[o] += bsum;
  }
}

/* ----------------------------------------------------------- attention */
void orc_attention_forward(float* out, float* att, float* lse, const float* qkv, int B, int T, int C, int NH) {
  const int hs = C / NH;
  const float scale = 1.0f / sqrtf((float)hs);
  const int C3 = 3 * C;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < NH; ++h) {
      float* A = att + ((size_t)b * NH + h) * T * T;
      for (int t = 0; t < T; ++t) {
        const float* q = qkv + ((size_t)b * T + t) * C3 + h * hs;
        float* row = A + (size_t)t * T;
        /* pre_att = q.k * scale for t1 <= t (attention.cpp:36) */
        float maxv = -INFINITY;
        for (int t1 = 0; t1 <= t; ++t1) {
          const float* k = qkv + ((size_t)b * T + t1) * C3 + C + h * hs;
          float s = 0.0f;
          for (int i = 0; i < hs; ++i) s += q[i] * k[i];
          s *= scale;
          row[t1] = s;
          if (s > maxv) maxv = s;
        }
        /* softmax over t1 <= t (attention.cpp:38-47) */
        float sum = 0.0f;
        for (int t1 = 0; t1 <= t; ++t1) {
          float e = expf(row[t1] - maxv);
          row[t1] = e;
          sum += e;
        }
        const float inv = sum == 0.0f ? 0.0f : 1.0f / sum;
        for (int t1 = 0; t1 <= t; ++t1) row[t1] *= inv;
        for (int t1 = t + 1; t1 < T; ++t1) row[t1] = 0.0f;
        if (lse) lse[((size_t)b * NH + h) * T + t] = maxv + logf(sum);
        /* out = att * v (attention.cpp:49) */
        float* o = out + ((size_t)b * T + t) * C + h * hs;
        for (int i = 0; i < hs; ++i) o[i] = 0.0f;
        for (int t1 = 0; t1 <= t; ++t1) {
          const float* v = qkv + ((size_t)b * T + t1) * C3 + 2 * C + h * hs;
          const float a = row[t1];
          for (int i = 0; i < hs; ++i) o[i] += a * v[i];
        }
      }
    }
  }
}

void orc_attention_backward(float* dqkv, const float* dout, const float* qkv, const float* att, int B, int T, int C,
                            int NH) {
  const int hs = C / NH;
  const float scale = 1.0f / sqrtf((float)hs);
  const int C3 = 3 * C;
#pragma omp parallel
  {
    float* dpre = (float*)malloc(sizeof(float) * (size_t)T);
#pragma omp for collapse(2) schedule(dynamic, 1)
    for (int b = 0; b < B; ++b) {
      for (int h = 0; h < NH; ++h) {
        const float* A = att + ((size_t)b * NH + h) * T * T;
        for (int t = 0; t < T; ++t) {
          const float* row = A + (size_t)t * T;
          const float* dO = dout + ((size_t)b * T + t) * C + h * hs;
          /* d_att(t,t1) = dO_t . v_t1 (attention.cpp:100) and the softmax
           * Jacobian sum over t1 (attention.cpp:104-113) */
          float dot = 0.0f;
          for (int t1 = 0; t1 <= t; ++t1) {
            const float* v = qkv + ((size_t)b * T + t1) * C3 + 2 * C + h * hs;
            float s = 0.0f;
            for (int i = 0; i < hs; ++i) s += dO[i] * v[i];
            dpre[t1] = s;
            dot += row[t1] * s;
          }
          for (int t1 = 0; t1 <= t; ++t1) dpre[t1] = row[t1] * (dpre[t1] - dot);
          /* dV, dK, dQ (attention.cpp:115-119) */
          const float* q = qkv + ((size_t)b * T + t) * C3 + h * hs;
          float* dq = dqkv + ((size_t)b * T + t) * C3 + h * hs;
          for (int t1 = 0; t1 <= t; ++t1) {
            const float* k = qkv + ((size_t)b * T + t1) * C3 + C + h * hs;
            float* dk = dqkv + ((size_t)b * T + t1) * C3 + C + h * hs;
            float* dv = dqkv + ((size_t)b * T + t1) * C3 + 2 * C + h * hs;
            const float a = row[t1];
            const float g = dpre[t1] * scale;
            for (int i = 0; i < hs; ++i) {
              dv[i] += a * dO[i];
              dk[i] += g * q[i];
              dq[i] += g * k[i];
            }
          }
        }
      }
    }
    free(dpre);
  }
}

/* ----------------------------------------------------------- layernorm */
void orc_layernorm_forward(float* out, float* mean, float* rstd, const float* inp, const float* gamma,
                           const float* beta, int N, int C) {
  const float eps = 1e-5f;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; ++r) {
    const float* x = inp + (size_t)r * C;
    float m = 0.0f;
    for (int c = 0; c < C; ++c) m += x[c];
    m /= (float)C;
    float v = 0.0f;
    for (int c = 0; c < C; ++c) {
      float d = x[c] - m;
      v += d * d;
    }
    v /= (float)C;
    const float s = 1.0f / sqrtf(v + eps);
    float* y = out + (size_t)r * C;
    for (int c = 0; c < C; ++c) y[c] = (x[c] - m) * gamma[c] * s + beta[c];
    if (mean) mean[r] = m;
    if (rstd) rstd[r] = s;
  }
}

void orc_layernorm_backward(float* dinp, float* dgamma, float* dbeta, const float* dout, const float* inp,
                            const float* gamma, const float* mean, const float* rstd, int N, int C) {
  /* d_gamma += sum dy * xhat; d_beta += sum dy (layernorm.cpp:49-52) */
#pragma omp parallel for schedule(static)
  for (int c = 0; c < C; ++c) {
    float g = 0.0f, bsum = 0.0f;
    for (int r = 0; r < N; ++r) {
      const float dy = dout[(size_t)r * C + c];
      g += dy * (inp[(size_t)r * C + c] - mean[r]) * rstd[r];
      bsum += dy;
    }
    dgamma[c] += g;
    dbeta[c] += bsum;
  }
  /* dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)) (layernorm.cpp:66-69) */
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; ++r) {
    const float* dy = dout + (size_t)r * C;
    const float* x = inp + (size_t)r * C;
    float s1 = 0.0f, s2 = 0.0f;
    for (int c = 0; c < C; ++c) {
      const float gdy = gamma[c] * dy[c];
      s1 += gdy;
      s2 += gdy * (x[c] - mean[r]) * rstd[r];
    }
    s1 /= (float)C;
    s2 /= (float)C;
    float* dx = dinp + (size_t)r * C;
    for (int c = 0; c < C; ++c) {
      const float xhat = (x[c] - mean[r]) * rstd[r];
      dx[c] = rstd[r] * ((gamma[c] * dy[c] - xhat * s2) - s1);
    }
  }
}

/* -------------------------------------------------------- elementwise */
static const float kGeluC1 = 0.7978845608f; /* sqrt(2/pi), gelu.h:7 */
static const float kGeluC2 = 0.044715f;     /* gelu.h:8 */

void orc_gelu_forward(float* out, const float* inp, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) {
    const float x = inp[i];
    out[i] = 0.5f * x * (1.0f + tanhf(kGeluC1 * (x + kGeluC2 * x * x * x)));
  }
}

void orc_gelu_backward(float* dinp, const float* dout, const float* inp, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) {
    const float x = inp[i];
    const float u = kGeluC1 * (x + kGeluC2 * x * x * x);
    const float th = tanhf(u);
    const float ch = coshf(u);
    const float sech2 = 1.0f / (ch * ch);
    const float g = 0.5f * (1.0f + th) + x * 0.5f * sech2 * kGeluC1 * (1.0f + 3.0f * kGeluC2 * x * x);
    dinp[i] = g * dout[i];
  }
}

void orc_residual_forward(float* out, const float* a, const float* b, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

void orc_softmax(float* probs, const float* logits, int BT, int V, int ld) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < BT; ++r) {
    const float* x = logits + (size_t)r * ld;
    float* p = probs + (size_t)r * V;
    float m = -INFINITY;
    for (int c = 0; c < V; ++c) m = x[c] > m ? x[c] : m;
    float s = 0.0f;
    for (int c = 0; c < V; ++c) {
      p[c] = expf(x[c] - m);
      s += p[c];
    }
    const float inv = s == 0.0f ? 0.0f : 1.0f / s;
    for (int c = 0; c < V; ++c) p[c] *= inv;
  }
}

float orc_cross_entropy(float* losses, const float* probs, const int* targets, int BT, int V) {
  float mean = 0.0f;
  for (int r = 0; r < BT; ++r) {
    const float l = -logf(probs[(size_t)r * V + targets[r]]);
    if (losses) losses[r] = l;
    mean += l;
  }
  return mean / (float)BT;
}

void orc_cross_entropy_softmax_backward(float* dlogits, const float* probs, const int* targets, int BT, int V,
                                        int ld) {
  const float inv = 1.0f / (float)BT;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < BT; ++r) {
    float* d = dlogits + (size_t)r * ld;
    const float* p = probs + (size_t)r * V;
    for (int c = 0; c < V; ++c) d[c] = (d[c] + p[c] - (targets[r] == c ? 1.0f : 0.0f)) * inv;
  }
}

void orc_encoder_forward(float* out, const int* tokens, const float* wte, const float* wpe, int B, int T, int C) {
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) {
      const float* e = wte + (size_t)tokens[b * T + t] * C;
      const float* p = wpe + (size_t)t * C;
      float* o = out + ((size_t)b * T + t) * C;
      for (int c = 0; c < C; ++c) o[c] = e[c] + p[c];
    }
}

void orc_encoder_backward(float* dwte, float* dwpe, const float* dout, const int* tokens, int B, int T, int C) {
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t) {
      const float* d = dout + ((size_t)b * T + t) * C;
      float* we = dwte + (size_t)tokens[b * T + t] * C;
      float* wp = dwpe + (size_t)t * C;
      for (int c = 0; c < C; ++c) {
        wp[c] += d[c];
        we[c] += d[c];
      }
    }
}

void orc_adamw(float* p, const float* g, float* m, float* v, size_t n, float lr, float beta1, float beta2, float eps,
               float weight_decay, int t) {
  /* bias corrections as the reference evaluates them: std::pow(float,int) is double */
  const double c1 = 1.0 - pow((double)beta1, t);
  const double c2 = 1.0 - pow((double)beta2, t);
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) {
    const float param = p[i], grad = g[i];
    const float m_ = beta1 * m[i] + (1.0f - beta1) * grad;
    const float v_ = beta2 * v[i] + (1.0f - beta2) * grad * grad;
    const float mh = (float)(m_ / c1);
    const float vh = (float)(v_ / c2);
    m[i] = m_;
    v[i] = v_;
    p[i] -= lr * (mh / (sqrtf(vh) + eps) + weight_decay * param);
  }
}

/* --------------------------------------------------------------- model */
size_t orc_gpt2_param_sizes(const orc_config* cfg, size_t sizes[16]) {
  const size_t Vp = cfg->padded_vocab_size, C = cfg->channels, L = cfg->num_layers, maxT = cfg->max_seq_len;
  sizes[0] = Vp * C;
  sizes[1] = maxT * C;
  sizes[2] = L * C;
  sizes[3] = L * C;
  sizes[4] = L * 3 * C * C;
  sizes[5] = L * 3 * C;
  sizes[6] = L * C * C;
  sizes[7] = L * C;
  sizes[8] = L * C;
  sizes[9] = L * C;
  sizes[10] = L * 4 * C * C;
  sizes[11] = L * 4 * C;
  sizes[12] = L * 4 * C * C;
  sizes[13] = L * C;
  sizes[14] = C;
  sizes[15] = C;
  size_t n = 0;
  for (int i = 0; i < 16; ++i) n += sizes[i];
  return n;
}

void orc_gpt2_init_params(float* params, const orc_config* cfg, uint64_t seed) {
  size_t sz[16];
  const size_t n = orc_gpt2_param_sizes(cfg, sz);
  memset(params, 0, n * sizeof(float));
  orc_rng r;
  orc_rng_seed(&r, seed, 0);
  const double two_pi = 6.283185307179586476925286766559;
  const float resid_scale = 1.0f / sqrtf(2.0f * (float)cfg->num_layers);
  float* p = params;
  for (int i = 0; i < 16; ++i) {
    const int is_weight = (i == 0 || i == 1 || i == 4 || i == 6 || i == 10 || i == 12);
    const int is_gamma = (i == 2 || i == 8 || i == 14);
    if (is_weight) {
      const double sd = 0.02 * ((i == 6 || i == 12) ? (double)resid_scale : 1.0);
      for (size_t j = 0; j < sz[i]; ++j) {
        double u1 = orc_rng_uniform(&r), u2 = orc_rng_uniform(&r);
        p[j] = (float)(sqrt(-2.0 * log(u1)) * cos(two_pi * u2) * sd);
      }
      if (i == 0) /* padded vocabulary rows are zero */
        memset(p + (size_t)cfg->vocab_size * cfg->channels, 0,
               sizeof(float) * (size_t)(cfg->padded_vocab_size - cfg->vocab_size) * cfg->channels);
    } else if (is_gamma) {
      for (size_t j = 0; j < sz[i]; ++j) p[j] = 1.0f;
    }
    p += sz[i];
  }
}

struct orc_gpt2 {
  orc_config cfg;
  int B, T;
  size_t sizes[16], n;
  float *params, *grads, *m, *v;
  float* P[16]; /* tensor views into params */
  float* G[16]; /* and grads */
  int *inputs, *targets;
  /* activations (per layer where marked L) */
  float *encoded, *ln1, *ln1_mean, *ln1_rstd, *qkv, *atty, *att, *lse, *attproj, *res2, *ln2, *ln2_mean, *ln2_rstd,
      *fch, *fch_gelu, *fcproj, *res3, *lnf, *lnf_mean, *lnf_rstd, *logits, *probs, *losses;
  float mean_loss;
};

static float* zalloc(size_t n) { return (float*)calloc(n ? n : 1, sizeof(float)); }

orc_gpt2* orc_gpt2_create(const orc_config* cfg, const float* params, int B, int T) {
  orc_gpt2* m = (orc_gpt2*)calloc(1, sizeof(orc_gpt2));
  m->cfg = *cfg;
  m->B = B;
  m->T = T;
  m->n = orc_gpt2_param_sizes(cfg, m->sizes);
  m->params = zalloc(m->n);
  m->grads = zalloc(m->n);
  m->m = zalloc(m->n);
  m->v = zalloc(m->n);
  memcpy(m->params, params, m->n * sizeof(float));
  size_t off = 0;
  for (int i = 0; i < 16; ++i) {
    m->P[i] = m->params + off;
    m->G[i] = m->grads + off;
    off += m->sizes[i];
  }
  const size_t L = cfg->num_layers, C = cfg->channels, NH = cfg->num_heads, BT = (size_t)B * T, Vp = cfg->padded_vocab_size,
               V = cfg->vocab_size;
  m->inputs = (int*)calloc(BT, sizeof(int));
  m->targets = (int*)calloc(BT, sizeof(int));
  m->encoded = zalloc(BT * C);
  m->ln1 = zalloc(L * BT * C);
  m->ln1_mean = zalloc(L * BT);
  m->ln1_rstd = zalloc(L * BT);
  m->qkv = zalloc(L * BT * 3 * C);
  m->atty = zalloc(L * BT * C);
  m->att = zalloc(L * B * NH * (size_t)T * T);
  m->lse = zalloc(L * B * NH * (size_t)T);
  m->attproj = zalloc(L * BT * C);
  m->res2 = zalloc(L * BT * C);
  m->ln2 = zalloc(L * BT * C);
  m->ln2_mean = zalloc(L * BT);
  m->ln2_rstd = zalloc(L * BT);
  m->fch = zalloc(L * BT * 4 * C);
  m->fch_gelu = zalloc(L * BT * 4 * C);
  m->fcproj = zalloc(L * BT * C);
  m->res3 = zalloc(L * BT * C);
  m->lnf = zalloc(BT * C);
  m->lnf_mean = zalloc(BT);
  m->lnf_rstd = zalloc(BT);
  m->logits = zalloc(BT * Vp);
  m->probs = zalloc(BT * V);
  m->losses = zalloc(BT);
  return m;
}

void orc_gpt2_free(orc_gpt2* m) {
  if (!m) return;
  float* bufs[] = {m->params, m->grads, m->m, m->v, m->encoded, m->ln1, m->ln1_mean, m->ln1_rstd, m->qkv, m->atty,
                   m->att, m->lse, m->attproj, m->res2, m->ln2, m->ln2_mean, m->ln2_rstd, m->fch, m->fch_gelu,
                   m->fcproj, m->res3, m->lnf, m->lnf_mean, m->lnf_rstd, m->logits, m->probs, m->losses};
  for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); ++i) free(bufs[i]);
  free(m->inputs);
  free(m->targets);
  free(m);
}

float orc_gpt2_forward(orc_gpt2* m, const int* inputs, const int* targets) {
  const int B = m->B, T = m->T, C = m->cfg.channels, NH = m->cfg.num_heads, L = m->cfg.num_layers;
  const int V = m->cfg.vocab_size, Vp = m->cfg.padded_vocab_size;
  const size_t BT = (size_t)B * T;
  memcpy(m->inputs, inputs, BT * sizeof(int));
  if (targets) memcpy(m->targets, targets, BT * sizeof(int));
  orc_encoder_forward(m->encoded, inputs, m->P[0], m->P[1], B, T, C);
  const float* residual = m->encoded;
  for (int l = 0; l < L; ++l) {
    /* Layer::Forward, gpt2/layer.cpp:35-80 */
    float* ln1 = m->ln1 + l * BT * C;
    float* qkv = m->qkv + l * BT * 3 * C;
    float* atty = m->atty + l * BT * C;
    float* att = m->att + (size_t)l * B * NH * T * T;
    float* attproj = m->attproj + l * BT * C;
    float* res2 = m->res2 + l * BT * C;
    float* ln2 = m->ln2 + l * BT * C;
    float* fch = m->fch + l * BT * 4 * C;
    float* gelu = m->fch_gelu + l * BT * 4 * C;
    float* fcproj = m->fcproj + l * BT * C;
    float* res3 = m->res3 + l * BT * C;
    orc_layernorm_forward(ln1, m->ln1_mean + l * BT, m->ln1_rstd + l * BT, residual, m->P[2] + l * C,
                          m->P[3] + l * C, (int)BT, C);
    orc_matmul_forward(qkv, ln1, m->P[4] + (size_t)l * 3 * C * C, m->P[5] + l * 3 * C, (int)BT, C, 3 * C);
    orc_attention_forward(atty, att, m->lse + (size_t)l * B * NH * T, qkv, B, T, C, NH);
    orc_matmul_forward(attproj, atty, m->P[6] + (size_t)l * C * C, m->P[7] + l * C, (int)BT, C, C);
    orc_residual_forward(res2, residual, attproj, BT * C);
    orc_layernorm_forward(ln2, m->ln2_mean + l * BT, m->ln2_rstd + l * BT, res2, m->P[8] + l * C, m->P[9] + l * C,
                          (int)BT, C);
    orc_matmul_forward(fch, ln2, m->P[10] + (size_t)l * 4 * C * C, m->P[11] + l * 4 * C, (int)BT, C, 4 * C);
    orc_gelu_forward(gelu, fch, BT * 4 * C);
    orc_matmul_forward(fcproj, gelu, m->P[12] + (size_t)l * 4 * C * C, m->P[13] + l * C, (int)BT, 4 * C, C);
    orc_residual_forward(res3, res2, fcproj, BT * C);
    residual = res3;
  }
  orc_layernorm_forward(m->lnf, m->lnf_mean, m->lnf_rstd, residual, m->P[14], m->P[15], (int)BT, C);
  orc_matmul_forward(m->logits, m->lnf, m->P[0], NULL, (int)BT, C, Vp); /* tied lm_head, gpt2.cpp:259 */
  orc_softmax(m->probs, m->logits, (int)BT, V, Vp);
  m->mean_loss = targets ? orc_cross_entropy(m->losses, m->probs, targets, (int)BT, V) : -1.0f;
  return m->mean_loss;
}

void orc_gpt2_zero_grad(orc_gpt2* m) { memset(m->grads, 0, m->n * sizeof(float)); }

void orc_gpt2_backward(orc_gpt2* m) {
  const int B = m->B, T = m->T, C = m->cfg.channels, NH = m->cfg.num_heads, L = m->cfg.num_layers;
  const int V = m->cfg.vocab_size, Vp = m->cfg.padded_vocab_size;
  const size_t BT = (size_t)B * T;
  float* dlogits = zalloc(BT * Vp);
  float* dlnf = zalloc(BT * C);
  float* dres = zalloc(BT * C);     /* gradient flowing into the current layer's output */
  float* dres_in = zalloc(BT * C);  /* gradient of the current layer's input */
  float* dbt4c_a = zalloc(BT * 4 * C);
  float* dbt4c_b = zalloc(BT * 4 * C);
  float* dln = zalloc(BT * C);
  float* datty = zalloc(BT * C);
  float* dqkv = zalloc(BT * 3 * C);
  float* dtmp = zalloc(BT * C);
  /* gpt2.cpp:283-300 */
  orc_cross_entropy_softmax_backward(dlogits, m->probs, m->targets, (int)BT, V, Vp);
  orc_matmul_backward(dlnf, m->G[0], NULL, dlogits, m->lnf, m->P[0], (int)BT, C, Vp); /* padded dlogits columns are 0 */
  const float* res_last = L > 0 ? m->res3 + (size_t)(L - 1) * BT * C : m->encoded;
  orc_layernorm_backward(dres, m->G[14], m->G[15], dlnf, res_last, m->P[14], m->lnf_mean, m->lnf_rstd, (int)BT, C);
  for (int l = L - 1; l >= 0; --l) {
    /* Layer::Backward, gpt2/layer.cpp:82-142; dres = d(res3) */
    const float* residual = l > 0 ? m->res3 + (size_t)(l - 1) * BT * C : m->encoded;
    const float* ln1 = m->ln1 + l * BT * C;
    const float* qkv = m->qkv + l * BT * 3 * C;
    const float* atty = m->atty + l * BT * C;
    const float* att = m->att + (size_t)l * B * NH * T * T;
    const float* res2 = m->res2 + l * BT * C;
    const float* ln2 = m->ln2 + l * BT * C;
    const float* fch = m->fch + l * BT * 4 * C;
    const float* gelu = m->fch_gelu + l * BT * 4 * C;
    /* dl_residual2 = dres; dl_fcproj = dres */
    memset(dbt4c_a, 0, BT * 4 * C * sizeof(float));
    orc_matmul_backward(dbt4c_a, m->G[12] + (size_t)l * 4 * C * C, m->G[13] + l * C, dres, gelu,
                        m->P[12] + (size_t)l * 4 * C * C, (int)BT, 4 * C, C);
    orc_gelu_backward(dbt4c_b, dbt4c_a, fch, BT * 4 * C);
    memset(dln, 0, BT * C * sizeof(float));
    orc_matmul_backward(dln, m->G[10] + (size_t)l * 4 * C * C, m->G[11] + l * 4 * C, dbt4c_b, ln2,
                        m->P[10] + (size_t)l * 4 * C * C, (int)BT, C, 4 * C);
    orc_layernorm_backward(dtmp, m->G[8] + l * C, m->G[9] + l * C, dln, res2, m->P[8] + l * C, m->ln2_mean + l * BT,
                           m->ln2_rstd + l * BT, (int)BT, C);
    for (size_t i = 0; i < BT * C; ++i) dres[i] += dtmp[i]; /* dl_residual2 */
    memset(datty, 0, BT * C * sizeof(float));
    orc_matmul_backward(datty, m->G[6] + (size_t)l * C * C, m->G[7] + l * C, dres, atty, m->P[6] + (size_t)l * C * C,
                        (int)BT, C, C);
    memset(dqkv, 0, BT * 3 * C * sizeof(float));
    orc_attention_backward(dqkv, datty, qkv, att, B, T, C, NH);
    memset(dln, 0, BT * C * sizeof(float));
    orc_matmul_backward(dln, m->G[4] + (size_t)l * 3 * C * C, m->G[5] + l * 3 * C, dqkv, ln1,
                        m->P[4] + (size_t)l * 3 * C * C, (int)BT, C, 3 * C);
    orc_layernorm_backward(dtmp, m->G[2] + l * C, m->G[3] + l * C, dln, residual, m->P[2] + l * C,
                           m->ln1_mean + l * BT, m->ln1_rstd + l * BT, (int)BT, C);
    for (size_t i = 0; i < BT * C; ++i) dres_in[i] = dres[i] + dtmp[i];
    float* t = dres;
    dres = dres_in;
    dres_in = t;
  }
  orc_encoder_backward(m->G[0], m->G[1], dres, m->inputs, B, T, C); /* gpt2.cpp:313 */
  free(dlogits);
  free(dlnf);
  free(dres);
  free(dres_in);
  free(dbt4c_a);
  free(dbt4c_b);
  free(dln);
  free(datty);
  free(dqkv);
  free(dtmp);
}

void orc_gpt2_update(orc_gpt2* m, float lr, float b1, float b2, float eps, float wd, int t) {
  orc_adamw(m->params, m->grads, m->m, m->v, m->n, lr, b1, b2, eps, wd, t);
}

float* orc_gpt2_params(orc_gpt2* m) { return m->params; }
float* orc_gpt2_grads(orc_gpt2* m) { return m->grads; }
size_t orc_gpt2_num_params(orc_gpt2* m) { return m->n; }

const float* orc_gpt2_activation(orc_gpt2* m, const char* name) {
  if (!strcmp(name, "logits")) return m->logits;
  if (!strcmp(name, "lnf")) return m->lnf;
  if (!strcmp(name, "encoded")) return m->encoded;
  if (!strcmp(name, "probs")) return m->probs;
  return NULL;
}
