/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for wkvm_b200's parity tests and
 * bench.py's CPU baseline. Nothing in the product (wkvm_b200/) links, loads
 * or calls this file.
 *
 * A plain-C fp32 restatement of the recurrences wkvm runs through the
 * third-party package flash-linear-attention (fla) 0.5.1, which is not
 * vendored in the wkvm tree (wkvm/models/rwkv7.py:113 loads fla's RWKV-7
 * model; wkvm/runner/state.py:70 seeds fla's Cache). Its algorithm is pinned
 * against golden vectors produced by fla's own torch reference functions
 * (tests/golden/make_golden.py) in tests/test_oracle.py.
 *
 * Semantics followed, token by token, per (sequence, head):
 *
 * oracle_dplr  — fla/ops/rwkv7/fused_recurrent.py:94-100 (decode) and
 *   :103-118 (T loop); same update as fla/ops/generalized_delta_rule/dplr/
 *   naive.py:34-36 (dplr_recurrence) without its forced q * K^-0.5 (:23):
 *     sa[v] = sum_k a[k] h[k][v]           (state before this token)
 *     h[k][v] = exp(w[k]) h[k][v] + b[k] sa[v]
 *     h[k][v] += k[k] v[v]
 *     o[v] = sum_k h[k][v] (r[k] scale)
 *   RWKV-7 (fla/layers/rwkv7.py:308-334) uses a = -kk, b = kk * a_gate, scale 1.
 *
 * oracle_gdn   — fla/ops/gated_delta_rule/fused_recurrent.py:104-151 and
 *   fla/ops/gated_delta_rule/naive.py:44-56:
 *     (optional) q /= sqrt(sum q^2 + 1e-6), k /= sqrt(sum k^2 + 1e-6)
 *     h *= exp(g) ; v' = beta (v - sum_k h[k][v] k[k]) ; h += k v'^T
 *     o[v] = sum_k h[k][v] (q[k] scale)
 *
 * Layouts: activations [tokens, H, D] (token = bos + t), states [N, H, K, V]
 * updated in place. cu_seqlens (may be NULL) gives varlen sequence bounds.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void seq_bounds(const int64_t* cu, int n, int T, int64_t* bos, int64_t* len) {
  if (cu) {
    *bos = cu[n];
    *len = cu[n + 1] - cu[n];
  } else {
    *bos = (int64_t)n * T;
    *len = T;
  }
}

/* Work items (sequence, head) are handed out from a shared counter to
 * `threads` pthreads; each item touches only its own state and outputs. */
typedef struct {
  const float *r, *w, *k, *v, *a, *b;
  float *o, *h;
  const int64_t* cu;
  int N, T, H, HV, K, V, l2norm;
  float scale;
  int next;
  pthread_mutex_t mu;
} Job;

static int take(Job* j) {
  pthread_mutex_lock(&j->mu);
  int x = j->next++;
  pthread_mutex_unlock(&j->mu);
  return x;
}

static void run_pool(Job* j, void* (*fn)(void*), int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  pthread_mutex_init(&j->mu, NULL);
  j->next = 0;
  for (int i = 1; i < threads; ++i) pthread_create(&tid[i], NULL, fn, j);
  fn(j);
  for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
  pthread_mutex_destroy(&j->mu);
}

static void* dplr_worker(void* arg) {
  Job* J = (Job*)arg;
  const float *r = J->r, *w = J->w, *k = J->k, *v = J->v, *a = J->a, *b = J->b;
  float *o = J->o, *h = J->h;
  const int64_t* cu = J->cu;
  const int N = J->N, T = J->T, H = J->H, K = J->K, V = J->V;
  const float scale = J->scale;
  for (int nh = take(J); nh < N * H; nh = take(J)) {
    const int n = nh / H, hh = nh % H;
    int64_t bos, len;
    seq_bounds(cu, n, T, &bos, &len);
    float* S = h + (int64_t)nh * K * V;
    float* sa = (float*)malloc(sizeof(float) * V);
    for (int64_t t = 0; t < len; ++t) {
      const int64_t bk = ((bos + t) * H + hh) * K;
      const int64_t bv = ((bos + t) * H + hh) * V;
      for (int j = 0; j < V; ++j) sa[j] = 0.f;
      for (int i = 0; i < K; ++i) {
        const float ai = a[bk + i];
        for (int j = 0; j < V; ++j) sa[j] += ai * S[i * V + j];
      }
      for (int i = 0; i < K; ++i) {
        const float ew = expf(w[bk + i]);
        const float bi = b[bk + i];
        const float ki = k[bk + i];
        for (int j = 0; j < V; ++j) {
          float x = ew * S[i * V + j] + bi * sa[j];
          S[i * V + j] = x + ki * v[bv + j];
        }
      }
      for (int j = 0; j < V; ++j) sa[j] = 0.f;
      for (int i = 0; i < K; ++i) {
        const float ri = r[bk + i] * scale;
        for (int j = 0; j < V; ++j) sa[j] += S[i * V + j] * ri;
      }
      memcpy(o + bv, sa, sizeof(float) * V);
    }
    free(sa);
  }
  return NULL;
}

int oracle_dplr(const float* r, const float* w, const float* k, const float* v,
                const float* a, const float* b, float* o, float* h, const int64_t* cu,
                int N, int T, int H, int K, int V, float scale, int threads) {
  Job j = {r, w, k, v, a, b, o, h, cu, N, T, H, H, K, V, 0, scale, 0};
  run_pool(&j, dplr_worker, threads);
  return 0;
}

static void* gdn_worker(void* arg) {
  Job* J = (Job*)arg;
  const float *q = J->r, *k = J->k, *v = J->v, *g = J->w, *beta = J->a;
  float *o = J->o, *h = J->h;
  const int64_t* cu = J->cu;
  const int N = J->N, T = J->T, H = J->H, HV = J->HV, K = J->K, V = J->V, l2norm = J->l2norm;
  const float scale = J->scale;
  for (int nh = take(J); nh < N * HV; nh = take(J)) {
    const int n = nh / HV, hv = nh % HV, hq = hv / (HV / H);
    int64_t bos, len;
    seq_bounds(cu, n, T, &bos, &len);
    float* S = h + (int64_t)nh * K * V;
    float* qs = (float*)malloc(sizeof(float) * K);
    float* ks = (float*)malloc(sizeof(float) * K);
    float* vn = (float*)malloc(sizeof(float) * V);
    for (int64_t t = 0; t < len; ++t) {
      const int64_t tok = bos + t;
      const int64_t bq = (tok * H + hq) * K;
      const int64_t bv = (tok * HV + hv) * V;
      float nq = 1.f, nk = 1.f;
      if (l2norm) {
        float sq = 0.f, sk = 0.f;
        for (int i = 0; i < K; ++i) {
          sq += q[bq + i] * q[bq + i];
          sk += k[bq + i] * k[bq + i];
        }
        nq = sqrtf(sq + 1e-6f);
        nk = sqrtf(sk + 1e-6f);
      }
      for (int i = 0; i < K; ++i) {
        qs[i] = q[bq + i] / nq * scale;
        ks[i] = k[bq + i] / nk;
      }
      const float eg = expf(g[tok * HV + hv]);
      const float bt = beta[tok * HV + hv];
      for (int64_t e = 0; e < (int64_t)K * V; ++e) S[e] *= eg;
      for (int j = 0; j < V; ++j) vn[j] = 0.f;
      for (int i = 0; i < K; ++i)
        for (int j = 0; j < V; ++j) vn[j] += S[i * V + j] * ks[i];
      for (int j = 0; j < V; ++j) vn[j] = bt * (v[bv + j] - vn[j]);
      for (int i = 0; i < K; ++i)
        for (int j = 0; j < V; ++j) S[i * V + j] += ks[i] * vn[j];
      for (int j = 0; j < V; ++j) vn[j] = 0.f;
      for (int i = 0; i < K; ++i)
        for (int j = 0; j < V; ++j) vn[j] += S[i * V + j] * qs[i];
      memcpy(o + bv, vn, sizeof(float) * V);
    }
    free(qs);
    free(ks);
    free(vn);
  }
  return NULL;
}

int oracle_gdn(const float* q, const float* k, const float* v, const float* g,
               const float* beta, float* o, float* h, const int64_t* cu, int N, int T,
               int H, int HV, int K, int V, float scale, int l2norm, int threads) {
  Job j = {q, g, k, v, beta, NULL, o, h, cu, N, T, H, HV, K, V, l2norm, scale, 0};
  run_pool(&j, gdn_worker, threads);
  return 0;
}
