/* attn_ref_f64.c -- fp64 CPU oracle for attention forward and backward.
 * TEST INFRASTRUCTURE ONLY: loaded by tests/ (and nothing in the product).
 *
 * Restates, in plain C with a GQA head mapping added:
 *   oracle_fwd_f64  -- attention_ref_f64  (reference attention.cu:72-102),
 *                      plus the row log-sum-exp the kernels emit
 *                      (flash_fwd.cuh:321-330: lse = m + ln(l));
 *   oracle_bwd_f64  -- bwd_ref_f64        (reference bwd.cu:20-69);
 *   oracle_loss_f64 -- loss_f64 = sum(dO o O) with one input entry perturbed
 *                      (reference bwd.cu:73-105), for finite differences.
 * Layout: q, dO, o, dq (B, Hq, N, D); k, v, dk, dv (B, Hkv, N, D); lse (B, Hq, N);
 * all row-major doubles. Query head h reads kv head h / (Hq / Hkv).
 * Scale is 1/sqrt(D); causal means key j is visible to query i iff j <= i.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

static const double* head(const double* base, int b, int h, int H, int N, int D) {
  return base + ((size_t)b * H + h) * (size_t)N * D;
}

/* Probabilities of query row i of one head into p[0..lim); returns lim. */
static int row_probs(const double* qh, const double* kh, int i, int N, int D, int causal,
                     double scale, double* p, double* lse_out) {
  const int lim = causal ? i + 1 : N;
  double mx = -INFINITY;
  for (int j = 0; j < lim; ++j) {
    double acc = 0.0;
    for (int d = 0; d < D; ++d) acc += qh[(size_t)i * D + d] * kh[(size_t)j * D + d];
    p[j] = acc * scale;
    if (p[j] > mx) mx = p[j];
  }
  double sum = 0.0;
  for (int j = 0; j < lim; ++j) {
    p[j] = exp(p[j] - mx);
    sum += p[j];
  }
  for (int j = 0; j < lim; ++j) p[j] /= sum;
  if (lse_out) *lse_out = mx + log(sum);
  return lim;
}

void oracle_fwd_f64(const double* q, const double* k, const double* v, double* o, double* lse,
                    int B, int Hq, int Hkv, int N, int D, int causal) {
  const int G = Hq / Hkv;
  const double scale = 1.0 / sqrt((double)D);
  double* p = (double*)malloc(sizeof(double) * (size_t)N);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const double* qh = head(q, b, h, Hq, N, D);
      const double* kh = head(k, b, h / G, Hkv, N, D);
      const double* vh = head(v, b, h / G, Hkv, N, D);
      double* oh = o + ((size_t)b * Hq + h) * (size_t)N * D;
      for (int i = 0; i < N; ++i) {
        double l;
        const int lim = row_probs(qh, kh, i, N, D, causal, scale, p, &l);
        if (lse) lse[((size_t)b * Hq + h) * N + i] = l;
        for (int d = 0; d < D; ++d) {
          double acc = 0.0;
          for (int j = 0; j < lim; ++j) acc += p[j] * vh[(size_t)j * D + d];
          oh[(size_t)i * D + d] = acc;
        }
      }
    }
  free(p);
}

void oracle_bwd_f64(const double* q, const double* k, const double* v, const double* dO,
                    double* dq, double* dk, double* dv, int B, int Hq, int Hkv, int N, int D,
                    int causal) {
  const int G = Hq / Hkv;
  const double scale = 1.0 / sqrt((double)D);
  memset(dq, 0, sizeof(double) * (size_t)B * Hq * N * D);
  memset(dk, 0, sizeof(double) * (size_t)B * Hkv * N * D);
  memset(dv, 0, sizeof(double) * (size_t)B * Hkv * N * D);
  double* p = (double*)malloc(sizeof(double) * (size_t)N);
  double* orow = (double*)malloc(sizeof(double) * (size_t)D);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const double* qh = head(q, b, h, Hq, N, D);
      const double* gh = head(dO, b, h, Hq, N, D);
      const double* kh = head(k, b, h / G, Hkv, N, D);
      const double* vh = head(v, b, h / G, Hkv, N, D);
      double* dqh = dq + ((size_t)b * Hq + h) * (size_t)N * D;
      double* dkh = dk + ((size_t)b * Hkv + h / G) * (size_t)N * D;
      double* dvh = dv + ((size_t)b * Hkv + h / G) * (size_t)N * D;
      for (int i = 0; i < N; ++i) {
        const int lim = row_probs(qh, kh, i, N, D, causal, scale, p, NULL);
        double dvec = 0.0;
        for (int d = 0; d < D; ++d) {
          double acc = 0.0;
          for (int j = 0; j < lim; ++j) acc += p[j] * vh[(size_t)j * D + d];
          orow[d] = acc;
          dvec += gh[(size_t)i * D + d] * acc;
        }
        for (int j = 0; j < lim; ++j) {
          double dp = 0.0;
          for (int d = 0; d < D; ++d) dp += gh[(size_t)i * D + d] * vh[(size_t)j * D + d];
          const double ds = p[j] * (dp - dvec);
          for (int d = 0; d < D; ++d) {
            dvh[(size_t)j * D + d] += p[j] * gh[(size_t)i * D + d];
            dqh[(size_t)i * D + d] += ds * scale * kh[(size_t)j * D + d];
            dkh[(size_t)j * D + d] += ds * scale * qh[(size_t)i * D + d];
          }
        }
      }
    }
  free(orow);
  free(p);
}

/* sum(dO o O) with input `which` (0 q, 1 k, 2 v) entry `idx` moved by `pert`. */
double oracle_loss_f64(const double* q, const double* k, const double* v, const double* dO,
                       int B, int Hq, int Hkv, int N, int D, int causal, int which, size_t idx,
                       double pert) {
  const size_t nq = (size_t)B * Hq * N * D, nk = (size_t)B * Hkv * N * D;
  double* qc = (double*)malloc(sizeof(double) * nq);
  double* kc = (double*)malloc(sizeof(double) * nk);
  double* vc = (double*)malloc(sizeof(double) * nk);
  double* o = (double*)malloc(sizeof(double) * nq);
  memcpy(qc, q, sizeof(double) * nq);
  memcpy(kc, k, sizeof(double) * nk);
  memcpy(vc, v, sizeof(double) * nk);
  if (which == 0) qc[idx] += pert;
  if (which == 1) kc[idx] += pert;
  if (which == 2) vc[idx] += pert;
  oracle_fwd_f64(qc, kc, vc, o, NULL, B, Hq, Hkv, N, D, causal);
  double loss = 0.0;
  for (size_t i = 0; i < nq; ++i) loss += o[i] * dO[i];
  free(qc);
  free(kc);
  free(vc);
  free(o);
  return loss;
}
