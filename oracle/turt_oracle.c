/*
 * turt_oracle.c -- CPU restatement of turt's reference autodiff GPT training step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA library
 * (turt_b200/csrc) and the timed CPU baseline ("port" of the reference's CPU
 * data-parallel worker pool).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product path
 * never calls into it.
 *
 * What it restates (reference paths are relative to the turt project root):
 *   - src/math/random.ts:8-25        mulberry32 + Box-Muller gaussian
 *   - src/math/tensor.ts:83-88       Tensor.randn (f32 storage of gaussian*std)
 *   - src/math/tensor.ts:180-293     binary/unary element-wise ops and their closures
 *   - src/math/tensor.ts:301-347     sum / mean along the last axis
 *   - src/math/tensor.ts:352-394     matmul (i-k-j forward with f32 accumulation,
 *                                    backward dot products accumulated in double)
 *   - src/math/tensor.ts:397-454     transpose / reshape / permute
 *   - src/math/tensor.ts:457-514     bmm
 *   - src/math/tensor.ts:520-539     gatherRows (+ scatter-add backward)
 *   - src/math/tensor.ts:542-604     softmax, maskedFillCausal(-1e9)
 *   - src/math/tensor.ts:607-700     gelu (tanh approx), silu, rope (interleaved pairs)
 *   - src/math/tensor.ts:708-745     crossEntropyLogits
 *   - src/nn/rmsnorm.ts:24-27, src/nn/layernorm.ts:20-26  composite norms
 *   - src/models/gpt.ts:69-283       mlpHidden, attention, MLPs, Block, GPT init order + tied head
 *   - src/optim/adam.ts:31-54, src/optim/clip.ts:7-24    AdamW step, global-norm clip
 *   - scripts/train-gpt.ts:105-123,200-242, scripts/params.ts   DP shard / weighted mean
 *
 * Numerics: the reference stores every tensor as Float32Array while JavaScript does
 * its arithmetic in double.  Each op here therefore computes in double and rounds to
 * `real` (f32) exactly where the reference stores into a Float32Array.  Where one
 * tensor receives gradient contributions from several consumers, they are added in
 * the order the reference's reverse-topological backward replays them
 * (tensor.ts:127-166).  Build with -DORACLE_F64 for an all-double variant used only
 * for central-difference gradient checks.
 *
 * Loop-order note: mm_bwd_b (dB = A^T g) adds, for every output element, the same
 * terms in the same order (row index ascending) as tensor.ts:385-391, but iterates
 * rows in the outer loop so it streams memory; the arithmetic is identical.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef ORACLE_F64
typedef double real;
#else
typedef float real;
#endif

#define EXPORT __attribute__((visibility("default")))

static inline real R(double v) { return (real)v; }

/* ------------------------------------------------------------------ RNG */

/* mulberry32 step, src/math/random.ts:8-17 (Math.imul == wrapping uint32 multiply). */
EXPORT double oc_rng_next(uint32_t* state) {
  *state = *state + 0x6d2b79f5u;
  uint32_t t = *state;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

/* Box-Muller, src/math/random.ts:20-25. */
EXPORT double oc_gaussian(uint32_t* state) {
  double u = 0.0;
  while (u == 0.0) u = oc_rng_next(state);
  double v = oc_rng_next(state);
  return sqrt(-2.0 * log(u)) * cos(2.0 * M_PI * v);
}

/* Tensor.randn, src/math/tensor.ts:83-88. */
EXPORT void oc_randn(real* out, size_t n, uint32_t* state, double stddev) {
  for (size_t i = 0; i < n; i++) out[i] = R(oc_gaussian(state) * stddev);
}

/* ------------------------------------------------------------ primitives */

/* Y[M,N] = A[M,K] @ B[K,N]; tensor.ts:362-371 (i-k-j, f32 accumulation, zero skip). */
EXPORT void oc_mm_fwd(const real* A, const real* B, real* Y, int M, int K, int N) {
  memset(Y, 0, sizeof(real) * (size_t)M * N);
  for (int i = 0; i < M; i++) {
    real* y = Y + (size_t)i * N;
    for (int p = 0; p < K; p++) {
      double av = A[(size_t)i * K + p];
      if (av == 0.0) continue;
      const real* b = B + (size_t)p * N;
      for (int j = 0; j < N; j++) y[j] = R((double)y[j] + av * (double)b[j]);
    }
  }
}

/* dA[M,K] += g[M,N] @ B[K,N]^T; tensor.ts:374-381 (double dot over j ascending). */
EXPORT void oc_mm_bwd_a(const real* g, const real* B, real* dA, int M, int K, int N) {
  for (int i = 0; i < M; i++) {
    const real* gi = g + (size_t)i * N;
    int p = 0;
    for (; p + 4 <= K; p += 4) {
      const real* b0 = B + (size_t)p * N;
      const real* b1 = b0 + N;
      const real* b2 = b1 + N;
      const real* b3 = b2 + N;
      double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
      for (int j = 0; j < N; j++) {
        double gv = gi[j];
        s0 += gv * (double)b0[j];
        s1 += gv * (double)b1[j];
        s2 += gv * (double)b2[j];
        s3 += gv * (double)b3[j];
      }
      real* da = dA + (size_t)i * K + p;
      da[0] = R((double)da[0] + s0);
      da[1] = R((double)da[1] + s1);
      da[2] = R((double)da[2] + s2);
      da[3] = R((double)da[3] + s3);
    }
    for (; p < K; p++) {
      const real* bp = B + (size_t)p * N;
      double s = 0;
      for (int j = 0; j < N; j++) s += (double)gi[j] * (double)bp[j];
      dA[(size_t)i * K + p] = R((double)dA[(size_t)i * K + p] + s);
    }
  }
}

/* dB[K,N] += A[M,K]^T @ g[M,N]; tensor.ts:383-391 (double sum over i ascending). */
EXPORT void oc_mm_bwd_b(const real* A, const real* g, real* dB, int M, int K, int N) {
  double* acc = (double*)calloc((size_t)K * N, sizeof(double));
  for (int i = 0; i < M; i++) {
    const real* gi = g + (size_t)i * N;
    for (int p = 0; p < K; p++) {
      double a = A[(size_t)i * K + p];
      double* ap = acc + (size_t)p * N;
      for (int j = 0; j < N; j++) ap[j] += a * (double)gi[j];
    }
  }
  for (size_t q = 0; q < (size_t)K * N; q++) dB[q] = R((double)dB[q] + acc[q]);
  free(acc);
}

/* bmm, tensor.ts:457-514: per group the same three loops as matmul. */
EXPORT void oc_bmm_fwd(const real* A, const real* B, real* Y, int G, int M, int K, int N) {
  for (int g = 0; g < G; g++)
    oc_mm_fwd(A + (size_t)g * M * K, B + (size_t)g * K * N, Y + (size_t)g * M * N, M, K, N);
}
EXPORT void oc_bmm_bwd(const real* A, const real* B, const real* gY, real* dA, real* dB, int G, int M,
                       int K, int N) {
  for (int g = 0; g < G; g++) {
    if (dA) oc_mm_bwd_a(gY + (size_t)g * M * N, B + (size_t)g * K * N, dA + (size_t)g * M * K, M, K, N);
    if (dB) oc_mm_bwd_b(A + (size_t)g * M * K, gY + (size_t)g * M * N, dB + (size_t)g * K * N, M, K, N);
  }
}

/* softmax over the last dim, tensor.ts:542-571. */
EXPORT void oc_softmax_fwd(const real* x, real* y, int rows, int d) {
  for (int r = 0; r < rows; r++) {
    const real* xr = x + (size_t)r * d;
    real* yr = y + (size_t)r * d;
    double mx = -INFINITY;
    for (int j = 0; j < d; j++)
      if (xr[j] > mx) mx = xr[j];
    double sum = 0;
    for (int j = 0; j < d; j++) {
      double e = exp((double)xr[j] - mx);
      yr[j] = R(e);
      sum += e;
    }
    for (int j = 0; j < d; j++) yr[j] = R((double)yr[j] / sum);
  }
}
EXPORT void oc_softmax_bwd(const real* y, const real* g, real* gx, int rows, int d) {
  for (int r = 0; r < rows; r++) {
    const real* yr = y + (size_t)r * d;
    const real* gr = g + (size_t)r * d;
    real* ga = gx + (size_t)r * d;
    double dot = 0;
    for (int j = 0; j < d; j++) dot += (double)gr[j] * (double)yr[j];
    for (int j = 0; j < d; j++) ga[j] = R((double)ga[j] + (double)yr[j] * ((double)gr[j] - dot));
  }
}

/* maskedFillCausal(-1e9), tensor.ts:579-604. */
EXPORT void oc_mask_fwd(const real* x, real* y, int groups, int t) {
  for (int g = 0; g < groups; g++)
    for (int r = 0; r < t; r++)
      for (int c = 0; c < t; c++) {
        size_t o = (size_t)g * t * t + (size_t)r * t + c;
        y[o] = c > r ? R(-1e9) : x[o];
      }
}
EXPORT void oc_mask_bwd(const real* g, real* gx, int groups, int t) {
  for (int gg = 0; gg < groups; gg++)
    for (int r = 0; r < t; r++)
      for (int c = 0; c <= r; c++) {
        size_t o = (size_t)gg * t * t + (size_t)r * t + c;
        gx[o] = R((double)gx[o] + (double)g[o]);
      }
}

/* GELU tanh approximation, tensor.ts:607-619. */
static const double GELU_C = 0.7978845608028654; /* Math.sqrt(2 / Math.PI) */
EXPORT void oc_gelu_fwd(const real* x, real* y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    double v = x[i];
    y[i] = R(0.5 * v * (1 + tanh(GELU_C * (v + 0.044715 * v * v * v))));
  }
}
EXPORT void oc_gelu_bwd(const real* x, const real* g, real* gx, size_t n) {
  for (size_t i = 0; i < n; i++) {
    double v = x[i];
    double inner = GELU_C * (v + 0.044715 * v * v * v);
    double t = tanh(inner);
    double dinner = GELU_C * (1 + 3 * 0.044715 * v * v);
    gx[i] = R((double)gx[i] + (double)g[i] * (0.5 * (1 + t) + 0.5 * v * (1 - t * t) * dinner));
  }
}

/* SiLU, tensor.ts:625-635. */
EXPORT void oc_silu_fwd(const real* x, real* y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    double v = x[i];
    y[i] = R(v / (1 + exp(-v)));
  }
}
EXPORT void oc_silu_bwd(const real* x, const real* y, const real* g, real* gx, size_t n) {
  for (size_t i = 0; i < n; i++) {
    double s = 1 / (1 + exp(-(double)x[i]));
    gx[i] = R((double)gx[i] + (double)g[i] * (s + (double)y[i] * (1 - s)));
  }
}

/* RoPE over [groups, t, hd], tensor.ts:650-700 (f32 cos/sin tables). */
static void rope_tables(int t, int hd, double base, real* cs, real* sn) {
  int half = hd / 2;
  for (int p = 0; p < t; p++)
    for (int i = 0; i < half; i++) {
      double theta = (double)p / pow(base, (double)(2 * i) / (double)hd);
      cs[p * half + i] = R(cos(theta));
      sn[p * half + i] = R(sin(theta));
    }
}
EXPORT void oc_rope_fwd(const real* x, real* y, int groups, int t, int hd, double base) {
  int half = hd / 2;
  real* cs = (real*)malloc(sizeof(real) * t * half);
  real* sn = (real*)malloc(sizeof(real) * t * half);
  rope_tables(t, hd, base, cs, sn);
  for (int g = 0; g < groups; g++)
    for (int p = 0; p < t; p++) {
      size_t off = ((size_t)g * t + p) * hd;
      for (int i = 0; i < half; i++) {
        double c = cs[p * half + i], s = sn[p * half + i];
        double x0 = x[off + 2 * i], x1 = x[off + 2 * i + 1];
        y[off + 2 * i] = R(x0 * c - x1 * s);
        y[off + 2 * i + 1] = R(x0 * s + x1 * c);
      }
    }
  free(cs);
  free(sn);
}
EXPORT void oc_rope_bwd(const real* g, real* gx, int groups, int t, int hd, double base) {
  int half = hd / 2;
  real* cs = (real*)malloc(sizeof(real) * t * half);
  real* sn = (real*)malloc(sizeof(real) * t * half);
  rope_tables(t, hd, base, cs, sn);
  for (int gg = 0; gg < groups; gg++)
    for (int p = 0; p < t; p++) {
      size_t off = ((size_t)gg * t + p) * hd;
      for (int i = 0; i < half; i++) {
        double c = cs[p * half + i], s = sn[p * half + i];
        double g0 = g[off + 2 * i], g1 = g[off + 2 * i + 1];
        gx[off + 2 * i] = R((double)gx[off + 2 * i] + (g0 * c + g1 * s));
        gx[off + 2 * i + 1] = R((double)gx[off + 2 * i + 1] + (-g0 * s + g1 * c));
      }
    }
  free(cs);
  free(sn);
}

/* gatherRows, tensor.ts:520-539.  Returns -1 on an out-of-range index (the reference throws). */
EXPORT int oc_gather_fwd(const real* table, const int32_t* idx, real* out, int n, int vocab, int dim) {
  for (int i = 0; i < n; i++) {
    int r = idx[i];
    if (r < 0 || r >= vocab) return -1;
    memcpy(out + (size_t)i * dim, table + (size_t)r * dim, sizeof(real) * dim);
  }
  return 0;
}
EXPORT void oc_gather_bwd(const int32_t* idx, const real* g, real* gtable, int n, int dim) {
  for (int i = 0; i < n; i++) {
    real* row = gtable + (size_t)idx[i] * dim;
    const real* gi = g + (size_t)i * dim;
    for (int j = 0; j < dim; j++) row[j] = R((double)row[j] + (double)gi[j]);
  }
}

/* crossEntropyLogits, tensor.ts:708-745.  probs (f32) is kept for the backward.
   Returns the f32 mean loss; -1 (and *err=1) on an out-of-range target. */
EXPORT double oc_ce_fwd(const real* logits, const int32_t* tgt, real* probs, int n, int vocab, int* err) {
  double total = 0;
  if (err) *err = 0;
  for (int i = 0; i < n; i++) {
    const real* x = logits + (size_t)i * vocab;
    real* pr = probs + (size_t)i * vocab;
    double mx = -INFINITY;
    for (int j = 0; j < vocab; j++)
      if (x[j] > mx) mx = x[j];
    double sum = 0;
    for (int j = 0; j < vocab; j++) {
      double e = exp((double)x[j] - mx);
      pr[j] = R(e);
      sum += e;
    }
    for (int j = 0; j < vocab; j++) pr[j] = R((double)pr[j] / sum);
    int t = tgt[i];
    if (t < 0 || t >= vocab) {
      if (err) *err = 1;
      return -1;
    }
    total += mx + log(sum) - (double)x[t];
  }
  return (double)R(total / n);
}
EXPORT void oc_ce_bwd(const real* probs, const int32_t* tgt, double gloss, real* glogits, int n, int vocab) {
  double scale = gloss / n;
  for (int i = 0; i < n; i++) {
    real* ga = glogits + (size_t)i * vocab;
    const real* pr = probs + (size_t)i * vocab;
    for (int j = 0; j < vocab; j++) ga[j] = R((double)ga[j] + scale * (double)pr[j]);
    ga[tgt[i]] = R((double)ga[tgt[i]] - scale);
  }
}

/* General N-d permute (tensor.ts:425-454): out[o] = in[map[o]]; backward scatters. */
static void permute_map(const int* shape, const int* perm, int nd, int64_t* map) {
  int64_t in_str[8], out_shape[8], out_str[8], n = 1;
  for (int d = nd - 1, s = 1; d >= 0; d--) {
    in_str[d] = s;
    s *= shape[d];
  }
  for (int d = 0; d < nd; d++) {
    out_shape[d] = shape[perm[d]];
    n *= shape[d];
  }
  for (int d = nd - 1, s = 1; d >= 0; d--) {
    out_str[d] = s;
    s *= (int)out_shape[d];
  }
  for (int64_t o = 0; o < n; o++) {
    int64_t rem = o, src = 0;
    for (int d = 0; d < nd; d++) {
      int64_t c = rem / out_str[d];
      rem -= c * out_str[d];
      src += c * in_str[perm[d]];
    }
    map[o] = src;
  }
}
EXPORT void oc_permute_fwd(const real* x, real* y, const int* shape, const int* perm, int nd) {
  int64_t n = 1;
  for (int d = 0; d < nd; d++) n *= shape[d];
  int64_t* map = (int64_t*)malloc(sizeof(int64_t) * n);
  permute_map(shape, perm, nd, map);
  for (int64_t o = 0; o < n; o++) y[o] = x[map[o]];
  free(map);
}
EXPORT void oc_permute_bwd(const real* g, real* gx, const int* shape, const int* perm, int nd) {
  int64_t n = 1;
  for (int d = 0; d < nd; d++) n *= shape[d];
  int64_t* map = (int64_t*)malloc(sizeof(int64_t) * n);
  permute_map(shape, perm, nd, map);
  for (int64_t o = 0; o < n; o++) gx[map[o]] = R((double)gx[map[o]] + (double)g[o]);
  free(map);
}

/* ------------------------------------------------------ composite norms */

/* RMSNorm as composed in src/nn/rmsnorm.ts:24-27:
     s1 = x*x; ms = sum(s1,-1)*f32(1/d); r = sqrt(ms + f32(eps)); xn = x / r; y = xn * gamma
   Saved: xn[rows,d], r[rows] (plus recomputable pieces). */
typedef struct {
  real *xn, *rms, *ms_eps;
} rms_saved;

static void rms_fwd(const real* x, const real* gamma, real* y, int rows, int d, double eps, real* xn,
                    real* rms, real* ms_eps_out) {
  real inv_d = R(1.0 / d), epsf = R(eps);
  for (int r = 0; r < rows; r++) {
    const real* xr = x + (size_t)r * d;
    real acc = 0;
    for (int j = 0; j < d; j++) acc = R((double)acc + (double)R((double)xr[j] * xr[j]));
    real ms = R((double)acc * inv_d);
    real mse = R((double)ms + epsf);
    real rr = R(sqrt((double)mse));
    ms_eps_out[r] = mse;
    rms[r] = rr;
    for (int j = 0; j < d; j++) {
      real v = R((double)xr[j] / rr);
      xn[(size_t)r * d + j] = v;
      y[(size_t)r * d + j] = R((double)v * gamma[j]);
    }
  }
}

/* Backward of the composite, following the closures' reverse order:
   mul(xn,gamma) -> div(x,r) -> sqrt -> addScalar -> mulScalar -> sum -> mul(x,x).
   dx receives [div, mul-a, mul-b] contributions in that order (dx is accumulated). */
static void rms_bwd(const real* x, const real* gamma, const real* gy, const real* xn, const real* rms,
                    int rows, int d, real* dx, real* dgamma) {
  real inv_d = R(1.0 / d);
  real* dxn = (real*)malloc(sizeof(real) * d);
  for (int r = 0; r < rows; r++) {
    const real* g = gy + (size_t)r * d;
    const real* xr = x + (size_t)r * d;
    const real* xnr = xn + (size_t)r * d;
    real* dxr = dx + (size_t)r * d;
    double rr = rms[r];
    /* mul(xn, gamma): a then b */
    for (int j = 0; j < d; j++) dxn[j] = R((double)g[j] * gamma[j]);
    if (dgamma)
      for (int j = 0; j < d; j++) dgamma[j] = R((double)dgamma[j] + (double)g[j] * xnr[j]);
    /* div(x, r): dx += g / r ; dr += -g*x / (r*r) */
    for (int j = 0; j < d; j++) dxr[j] = R((double)dxr[j] + (double)dxn[j] / rr);
    real dr = 0;
    for (int j = 0; j < d; j++) dr = R((double)dr + (-(double)dxn[j] * xr[j]) / (rr * rr));
    /* sqrt: d(ms_eps) += g / (2 y) */
    real dmse = R((double)dr / (2 * rr));
    /* addScalar: d(ms) += g */
    real dms = dmse;
    /* mulScalar(1/d): d(sum) += g * f32(1/d) */
    real dsum = R((double)dms * inv_d);
    /* sum backward: d(s1)[j] += dsum ; mul(x,x): dx += g*x (a), dx += g*x (b) */
    for (int j = 0; j < d; j++) dxr[j] = R((double)dxr[j] + (double)dsum * xr[j]);
    for (int j = 0; j < d; j++) dxr[j] = R((double)dxr[j] + (double)dsum * xr[j]);
  }
  free(dxn);
}

/* LayerNorm as composed in src/nn/layernorm.ts:20-26:
     mu = sum(x)*f32(1/d); c = x - mu; var = sum(c*c)*f32(1/d); sd = sqrt(var + f32(eps));
     nrm = c / sd; y = nrm*gamma + beta */
static void ln_fwd(const real* x, const real* gamma, const real* beta, real* y, int rows, int d,
                   double eps, real* cen, real* nrm, real* sd) {
  real inv_d = R(1.0 / d), epsf = R(eps);
  for (int r = 0; r < rows; r++) {
    const real* xr = x + (size_t)r * d;
    real* cr = cen + (size_t)r * d;
    real acc = 0;
    for (int j = 0; j < d; j++) acc = R((double)acc + xr[j]);
    real mu = R((double)acc * inv_d);
    for (int j = 0; j < d; j++) cr[j] = R((double)xr[j] - mu);
    real acc2 = 0;
    for (int j = 0; j < d; j++) acc2 = R((double)acc2 + (double)R((double)cr[j] * cr[j]));
    real var = R((double)acc2 * inv_d);
    real s = R(sqrt((double)R((double)var + epsf)));
    sd[r] = s;
    for (int j = 0; j < d; j++) {
      real v = R((double)cr[j] / s);
      nrm[(size_t)r * d + j] = v;
      y[(size_t)r * d + j] = R((double)R((double)v * gamma[j]) + beta[j]);
    }
  }
}

/* Reverse order: add(.,beta) -> mul(nrm,gamma) -> div(c,sd) -> sqrt -> addScalar -> mulScalar
   -> sum -> mul(c,c) -> sub(x,mu) -> mulScalar -> sum(x).  dc gets [div, mul-a, mul-b];
   dx gets [sub-a, sum] (accumulated onto whatever dx already holds). */
static void ln_bwd(const real* gy, const real* gamma, const real* cen, const real* nrm, const real* sd,
                   int rows, int d, real* dx, real* dgamma, real* dbeta) {
  real inv_d = R(1.0 / d);
  real* dn = (real*)malloc(sizeof(real) * d);
  real* dc = (real*)malloc(sizeof(real) * d);
  for (int r = 0; r < rows; r++) {
    const real* g = gy + (size_t)r * d;
    const real* cr = cen + (size_t)r * d;
    const real* nr = nrm + (size_t)r * d;
    real* dxr = dx + (size_t)r * d;
    double s = sd[r];
    /* add(nm, beta): dnm = g ; dbeta += g */
    if (dbeta)
      for (int j = 0; j < d; j++) dbeta[j] = R((double)dbeta[j] + g[j]);
    /* mul(nrm, gamma) */
    for (int j = 0; j < d; j++) dn[j] = R((double)g[j] * gamma[j]);
    if (dgamma)
      for (int j = 0; j < d; j++) dgamma[j] = R((double)dgamma[j] + (double)g[j] * nr[j]);
    /* div(c, sd) */
    for (int j = 0; j < d; j++) dc[j] = R((double)dn[j] / s);
    real dsd = 0;
    for (int j = 0; j < d; j++) dsd = R((double)dsd + (-(double)dn[j] * cr[j]) / (s * s));
    real dve = R((double)dsd / (2 * s));
    real dvar = dve;
    real dsum2 = R((double)dvar * inv_d);
    /* mul(c,c): dc += g*c twice */
    for (int j = 0; j < d; j++) dc[j] = R((double)dc[j] + (double)dsum2 * cr[j]);
    for (int j = 0; j < d; j++) dc[j] = R((double)dc[j] + (double)dsum2 * cr[j]);
    /* sub(x, mu): dx += dc ; dmu += -dc */
    for (int j = 0; j < d; j++) dxr[j] = R((double)dxr[j] + dc[j]);
    real dmu = 0;
    for (int j = 0; j < d; j++) dmu = R((double)dmu - (double)dc[j]);
    real dsum = R((double)dmu * inv_d);
    for (int j = 0; j < d; j++) dxr[j] = R((double)dxr[j] + dsum);
  }
  free(dn);
  free(dc);
}

/* Op-level exports of the composite norms (forward + backward against upstream grad gy). */
EXPORT void oc_rmsnorm(const real* x, const real* gamma, real* y, const real* gy, real* dx, real* dgamma,
                       int rows, int d, double eps) {
  real* xn = (real*)malloc(sizeof(real) * (size_t)rows * d);
  real* rr = (real*)malloc(sizeof(real) * rows);
  real* me = (real*)malloc(sizeof(real) * rows);
  rms_fwd(x, gamma, y, rows, d, eps, xn, rr, me);
  if (gy) rms_bwd(x, gamma, gy, xn, rr, rows, d, dx, dgamma);
  free(xn);
  free(rr);
  free(me);
}
EXPORT void oc_layernorm(const real* x, const real* gamma, const real* beta, real* y, const real* gy,
                         real* dx, real* dgamma, real* dbeta, int rows, int d, double eps) {
  real* c = (real*)malloc(sizeof(real) * (size_t)rows * d);
  real* nr = (real*)malloc(sizeof(real) * (size_t)rows * d);
  real* sd = (real*)malloc(sizeof(real) * rows);
  ln_fwd(x, gamma, beta, y, rows, d, eps, c, nr, sd);
  if (gy) ln_bwd(gy, gamma, c, nr, sd, rows, d, dx, dgamma, dbeta);
  free(c);
  free(nr);
  free(sd);
}

/* ----------------------------------------------------------------- GPT */

/* cfg[] = {vocab, block, n_layer, n_head, n_embd, arch(0 gpt2, 1 modern), hidden(0 = mlpHidden)} */
typedef struct {
  int V, T, L, H, E, modern, hid;
} gcfg;

static gcfg read_cfg(const int* c) {
  gcfg g = {c[0], c[1], c[2], c[3], c[4], c[5], c[6]};
  if (g.hid <= 0) {
    /* mlpHidden, src/models/gpt.ts:69-72 (Math.round == floor(x + 0.5) for x > 0) */
    g.hid = g.modern ? (int)fmax(64.0, floor((8.0 * g.E) / 3.0 / 64.0 + 0.5) * 64.0) : 4 * g.E;
  }
  return g;
}

typedef struct {
  size_t ln1g, ln1b, qW, qb, kW, kb, vW, vb, projW, projb, ln2g, ln2b, fcW, fcb, mpW, mpb, gateW, upW,
      downW;
} boff;
typedef struct {
  size_t wte, wpe, lnfg, lnfb, total;
  int ntensors;
  boff b[256];
} moff;

/* parameters() order: src/models/gpt.ts:225-239 + src/nn/module.ts:13-35 field walk
   (identical to src/models/gpu-gpt.ts:118-132). */
static void layout(const gcfg* c, moff* o) {
  size_t p = 0;
  int nt = 0;
#define TAKE(field, n) \
  do {                 \
    field = p;         \
    p += (n);          \
    nt++;              \
  } while (0)
  size_t E = c->E, EE = (size_t)c->E * c->E, Eh = (size_t)c->E * c->hid;
  TAKE(o->wte, (size_t)c->V * E);
  if (!c->modern) TAKE(o->wpe, (size_t)c->T * E);
  for (int l = 0; l < c->L; l++) {
    boff* b = &o->b[l];
    if (c->modern) {
      TAKE(b->ln1g, E);
      TAKE(b->qW, EE);
      TAKE(b->kW, EE);
      TAKE(b->vW, EE);
      TAKE(b->projW, EE);
      TAKE(b->ln2g, E);
      TAKE(b->gateW, Eh);
      TAKE(b->upW, Eh);
      TAKE(b->downW, Eh);
    } else {
      TAKE(b->ln1g, E);
      TAKE(b->ln1b, E);
      TAKE(b->qW, EE);
      TAKE(b->qb, E);
      TAKE(b->kW, EE);
      TAKE(b->kb, E);
      TAKE(b->vW, EE);
      TAKE(b->vb, E);
      TAKE(b->projW, EE);
      TAKE(b->projb, E);
      TAKE(b->ln2g, E);
      TAKE(b->ln2b, E);
      TAKE(b->fcW, Eh);
      TAKE(b->fcb, (size_t)c->hid);
      TAKE(b->mpW, Eh);
      TAKE(b->mpb, E);
    }
  }
  TAKE(o->lnfg, E);
  if (!c->modern) TAKE(o->lnfb, E);
#undef TAKE
  o->total = p;
  o->ntensors = nt;
}

EXPORT int oc_hidden(const int* cfg) { return read_cfg(cfg).hid; }
EXPORT size_t oc_num_params(const int* cfg) {
  gcfg c = read_cfg(cfg);
  moff o;
  layout(&c, &o);
  return o.total;
}
/* Writes [rows, cols] per tensor (1-D tensors get cols = 0); returns the tensor count. */
EXPORT int oc_param_shapes(const int* cfg, int* shapes) {
  gcfg c = read_cfg(cfg);
  int k = 0;
#define SH(r, cc)          \
  do {                     \
    shapes[2 * k] = (r);   \
    shapes[2 * k + 1] = (cc); \
    k++;                   \
  } while (0)
  SH(c.V, c.E);
  if (!c.modern) SH(c.T, c.E);
  for (int l = 0; l < c.L; l++) {
    if (c.modern) {
      SH(c.E, 0);
      SH(c.E, c.E);
      SH(c.E, c.E);
      SH(c.E, c.E);
      SH(c.E, c.E);
      SH(c.E, 0);
      SH(c.E, c.hid);
      SH(c.E, c.hid);
      SH(c.hid, c.E);
    } else {
      SH(c.E, 0);
      SH(c.E, 0);
      SH(c.E, c.E);
      SH(c.E, 0);
      SH(c.E, c.E);
      SH(c.E, 0);
      SH(c.E, c.E);
      SH(c.E, 0);
      SH(c.E, c.E);
      SH(c.E, 0);
      SH(c.E, 0);
      SH(c.E, 0);
      SH(c.E, c.hid);
      SH(c.hid, 0);
      SH(c.hid, c.E);
      SH(c.E, 0);
    }
  }
  SH(c.E, 0);
  if (!c.modern) SH(c.E, 0);
#undef SH
  return k;
}

/* GPT constructor init, src/models/gpt.ts:225-239 with Linear (src/nn/linear.ts:18-23):
   wte, [wpe], then per block q,k,v,proj, then gate,up,down | fc,proj.  Gains 1, biases 0. */
EXPORT void oc_init_state(const int* cfg, uint32_t* state, real* params);
EXPORT void oc_init(const int* cfg, uint32_t seed, real* params) {
  uint32_t st = seed;
  oc_init_state(cfg, &st, params);
}

/* Same, drawing from (and advancing) a caller-owned mulberry32 state, as when the reference
   shares one rng between GPT construction and generate (tests/models/gpt.test.ts:46-69). */
EXPORT void oc_init_state(const int* cfg, uint32_t* state, real* params) {
  gcfg c = read_cfg(cfg);
  moff o;
  layout(&c, &o);
  uint32_t st = *state;
  const double std0 = 0.02, stdr = 0.02 / sqrt(2.0 * c.L);
  size_t E = c.E, EE = E * E, Eh = E * (size_t)c.hid;
  oc_randn(params + o.wte, (size_t)c.V * E, &st, std0);
  if (!c.modern) oc_randn(params + o.wpe, (size_t)c.T * E, &st, std0);
  for (int l = 0; l < c.L; l++) {
    boff* b = &o.b[l];
    for (size_t i = 0; i < E; i++) params[b->ln1g + i] = 1;
    for (size_t i = 0; i < E; i++) params[b->ln2g + i] = 1;
    oc_randn(params + b->qW, EE, &st, std0);
    oc_randn(params + b->kW, EE, &st, std0);
    oc_randn(params + b->vW, EE, &st, std0);
    oc_randn(params + b->projW, EE, &st, stdr);
    if (c.modern) {
      oc_randn(params + b->gateW, Eh, &st, std0);
      oc_randn(params + b->upW, Eh, &st, std0);
      oc_randn(params + b->downW, Eh, &st, stdr);
    } else {
      memset(params + b->ln1b, 0, sizeof(real) * E);
      memset(params + b->ln2b, 0, sizeof(real) * E);
      memset(params + b->qb, 0, sizeof(real) * E);
      memset(params + b->kb, 0, sizeof(real) * E);
      memset(params + b->vb, 0, sizeof(real) * E);
      memset(params + b->projb, 0, sizeof(real) * E);
      memset(params + b->mpb, 0, sizeof(real) * E);
      memset(params + b->fcb, 0, sizeof(real) * c.hid);
      oc_randn(params + b->fcW, Eh, &st, std0);
      oc_randn(params + b->mpW, Eh, &st, stdr);
    }
  }
  for (size_t i = 0; i < E; i++) params[o.lnfg + i] = 1;
  if (!c.modern) memset(params + o.lnfb, 0, sizeof(real) * E);
  *state = st;
}

/* Per-layer saved activations. */
typedef struct {
  real *x;                 /* block input [N,E] (residual stream) */
  real *xn1, *r1, *y1;     /* norm1: normalized, rms / sd, output */
  real *c1;                /* gpt2: centered */
  real *q, *k, *v;         /* after split heads (+rope for q,k) [G,T,hd] */
  real *qpre, *kpre;       /* modern: split heads before rope (unused in bwd, kept for clarity) */
  real *P;                 /* softmax probs [G,T,T] */
  real *am;                /* merged attention output [N,E] */
  real *h;                 /* after attention residual */
  real *xn2, *r2, *y2, *c2;
  real *a1;                /* modern gate preact / gpt2 fc preact (with bias) [N,hid] */
  real *a2;                /* modern up [N,hid] */
  real *s1;                /* modern silu(gate) / gpt2 gelu output [N,hid] */
  real *hid;               /* modern silu*up [N,hid] */
} layer_act;

#define ALLOC(n) ((real*)calloc((size_t)(n), sizeof(real)))

/* x[N,E] -> heads [G,T,hd] (reshape/permute/reshape, gpt.ts:105-110). */
static void split_heads(const real* x, real* out, int b, int t, int H, int hd) {
  int E = H * hd;
  for (int bi = 0; bi < b; bi++)
    for (int h = 0; h < H; h++)
      for (int ti = 0; ti < t; ti++)
        memcpy(out + (((size_t)bi * H + h) * t + ti) * hd, x + ((size_t)bi * t + ti) * E + (size_t)h * hd,
               sizeof(real) * hd);
}
/* heads [G,T,hd] -> x[N,E] (gpt.ts:135-139) */
static void merge_heads(const real* in, real* x, int b, int t, int H, int hd) {
  int E = H * hd;
  for (int bi = 0; bi < b; bi++)
    for (int h = 0; h < H; h++)
      for (int ti = 0; ti < t; ti++)
        memcpy(x + ((size_t)bi * t + ti) * E + (size_t)h * hd, in + (((size_t)bi * H + h) * t + ti) * hd,
               sizeof(real) * hd);
}

/* out[N,n] = A @ W (+ bias broadcast, as Linear.forward then .add(bias)) */
static void linear_fwd(const real* A, const real* W, const real* bias, real* out, int N, int K, int n) {
  oc_mm_fwd(A, W, out, N, K, n);
  if (bias)
    for (int i = 0; i < N; i++)
      for (int j = 0; j < n; j++) out[(size_t)i * n + j] = R((double)out[(size_t)i * n + j] + bias[j]);
}
/* Backward of Linear (+bias): add(out, b) closure (a then b via segsum order), then matmul closure
   (dA then dW).  dA and dW are accumulated. */
static void linear_bwd(const real* A, const real* W, const real* g, real* dA, real* dW, real* db, int N, int K,
                       int n) {
  if (db)
    for (int i = 0; i < N; i++)
      for (int j = 0; j < n; j++) db[j] = R((double)db[j] + g[(size_t)i * n + j]);
  if (dA) oc_mm_bwd_a(g, W, dA, N, K, n);
  if (dW) oc_mm_bwd_b(A, g, dW, N, K, n);
}

/* One model forward (and optional backward).  Returns the f32 loss, or NAN with *err set
   on an out-of-range token / target (the reference throws in both cases, tensor.ts:527,728).
   logits_copy, when given, receives the [b*t, V] logits. */
static double gpt_run(const int* cfg, const real* params, real* grads, const int32_t* ids,
                      const int32_t* tgt, int b, int t, int* err, real* logits_copy) {
  gcfg c = read_cfg(cfg);
  moff o;
  layout(&c, &o);
  if (err) *err = 0;
  if (t > c.T) {
    if (err) *err = 2;
    return NAN;
  }
  const int N = b * t, E = c.E, H = c.H, hd = E / H, G = b * H, V = c.V, hidn = c.hid;
  const double eps = 1e-5, base = 10000.0;
  const real scale = R(1.0 / sqrt((double)hd));
  for (int i = 0; i < N; i++)
    if (ids[i] < 0 || ids[i] >= V || tgt[i] < 0 || tgt[i] >= V) {
      if (err) *err = 1;
      return NAN;
    }

  layer_act* A = (layer_act*)calloc(c.L, sizeof(layer_act));
  real* x = ALLOC((size_t)N * E);
  real* pos = NULL;
  /* embeddings (gpt.ts:262-270) */
  oc_gather_fwd(params + o.wte, ids, x, N, V, E);
  int32_t* pids = NULL;
  if (!c.modern) {
    pos = ALLOC((size_t)N * E);
    pids = (int32_t*)malloc(sizeof(int32_t) * N);
    for (int i = 0; i < N; i++) pids[i] = i % t;
    oc_gather_fwd(params + o.wpe, pids, pos, N, c.T, E);
    for (size_t i = 0; i < (size_t)N * E; i++) x[i] = R((double)x[i] + pos[i]);
  }
  real* tmpS = ALLOC((size_t)G * t * t);
  real* tmpH = ALLOC((size_t)G * t * hd);
  real* tmpN = ALLOC((size_t)N * E);
  real* tmpN2 = ALLOC((size_t)N * E);
  real* tmpN3 = ALLOC((size_t)N * E);
  real* kT = ALLOC((size_t)G * t * hd);
  for (int l = 0; l < c.L; l++) {
    boff* bo = &o.b[l];
    layer_act* a = &A[l];
    a->x = x;
    a->y1 = ALLOC((size_t)N * E);
    a->xn1 = ALLOC((size_t)N * E);
    a->r1 = ALLOC(N);
    real* me = ALLOC(N);
    if (c.modern) {
      rms_fwd(x, params + bo->ln1g, a->y1, N, E, eps, a->xn1, a->r1, me);
    } else {
      a->c1 = ALLOC((size_t)N * E);
      ln_fwd(x, params + bo->ln1g, params + bo->ln1b, a->y1, N, E, eps, a->c1, a->xn1, a->r1);
    }
    /* attention (gpt.ts:112-141) */
    a->q = ALLOC((size_t)G * t * hd);
    a->k = ALLOC((size_t)G * t * hd);
    a->v = ALLOC((size_t)G * t * hd);
    linear_fwd(a->y1, params + bo->qW, c.modern ? NULL : params + bo->qb, tmpN, N, E, E);
    split_heads(tmpN, c.modern ? tmpH : a->q, b, t, H, hd);
    if (c.modern) oc_rope_fwd(tmpH, a->q, G, t, hd, base);
    linear_fwd(a->y1, params + bo->kW, c.modern ? NULL : params + bo->kb, tmpN, N, E, E);
    split_heads(tmpN, c.modern ? tmpH : a->k, b, t, H, hd);
    if (c.modern) oc_rope_fwd(tmpH, a->k, G, t, hd, base);
    linear_fwd(a->y1, params + bo->vW, c.modern ? NULL : params + bo->vb, tmpN, N, E, E);
    split_heads(tmpN, a->v, b, t, H, hd);
    /* scores = q @ k^T * scale, masked, softmax */
    for (int g = 0; g < G; g++)
      for (int j = 0; j < t; j++)
        for (int p = 0; p < hd; p++) kT[((size_t)g * hd + p) * t + j] = a->k[((size_t)g * t + j) * hd + p];
    oc_bmm_fwd(a->q, kT, tmpS, G, t, hd, t);
    for (size_t i = 0; i < (size_t)G * t * t; i++) tmpS[i] = R((double)tmpS[i] * scale);
    oc_mask_fwd(tmpS, tmpS, G, t);
    a->P = ALLOC((size_t)G * t * t);
    oc_softmax_fwd(tmpS, a->P, G * t, t);
    oc_bmm_fwd(a->P, a->v, tmpH, G, t, t, hd);
    a->am = ALLOC((size_t)N * E);
    merge_heads(tmpH, a->am, b, t, H, hd);
    linear_fwd(a->am, params + bo->projW, c.modern ? NULL : params + bo->projb, tmpN, N, E, E);
    a->h = ALLOC((size_t)N * E);
    for (size_t i = 0; i < (size_t)N * E; i++) a->h[i] = R((double)x[i] + tmpN[i]);
    /* MLP */
    a->y2 = ALLOC((size_t)N * E);
    a->xn2 = ALLOC((size_t)N * E);
    a->r2 = ALLOC(N);
    if (c.modern) {
      rms_fwd(a->h, params + bo->ln2g, a->y2, N, E, eps, a->xn2, a->r2, me);
    } else {
      a->c2 = ALLOC((size_t)N * E);
      ln_fwd(a->h, params + bo->ln2g, params + bo->ln2b, a->y2, N, E, eps, a->c2, a->xn2, a->r2);
    }
    free(me);
    a->a1 = ALLOC((size_t)N * hidn);
    a->s1 = ALLOC((size_t)N * hidn);
    real* xo = ALLOC((size_t)N * E);
    if (c.modern) {
      /* SwiGLU, gpt.ts:187-192 */
      a->a2 = ALLOC((size_t)N * hidn);
      a->hid = ALLOC((size_t)N * hidn);
      oc_mm_fwd(a->y2, params + bo->gateW, a->a1, N, E, hidn);
      oc_silu_fwd(a->a1, a->s1, (size_t)N * hidn);
      oc_mm_fwd(a->y2, params + bo->upW, a->a2, N, E, hidn);
      for (size_t i = 0; i < (size_t)N * hidn; i++) a->hid[i] = R((double)a->s1[i] * a->a2[i]);
      oc_mm_fwd(a->hid, params + bo->downW, tmpN, N, hidn, E);
    } else {
      /* GeluMLP, gpt.ts:158-163 */
      linear_fwd(a->y2, params + bo->fcW, params + bo->fcb, a->a1, N, E, hidn);
      oc_gelu_fwd(a->a1, a->s1, (size_t)N * hidn);
      linear_fwd(a->s1, params + bo->mpW, params + bo->mpb, tmpN, N, hidn, E);
    }
    for (size_t i = 0; i < (size_t)N * E; i++) xo[i] = R((double)a->h[i] + tmpN[i]);
    x = xo;
  }
  /* final norm + tied head + CE (gpt.ts:271-283) */
  real* yf = ALLOC((size_t)N * E);
  real* xnf = ALLOC((size_t)N * E);
  real* rf = ALLOC(N);
  real* cf = NULL;
  {
    real* me = ALLOC(N);
    if (c.modern) {
      rms_fwd(x, params + o.lnfg, yf, N, E, eps, xnf, rf, me);
    } else {
      cf = ALLOC((size_t)N * E);
      ln_fwd(x, params + o.lnfg, params + o.lnfb, yf, N, E, eps, cf, xnf, rf);
    }
    free(me);
  }
  real* wteT = ALLOC((size_t)E * V);
  const real* wte = params + o.wte;
  for (int v = 0; v < V; v++)
    for (int p = 0; p < E; p++) wteT[(size_t)p * V + v] = wte[(size_t)v * E + p];
  real* logits = ALLOC((size_t)N * V);
  oc_mm_fwd(yf, wteT, logits, N, E, V);
  if (logits_copy) memcpy(logits_copy, logits, sizeof(real) * (size_t)N * V);
  real* probs = ALLOC((size_t)N * V);
  int cerr = 0;
  double loss = oc_ce_fwd(logits, tgt, probs, N, V, &cerr);

  if (grads) {
    /* ---------------- backward, in the reference's reverse-topological order */
    real* dlog = ALLOC((size_t)N * V);
    oc_ce_bwd(probs, tgt, 1.0, dlog, N, V);
    real* dyf = ALLOC((size_t)N * E);
    real* dwteT = ALLOC((size_t)E * V);
    oc_mm_bwd_a(dlog, wteT, dyf, N, E, V);
    oc_mm_bwd_b(yf, dlog, dwteT, N, E, V);
    free(dlog);
    real* dx = ALLOC((size_t)N * E);
    if (c.modern)
      rms_bwd(x, params + o.lnfg, dyf, xnf, rf, N, E, dx, grads + o.lnfg);
    else
      ln_bwd(dyf, params + o.lnfg, cf, xnf, rf, N, E, dx, grads + o.lnfg, grads + o.lnfb);
    real* dh = ALLOC((size_t)N * E);
    real* dhid = ALLOC((size_t)N * hidn);
    real* dhid2 = ALLOC((size_t)N * hidn);
    real* dy = ALLOC((size_t)N * E);
    real* dS = ALLOC((size_t)G * t * t);
    real* dS2 = ALLOC((size_t)G * t * t);
    real* dq = ALLOC((size_t)G * t * hd);
    real* dk = ALLOC((size_t)G * t * hd);
    real* dkT = ALLOC((size_t)G * hd * t);
    real* dv = ALLOC((size_t)G * t * hd);
    real* dqr = ALLOC((size_t)G * t * hd);
    for (int l = c.L - 1; l >= 0; l--) {
      boff* bo = &o.b[l];
      layer_act* a = &A[l];
      /* block output = h + mlp(ln2(h)): dh = dx (residual a), dmlp = dx (b) */
      memcpy(dh, dx, sizeof(real) * (size_t)N * E);
      memset(dy, 0, sizeof(real) * (size_t)N * E);
      if (c.modern) {
        memset(dhid, 0, sizeof(real) * (size_t)N * hidn);
        oc_mm_bwd_a(dx, params + bo->downW, dhid, N, hidn, E);
        oc_mm_bwd_b(a->hid, dx, grads + bo->downW, N, hidn, E);
        /* hid = s1 * a2: d(s1) = g*a2 (a), d(a2) = g*s1 (b) */
        for (size_t i = 0; i < (size_t)N * hidn; i++) {
          double g = dhid[i];
          dhid2[i] = R(g * a->s1[i]);
          dhid[i] = R(g * a->a2[i]);
        }
        /* silu bwd -> d(gate preact) */
        real* dgate = ALLOC((size_t)N * hidn);
        oc_silu_bwd(a->a1, a->s1, dhid, dgate, (size_t)N * hidn);
        /* gate matmul first, then up (reverse topo: mul, silu, gate mm, up mm) */
        oc_mm_bwd_a(dgate, params + bo->gateW, dy, N, E, hidn);
        oc_mm_bwd_b(a->y2, dgate, grads + bo->gateW, N, E, hidn);
        oc_mm_bwd_a(dhid2, params + bo->upW, dy, N, E, hidn);
        oc_mm_bwd_b(a->y2, dhid2, grads + bo->upW, N, E, hidn);
        free(dgate);
      } else {
        memset(dhid, 0, sizeof(real) * (size_t)N * hidn);
        linear_bwd(a->s1, params + bo->mpW, dx, dhid, grads + bo->mpW, grads + bo->mpb, N, hidn, E);
        memset(dhid2, 0, sizeof(real) * (size_t)N * hidn);
        oc_gelu_bwd(a->a1, dhid, dhid2, (size_t)N * hidn);
        linear_bwd(a->y2, params + bo->fcW, dhid2, dy, grads + bo->fcW, grads + bo->fcb, N, E, hidn);
      }
      /* ln2 backward into dh (already holds the residual contribution) */
      if (c.modern)
        rms_bwd(a->h, params + bo->ln2g, dy, a->xn2, a->r2, N, E, dh, grads + bo->ln2g);
      else
        ln_bwd(dy, params + bo->ln2g, a->c2, a->xn2, a->r2, N, E, dh, grads + bo->ln2g, grads + bo->ln2b);
      /* h = x + attn(ln1(x)): dx = dh (a), dattn = dh (b) */
      memcpy(dx, dh, sizeof(real) * (size_t)N * E);
      /* proj */
      memset(tmpN2, 0, sizeof(real) * (size_t)N * E);
      linear_bwd(a->am, params + bo->projW, dh, tmpN2, grads + bo->projW,
                 c.modern ? NULL : grads + bo->projb, N, E, E);
      split_heads(tmpN2, tmpH, b, t, H, hd); /* datt [G,T,hd] */
      /* att = P @ v */
      memset(dS, 0, sizeof(real) * (size_t)G * t * t);
      memset(dv, 0, sizeof(real) * (size_t)G * t * hd);
      oc_bmm_bwd(a->P, a->v, tmpH, dS, dv, G, t, t, hd);
      /* softmax */
      memset(dS2, 0, sizeof(real) * (size_t)G * t * t);
      oc_softmax_bwd(a->P, dS, dS2, G * t, t);
      /* mask */
      memset(dS, 0, sizeof(real) * (size_t)G * t * t);
      oc_mask_bwd(dS2, dS, G, t);
      /* scale */
      for (size_t i = 0; i < (size_t)G * t * t; i++) dS[i] = R((double)dS[i] * scale);
      /* scores = q @ kT */
      for (int g = 0; g < G; g++)
        for (int j = 0; j < t; j++)
          for (int p = 0; p < hd; p++) kT[((size_t)g * hd + p) * t + j] = a->k[((size_t)g * t + j) * hd + p];
      memset(dq, 0, sizeof(real) * (size_t)G * t * hd);
      memset(dkT, 0, sizeof(real) * (size_t)G * hd * t);
      oc_bmm_bwd(a->q, kT, dS, dq, dkT, G, t, hd, t);
      for (int g = 0; g < G; g++)
        for (int j = 0; j < t; j++)
          for (int p = 0; p < hd; p++) dk[((size_t)g * t + j) * hd + p] = dkT[((size_t)g * hd + p) * t + j];
      memset(dy, 0, sizeof(real) * (size_t)N * E);
      /* q chain (rope bwd, merge, matmul), then k, then v */
      if (c.modern) {
        memset(dqr, 0, sizeof(real) * (size_t)G * t * hd);
        oc_rope_bwd(dq, dqr, G, t, hd, base);
        merge_heads(dqr, tmpN3, b, t, H, hd);
      } else {
        merge_heads(dq, tmpN3, b, t, H, hd);
      }
      linear_bwd(a->y1, params + bo->qW, tmpN3, dy, grads + bo->qW, c.modern ? NULL : grads + bo->qb, N, E, E);
      if (c.modern) {
        memset(dqr, 0, sizeof(real) * (size_t)G * t * hd);
        oc_rope_bwd(dk, dqr, G, t, hd, base);
        merge_heads(dqr, tmpN3, b, t, H, hd);
      } else {
        merge_heads(dk, tmpN3, b, t, H, hd);
      }
      linear_bwd(a->y1, params + bo->kW, tmpN3, dy, grads + bo->kW, c.modern ? NULL : grads + bo->kb, N, E, E);
      merge_heads(dv, tmpN3, b, t, H, hd);
      linear_bwd(a->y1, params + bo->vW, tmpN3, dy, grads + bo->vW, c.modern ? NULL : grads + bo->vb, N, E, E);
      /* ln1 backward into dx (holds the residual contribution) */
      if (c.modern)
        rms_bwd(a->x, params + bo->ln1g, dy, a->xn1, a->r1, N, E, dx, grads + bo->ln1g);
      else
        ln_bwd(dy, params + bo->ln1g, a->c1, a->xn1, a->r1, N, E, dx, grads + bo->ln1g, grads + bo->ln1b);
    }
    /* embeddings: tok gather bwd, then pos gather bwd, then the head's transpose bwd */
    oc_gather_bwd(ids, dx, grads + o.wte, N, E);
    if (!c.modern) oc_gather_bwd(pids, dx, grads + o.wpe, N, E);
    real* gw = grads + o.wte;
    for (int v = 0; v < V; v++)
      for (int p = 0; p < E; p++)
        gw[(size_t)v * E + p] = R((double)gw[(size_t)v * E + p] + dwteT[(size_t)p * V + v]);
    free(dyf);
    free(dwteT);
    free(dx);
    free(dh);
    free(dhid);
    free(dhid2);
    free(dy);
    free(dS);
    free(dS2);
    free(dq);
    free(dk);
    free(dkT);
    free(dv);
    free(dqr);
  }

  for (int l = 0; l < c.L; l++) {
    layer_act* a = &A[l];
    free(a->x);
    free(a->xn1);
    free(a->r1);
    free(a->y1);
    free(a->c1);
    free(a->q);
    free(a->k);
    free(a->v);
    free(a->P);
    free(a->am);
    free(a->h);
    free(a->xn2);
    free(a->r2);
    free(a->y2);
    free(a->c2);
    free(a->a1);
    free(a->a2);
    free(a->s1);
    free(a->hid);
  }
  free(x);
  free(A);
  free(pos);
  free(pids);
  free(tmpS);
  free(tmpH);
  free(tmpN);
  free(tmpN2);
  free(tmpN3);
  free(kT);
  free(yf);
  free(xnf);
  free(rf);
  free(cf);
  free(wteT);
  free(logits);
  free(probs);
  if (cerr) {
    if (err) *err = 1;
    return NAN;
  }
  return loss;
}

EXPORT double oc_loss_grad(const int* cfg, const real* params, real* grads, const int32_t* ids,
                           const int32_t* tgt, int b, int t, int* err);
EXPORT int oc_logits(const int* cfg, const real* params, const int32_t* ids, int b, int t, real* logits_out);

/* --------------------------------------------------------- optimizer */

/* clipGradNorm, src/optim/clip.ts:7-24: double sum of squares; scale when norm > max. */
EXPORT double oc_clip(real* g, size_t n, double max_norm) {
  double s = 0;
  for (size_t i = 0; i < n; i++) s += (double)g[i] * (double)g[i];
  double norm = sqrt(s);
  if (norm > max_norm && norm > 0) {
    double sc = max_norm / norm;
    for (size_t i = 0; i < n; i++) g[i] = R((double)g[i] * sc);
  }
  return norm;
}

/* Adam/AdamW step for step counter t (already incremented), src/optim/adam.ts:35-54. */
EXPORT void oc_adamw(real* p, const real* g, real* m, real* v, size_t n, double lr, double b1, double b2,
                     double eps, double wd, int t) {
  double bc1 = 1 - pow(b1, t), bc2 = 1 - pow(b2, t);
  for (size_t i = 0; i < n; i++) {
    double gi = g[i];
    m[i] = R(b1 * (double)m[i] + (1 - b1) * gi);
    v[i] = R(b2 * (double)v[i] + (1 - b2) * gi * gi);
    double mh = (double)m[i] / bc1, vh = (double)v[i] / bc2;
    p[i] = R((double)p[i] - lr * (mh / (sqrt(vh) + eps) + wd * (double)p[i]));
  }
}

/* Same update with explicit bias corrections (the GPU engine's adamw signature,
   src/infer/webgpu/autograd.ts:783-788 / ADAMW kernel :516-531). */
EXPORT void oc_adamw_bc(real* p, const real* g, real* m, real* v, size_t n, double lr, double b1, double b2,
                        double eps, double wd, double bc1, double bc2) {
  for (size_t i = 0; i < n; i++) {
    double gi = g[i];
    m[i] = R(b1 * (double)m[i] + (1 - b1) * gi);
    v[i] = R(b2 * (double)v[i] + (1 - b2) * gi * gi);
    double mh = (double)m[i] / bc1, vh = (double)v[i] / bc2;
    p[i] = R((double)p[i] - lr * (mh / (sqrt(vh) + eps) + wd * (double)p[i]));
  }
}

/* ------------------------------------------------- data-parallel pool */

typedef struct {
  const int* cfg;
  const real* params;
  real* grads;
  const int32_t* ids;
  const int32_t* tgt;
  int rows, t;
  double loss;
  int err;
} shard_job;

static void* shard_worker(void* arg) {
  shard_job* j = (shard_job*)arg;
  j->loss = oc_loss_grad(j->cfg, j->params, j->grads, j->ids, j->tgt, j->rows, j->t, &j->err);
  return NULL;
}

/* distributedBackward, scripts/train-gpt.ts:200-219: contiguous shards (shard(), :105-123), one
   replica per shard on its own thread, then the row-weighted mean of the shard gradients
   accumulated in f32 (gradScratch[j] += grads[j] * weight).  grads_out is overwritten.
   Returns the weighted loss. */
EXPORT double oc_dp_grads(const int* cfg, const real* params, real* grads_out, const int32_t* ids,
                          const int32_t* tgt, int batch, int t, int workers, int* err) {
  size_t np = oc_num_params(cfg);
  if (workers < 1) workers = 1;
  if (workers > batch) workers = batch;
  shard_job* jobs = (shard_job*)calloc(workers, sizeof(shard_job));
  pthread_t* th = (pthread_t*)calloc(workers, sizeof(pthread_t));
  int base = batch / workers, rem = batch % workers, row = 0, ns = 0;
  for (int i = 0; i < workers; i++) {
    int size = base + (i < rem ? 1 : 0);
    if (size == 0) continue;
    shard_job* j = &jobs[ns++];
    j->cfg = cfg;
    j->params = params;
    j->grads = (real*)calloc(np, sizeof(real));
    j->ids = ids + (size_t)row * t;
    j->tgt = tgt + (size_t)row * t;
    j->rows = size;
    j->t = t;
    row += size;
  }
  for (int i = 0; i < ns; i++) pthread_create(&th[i], NULL, shard_worker, &jobs[i]);
  for (int i = 0; i < ns; i++) pthread_join(th[i], NULL);
  memset(grads_out, 0, sizeof(real) * np);
  double loss = 0;
  if (err) *err = 0;
  for (int i = 0; i < ns; i++) {
    double w = (double)jobs[i].rows / batch;
    const real* g = jobs[i].grads;
    for (size_t q = 0; q < np; q++) grads_out[q] = R((double)grads_out[q] + (double)g[q] * w);
    loss += jobs[i].loss * w;
    if (jobs[i].err && err) *err = jobs[i].err;
    free(jobs[i].grads);
  }
  free(jobs);
  free(th);
  return loss;
}

/* One full CPU data-parallel training step, scripts/train-gpt.ts:234-242:
   distributedBackward -> clipGradNorm(clip) -> AdamW.step (t = step, 1-based).
   grads is scratch of num_params; returns the weighted loss, *norm_out = pre-clip norm. */
EXPORT double oc_dp_step(const int* cfg, real* params, real* grads, real* m, real* v, int step,
                         const int32_t* ids, const int32_t* tgt, int batch, int t, int workers, double lr,
                         double b1, double b2, double eps, double wd, double clip, double* norm_out, int* err) {
  size_t np = oc_num_params(cfg);
  double loss = oc_dp_grads(cfg, params, grads, ids, tgt, batch, t, workers, err);
  double norm = clip > 0 ? oc_clip(grads, np, clip) : 0;
  if (norm_out) *norm_out = norm;
  oc_adamw(params, grads, m, v, np, lr, b1, b2, eps, wd, step);
  return loss;
}

/* ---------------------------------------------------- logits / generate */

EXPORT double oc_loss_grad(const int* cfg, const real* params, real* grads, const int32_t* ids,
                           const int32_t* tgt, int b, int t, int* err) {
  return gpt_run(cfg, params, grads, ids, tgt, b, t, err, NULL);
}

/* GPT.forward logits [b*t, V] (gpt.ts:253-276). */
EXPORT int oc_logits(const int* cfg, const real* params, const int32_t* ids, int b, int t, real* logits_out) {
  int N = b * t, err = 0;
  int32_t* tg = (int32_t*)calloc(N, sizeof(int32_t));
  gpt_run(cfg, params, NULL, ids, tg, b, t, &err, logits_out);
  free(tg);
  return err;
}

/* GPT.generate + sampleFromLogits, src/models/gpt.ts:291-341.  topk <= 0 disables top-k.
   out receives prompt followed by the sampled ids; returns the number written. */
EXPORT int oc_generate(const int* cfg, const real* params, const int32_t* prompt, int n_prompt, int max_new,
                       double temperature, int topk, uint32_t* rng_state, int32_t* out) {
  gcfg c = read_cfg(cfg);
  int n = n_prompt;
  memcpy(out, prompt, sizeof(int32_t) * n_prompt);
  real* logits = ALLOC((size_t)c.T * c.V);
  real* last = ALLOC(c.V);
  real* sorted = ALLOC(c.V);
  real* probs = ALLOC(c.V);
  for (int step = 0; step < max_new; step++) {
    int start = n > c.T ? n - c.T : 0;
    int t = n - start;
    oc_logits(cfg, params, out + start, 1, t, logits);
    const real* row = logits + (size_t)(t - 1) * c.V;
    for (int j = 0; j < c.V; j++) last[j] = R((double)row[j] / temperature);
    if (topk > 0 && topk < c.V) {
      memcpy(sorted, last, sizeof(real) * c.V);
      /* threshold = topk-th largest */
      for (int a = 0; a < topk; a++) {
        int bi = a;
        for (int q = a + 1; q < c.V; q++)
          if (sorted[q] > sorted[bi]) bi = q;
        real tmp = sorted[a];
        sorted[a] = sorted[bi];
        sorted[bi] = tmp;
      }
      real thr = sorted[topk - 1];
      for (int j = 0; j < c.V; j++)
        if (last[j] < thr) last[j] = -INFINITY;
    }
    double mx = -INFINITY;
    for (int j = 0; j < c.V; j++)
      if (last[j] > mx) mx = last[j];
    double sum = 0;
    for (int j = 0; j < c.V; j++) {
      double e = exp((double)last[j] - mx);
      probs[j] = R(e);
      sum += e;
    }
    double r = oc_rng_next(rng_state) * sum;
    int next = c.V - 1;
    for (int j = 0; j < c.V; j++) {
      r -= probs[j];
      if (r <= 0) {
        next = j;
        break;
      }
    }
    out[n++] = next;
  }
  free(logits);
  free(last);
  free(sorted);
  free(probs);
  return n;
}
