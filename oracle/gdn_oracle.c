/*
 * gdn_oracle.c -- CPU restatement of the reference's GDN layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke
 * check in __graft_entry__.py and the CPU-baseline leg of bench.py load it.
 * No product code links, imports or calls it.
 *
 * Parity status: PARITY UNPINNED against the reference.  The reference's
 * arithmetic runs in closed CANN 9.1.0 aclnn operators (aclnnFusedGdnGating,
 * aclnnRmsNorm, aclnnRecurrentGatedDeltaRule, aclnnChunkGatedDeltaRuleFwdH,
 * aclnnChunkFwdO, aclnnSilu, aclnnMul, aclnnMatmul) and in Triton-Ascend AOT
 * binaries that are not in the repository, and its own tests only pin
 * self-consistency (flat tail == batched tail == per-sequence tail).  This
 * restatement follows the reference's call sites operator by operator
 * (citations below, P = native/src/qwen38_geometry_normalized_gdn_provider.cpp)
 * and the published gated-delta-rule algorithm; tests cross-check it against
 * the independent PyTorch restatement in transformers 5.5.0
 * (models/qwen3_next/modeling_qwen3_next.py: torch_recurrent_gated_delta_rule,
 * torch_chunk_gated_delta_rule, Qwen3NextRMSNormGated) and commit golden
 * vectors generated from it under tests/golden/.
 *
 * Layouts: see include/gdn_b200.h.  Recurrent state is [Hv][Dv][Dk]: the
 * reference stores the recurrent-op layout and transposes it around the chunk
 * operator (P:1750-1753, 1831-1834).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------- bf16 -- */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* Round to nearest even, as the reference does for its bf16 constant
 * (P:1046-1051). */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) {
    return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  }
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline double round_bf16(double x) {
  return (double)bf16_to_f32(f32_to_bf16((float)x));
}

ORACLE_EXPORT void gdn_oracle_f32_to_bf16(const float* in, uint16_t* out,
                                          int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(in[i]);
}

ORACLE_EXPORT void gdn_oracle_bf16_to_f32(const uint16_t* in, float* out,
                                          int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

/* -------------------------------------------------------------- gating -- */

/* aclnnFusedGdnGating(A_log, a, b, dt_bias, beta=1.0, threshold=20.0)
 * (P:3310-3339): g = -exp(A_log) * softplus(a + dt_bias), g stored f32;
 * beta = sigmoid(b), stored bf16. */
ORACLE_EXPORT void gdn_oracle_gating(const uint16_t* a, const uint16_t* b,
                                     const float* A_log, const float* dt_bias,
                                     int64_t tokens, int32_t hv, float* g_out,
                                     uint16_t* beta_out) {
  for (int64_t t = 0; t < tokens; ++t) {
    for (int32_t h = 0; h < hv; ++h) {
      const int64_t i = t * hv + h;
      const double x = (double)bf16_to_f32(a[i]) + (double)dt_bias[h];
      const double sp = x > 20.0 ? x : log1p(exp(x));
      g_out[i] = (float)(-exp((double)A_log[h]) * sp);
      const double bb = (double)bf16_to_f32(b[i]);
      beta_out[i] = f32_to_bf16((float)(1.0 / (1.0 + exp(-bb))));
    }
  }
}

/* ------------------------------------------------------------- L2 norm -- */

/* q/k L2 normalisation done as RmsNorm with gamma = bf16(D^-1/2)
 * (P:1043-1057) and eps = 1e-6 / D (P:3301-3308): per row of D,
 * out = bf16(x * rsqrt(mean(x^2) + eps/D) * gamma). */
ORACLE_EXPORT void gdn_oracle_l2norm(const uint16_t* x, int64_t rows,
                                     int32_t d, uint16_t* out) {
  const double gamma = (double)bf16_to_f32(f32_to_bf16(1.0f / sqrtf((float)d)));
  const double eps = 1.0e-6 / (double)d;
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* row = x + r * d;
    double ss = 0.0;
    for (int32_t j = 0; j < d; ++j) {
      const double v = bf16_to_f32(row[j]);
      ss += v * v;
    }
    const double rstd = 1.0 / sqrt(ss / (double)d + eps);
    for (int32_t j = 0; j < d; ++j) {
      out[r * d + j] = f32_to_bf16((float)((double)bf16_to_f32(row[j]) * rstd * gamma));
    }
  }
}

/* ----------------------------------------------------- recurrent rule --- */

/* Token-serial gated delta rule for one (sequence, v-head), state in double.
 * aclnnRecurrentGatedDeltaRule semantics (P:1308-1369, 3387-3469), scale
 * D^-1/2 (P:1362, 3459):
 *   S <- exp(g_t) S;  kv = S k_t;  d = beta_t (v_t - kv);  S <- S + d k_t^T;
 *   o_t = scale * S q_t
 * with S[i][j] indexed [value i][key j]. */
static void recurrent_head(const uint16_t* qn, const uint16_t* kn,
                           const uint16_t* v, const float* g,
                           const uint16_t* beta, int64_t tokens, int32_t hk,
                           int32_t hv, int32_t d, int32_t h, float* state,
                           uint16_t* o) {
  const int32_t group = hv / hk;
  const int32_t kh = h / group;
  const double scale = 1.0 / sqrt((double)d);
  double* s = (double*)malloc(sizeof(double) * (size_t)d * d);
  double* kk = (double*)malloc(sizeof(double) * (size_t)d);
  double* qq = (double*)malloc(sizeof(double) * (size_t)d);
  for (int64_t i = 0; i < (int64_t)d * d; ++i) s[i] = state[i];
  for (int64_t t = 0; t < tokens; ++t) {
    const uint16_t* qr = qn + (t * hk + kh) * d;
    const uint16_t* kr = kn + (t * hk + kh) * d;
    const uint16_t* vr = v + (t * hv + h) * d;
    for (int32_t j = 0; j < d; ++j) {
      kk[j] = bf16_to_f32(kr[j]);
      qq[j] = bf16_to_f32(qr[j]);
    }
    const double decay = exp((double)g[t * hv + h]);
    const double bt = bf16_to_f32(beta[t * hv + h]);
    for (int32_t i = 0; i < d; ++i) {
      double* row = s + (int64_t)i * d;
      double kv = 0.0;
      for (int32_t j = 0; j < d; ++j) {
        row[j] *= decay;
        kv += row[j] * kk[j];
      }
      const double delta = bt * ((double)bf16_to_f32(vr[i]) - kv);
      double acc = 0.0;
      for (int32_t j = 0; j < d; ++j) {
        row[j] += delta * kk[j];
        acc += row[j] * qq[j];
      }
      o[(t * hv + h) * d + i] = f32_to_bf16((float)(scale * acc));
    }
  }
  for (int64_t i = 0; i < (int64_t)d * d; ++i) state[i] = (float)s[i];
  free(s);
  free(kk);
  free(qq);
}

/* ------------------------------------------------------- chunked rule --- */

/* Chunked form of the same rule, chunk C = 64, following the reference's
 * chain (P:1696-1830): cumsum of g inside the chunk (P:1696-1699),
 * A = beta_i (K K^T)_ij exp(G_i - G_j) strictly lower (P:1706-1711),
 * T = (I + A)^-1 (16x16 solve + merge, P:1712-1725),
 * W = T (beta exp(G) K), U = T (beta V) (P:1726-1734),
 * per chunk: v_new = U - W S;  O = scale [(Q exp(G)) S + (Q K^T . Gamma) v_new];
 * S <- exp(G_C) S + (K exp(G_C - G))^T v_new  (ChunkGatedDeltaRuleFwdH +
 * ChunkFwdO, P:1755-1830).  Here S is [key][value] as in the chunk op.
 * rounding = 0: every intermediate in double.
 * rounding = 1: bf16 at the points where the reference chain stores bf16
 * tensors: T (merge output, P:1719-1725), W and U (P:1726-1734), the state
 * snapshot h used by ChunkFwdO and v_new (P:1755-1830). */
static void chunked_head(const uint16_t* qn, const uint16_t* kn,
                         const uint16_t* v, const float* g,
                         const uint16_t* beta, int64_t tokens, int32_t hk,
                         int32_t hv, int32_t d, int32_t h, float* state,
                         uint16_t* o, int rounding) {
  enum { C = 64 };
  const int32_t group = hv / hk;
  const int32_t kh = h / group;
  const double scale = 1.0 / sqrt((double)d);
  const size_t dd = (size_t)d * d;
  double* s = (double*)malloc(sizeof(double) * dd);       /* [key][value] */
  double* sop = (double*)malloc(sizeof(double) * dd);     /* operand copy */
  double* K = (double*)malloc(sizeof(double) * C * d);
  double* Q = (double*)malloc(sizeof(double) * C * d);
  double* V = (double*)malloc(sizeof(double) * C * d);
  double* W = (double*)malloc(sizeof(double) * C * d);
  double* U = (double*)malloc(sizeof(double) * C * d);
  double* vn = (double*)malloc(sizeof(double) * C * d);
  double* A = (double*)malloc(sizeof(double) * C * C);
  double* Ti = (double*)malloc(sizeof(double) * C * C);
  double G[C], B[C];
  for (int32_t i = 0; i < d; ++i)
    for (int32_t j = 0; j < d; ++j) s[(int64_t)j * d + i] = state[(int64_t)i * d + j];

  for (int64_t c0 = 0; c0 < tokens; c0 += C) {
    const int32_t n = (int32_t)((tokens - c0) < C ? (tokens - c0) : C);
    double run = 0.0;
    for (int32_t t = 0; t < n; ++t) {
      const int64_t tt = c0 + t;
      run += (double)g[tt * hv + h];
      G[t] = run;
      B[t] = bf16_to_f32(beta[tt * hv + h]);
      for (int32_t j = 0; j < d; ++j) {
        K[t * d + j] = bf16_to_f32(kn[(tt * hk + kh) * d + j]);
        Q[t * d + j] = bf16_to_f32(qn[(tt * hk + kh) * d + j]);
        V[t * d + j] = bf16_to_f32(v[(tt * hv + h) * d + j]);
      }
    }
    /* A, strictly lower */
    for (int32_t i = 0; i < n; ++i) {
      for (int32_t j = 0; j < n; ++j) {
        double val = 0.0;
        if (j < i) {
          double dot = 0.0;
          for (int32_t x = 0; x < d; ++x) dot += K[i * d + x] * K[j * d + x];
          val = B[i] * dot * exp(G[i] - G[j]);
        }
        A[i * C + j] = val;
      }
    }
    /* T = (I + A)^-1 by forward substitution */
    for (int32_t i = 0; i < n; ++i) {
      for (int32_t j = 0; j < n; ++j) {
        double val = (i == j) ? 1.0 : 0.0;
        if (j < i) {
          double acc = 0.0;
          for (int32_t m = j; m < i; ++m) acc += A[i * C + m] * Ti[m * C + j];
          val = -acc;
        }
        Ti[i * C + j] = val;
      }
    }
    if (rounding)
      for (int32_t i = 0; i < n * C; ++i) Ti[i] = round_bf16(Ti[i]);
    /* W, U */
    for (int32_t i = 0; i < n; ++i) {
      for (int32_t x = 0; x < d; ++x) {
        double w = 0.0, u = 0.0;
        for (int32_t j = 0; j <= i; ++j) {
          w += Ti[i * C + j] * B[j] * exp(G[j]) * K[j * d + x];
          u += Ti[i * C + j] * B[j] * V[j * d + x];
        }
        W[i * d + x] = rounding ? round_bf16(w) : w;
        U[i * d + x] = rounding ? round_bf16(u) : u;
      }
    }
    for (size_t i = 0; i < dd; ++i) sop[i] = rounding ? round_bf16(s[i]) : s[i];
    /* v_new = U - W S */
    for (int32_t i = 0; i < n; ++i) {
      for (int32_t y = 0; y < d; ++y) {
        double acc = 0.0;
        for (int32_t x = 0; x < d; ++x) acc += W[i * d + x] * sop[(int64_t)x * d + y];
        const double val = U[i * d + y] - acc;
        vn[i * d + y] = rounding ? round_bf16(val) : val;
      }
    }
    /* output; A is reused for the masked, decayed Q K^T */
    for (int32_t i = 0; i < n; ++i) {
      for (int32_t j = 0; j <= i; ++j) {
        double qk = 0.0;
        for (int32_t x = 0; x < d; ++x) qk += Q[i * d + x] * K[j * d + x];
        A[i * C + j] = qk * exp(G[i] - G[j]);
      }
    }
    for (int32_t i = 0; i < n; ++i) {
      const double eg = exp(G[i]);
      for (int32_t y = 0; y < d; ++y) {
        double inter = 0.0;
        for (int32_t x = 0; x < d; ++x) inter += Q[i * d + x] * sop[(int64_t)x * d + y];
        double intra = 0.0;
        for (int32_t j = 0; j <= i; ++j) intra += A[i * C + j] * vn[j * d + y];
        o[((c0 + i) * hv + h) * d + y] = f32_to_bf16((float)(scale * (eg * inter + intra)));
      }
    }
    /* state */
    const double glast = G[n - 1];
    const double dl = exp(glast);
    for (int32_t x = 0; x < d; ++x) {
      for (int32_t y = 0; y < d; ++y) {
        double acc = 0.0;
        for (int32_t j = 0; j < n; ++j) acc += K[j * d + x] * exp(glast - G[j]) * vn[j * d + y];
        s[(int64_t)x * d + y] = dl * s[(int64_t)x * d + y] + acc;
      }
    }
  }
  for (int32_t i = 0; i < d; ++i)
    for (int32_t j = 0; j < d; ++j) state[(int64_t)i * d + j] = (float)s[(int64_t)j * d + i];
  free(s); free(sop); free(K); free(Q); free(V); free(W); free(U); free(vn);
  free(A); free(Ti);
}

/* core_mode: 0 = recurrent (ground truth), 1 = chunked exact,
 * 2 = chunked with the reference chain's bf16 rounding points. */
ORACLE_EXPORT void gdn_oracle_core(const uint16_t* qn, const uint16_t* kn,
                                   const uint16_t* v, const float* g,
                                   const uint16_t* beta, float* state,
                                   uint16_t* o, const int32_t* cu_seqlens,
                                   int32_t num_seqs, int32_t hk, int32_t hv,
                                   int32_t d, int32_t core_mode) {
  const int64_t work = (int64_t)num_seqs * hv;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t w = 0; w < work; ++w) {
    const int32_t sidx = (int32_t)(w / hv);
    const int32_t h = (int32_t)(w % hv);
    const int64_t t0 = cu_seqlens[sidx];
    const int64_t tl = cu_seqlens[sidx + 1] - t0;
    float* st = state + ((int64_t)sidx * hv + h) * d * d;
    if (tl <= 0) continue;
    if (core_mode == 0) {
      recurrent_head(qn + t0 * hk * d, kn + t0 * hk * d, v + t0 * hv * d,
                     g + t0 * hv, beta + t0 * hv, tl, hk, hv, d, h, st,
                     o + t0 * hv * d);
    } else {
      chunked_head(qn + t0 * hk * d, kn + t0 * hk * d, v + t0 * hv * d,
                   g + t0 * hv, beta + t0 * hv, tl, hk, hv, d, h, st,
                   o + t0 * hv * d, core_mode == 2);
    }
  }
}

/* ---------------------------------------------------------- output tail -- */

/* Gated RMSNorm prologue of the tail (P:1434-1494, 3498-3540):
 * mode 0 ("reference rounding"): n = bf16(o*rstd*gamma) (aclnnRmsNorm, eps),
 *   s = bf16(SiLU(z)) (aclnnSilu), gated = bf16(n*s) (aclnnMul);
 * mode 1 ("fused"): fp32 throughout, one bf16 cast at the end. */
ORACLE_EXPORT void gdn_oracle_tail_prologue(const uint16_t* o, const uint16_t* z,
                                            const uint16_t* gamma, int64_t rows,
                                            int32_t hv, int32_t d, float eps,
                                            int32_t mode, uint16_t* gated) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows * hv; ++r) {
    const uint16_t* orow = o + r * d;
    const uint16_t* zrow = z + r * d;
    double ss = 0.0;
    for (int32_t j = 0; j < d; ++j) {
      const double x = bf16_to_f32(orow[j]);
      ss += x * x;
    }
    const double rstd = 1.0 / sqrt(ss / (double)d + (double)eps);
    for (int32_t j = 0; j < d; ++j) {
      const double x = bf16_to_f32(orow[j]);
      const double zz = bf16_to_f32(zrow[j]);
      double nrm = x * rstd * (double)bf16_to_f32(gamma[j]);
      double sl = zz / (1.0 + exp(-zz));
      if (mode == 0) {
        nrm = round_bf16(nrm);
        sl = round_bf16(sl);
      }
      gated[r * d + j] = f32_to_bf16((float)(nrm * sl));
    }
  }
}

/* out[m][n] = bf16( sum_k a[m][k] * w[n][k] ), fp32 products of bf16
 * operands accumulated in double (FlatMatmulSharedWeight, P:1260-1274). */
ORACLE_EXPORT void gdn_oracle_gemm_bf16(const uint16_t* a, const uint16_t* w,
                                        int64_t m, int64_t n, int64_t k,
                                        uint16_t* out) {
  float* wf = (float*)malloc(sizeof(float) * (size_t)(n * k));
  for (int64_t i = 0; i < n * k; ++i) wf[i] = bf16_to_f32(w[i]);
#pragma omp parallel
  {
    float* af = (float*)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < m; ++r) {
      for (int64_t x = 0; x < k; ++x) af[x] = bf16_to_f32(a[r * k + x]);
      for (int64_t c = 0; c < n; ++c) {
        const float* wr = wf + c * k;
        float lanes[16] = {0};
        int64_t x = 0;
        for (; x + 16 <= k; x += 16)
          for (int l = 0; l < 16; ++l) lanes[l] += af[x + l] * wr[x + l];
        double acc = 0.0;
        for (int l = 0; l < 16; ++l) acc += lanes[l];
        for (; x < k; ++x) acc += (double)af[x] * wr[x];
        out[r * n + c] = f32_to_bf16((float)acc);
      }
    }
    free(af);
  }
  free(wf);
}

ORACLE_EXPORT void gdn_oracle_output_tail(const uint16_t* o, const uint16_t* z,
                                          const uint16_t* gamma,
                                          const uint16_t* w, int64_t rows,
                                          int32_t hv, int32_t d, int32_t hidden,
                                          float eps, int32_t mode,
                                          uint16_t* gated_out, uint16_t* out) {
  uint16_t* gated = gated_out;
  if (gated == NULL) gated = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(rows * hv * d));
  gdn_oracle_tail_prologue(o, z, gamma, rows, hv, d, eps, mode, gated);
  gdn_oracle_gemm_bf16(gated, w, rows, hidden, (int64_t)hv * d, out);
  if (gated_out == NULL) free(gated);
}

/* --------------------------------------------------------------- layer -- */

/* Whole post-projection layer for packed sequences: gating, q/k L2-norm,
 * core (core_mode as in gdn_oracle_core), output tail (reference rounding).
 * o_out / gated_out may be NULL. */
ORACLE_EXPORT void gdn_oracle_layer(const uint16_t* q, const uint16_t* k,
                                    const uint16_t* v, const uint16_t* a,
                                    const uint16_t* b, const uint16_t* z,
                                    const float* A_log, const float* dt_bias,
                                    const uint16_t* gamma, const uint16_t* w,
                                    float* state, uint16_t* out,
                                    const int32_t* cu_seqlens, int32_t num_seqs,
                                    int32_t hk, int32_t hv, int32_t d,
                                    int32_t hidden, int32_t core_mode,
                                    uint16_t* o_out, uint16_t* gated_out) {
  const int64_t tokens = cu_seqlens[num_seqs];
  float* g = (float*)malloc(sizeof(float) * (size_t)(tokens * hv));
  uint16_t* beta = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(tokens * hv));
  uint16_t* qn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(tokens * hk * d));
  uint16_t* kn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(tokens * hk * d));
  uint16_t* o = o_out ? o_out : (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(tokens * hv * d));
  gdn_oracle_gating(a, b, A_log, dt_bias, tokens, hv, g, beta);
  gdn_oracle_l2norm(q, tokens * hk, d, qn);
  gdn_oracle_l2norm(k, tokens * hk, d, kn);
  gdn_oracle_core(qn, kn, v, g, beta, state, o, cu_seqlens, num_seqs, hk, hv, d,
                  core_mode);
  gdn_oracle_output_tail(o, z, gamma, w, tokens, hv, d, hidden, 1.0e-6f, 0,
                         gated_out, out);
  free(g); free(beta); free(qn); free(kn);
  if (o_out == NULL) free(o);
}

ORACLE_EXPORT int32_t gdn_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* -------------------------------------------------- input side of the layer -- */

/* Depthwise causal conv1d over the projected qkv channels, width 4 (history
 * 3), SiLU, and the conv-state update, per packed sequence: the reference's
 * aclnnCausalConv1d call (P:3132-3179; weight input 5 [4, channels], state
 * region gdn.conv bf16 [S, 3, channels], zero history when the submission has
 * no context, P:3163-3171), with the activation of Qwen3-Next's
 * causal_conv1d_fn(activation="silu"):
 *   out[t][c] = bf16( silu( sum_{k=0..3} w[k][c] * x[t-3+k][c] ) ),
 * rows before the sequence taken from its state (zero when use_state is 0).
 * The sum is accumulated in float in tap order (w0 x0, then fmaf of taps 1,
 * 2, 3) and silu(y) = y / (1 + exp(-y)).  Afterwards the state of each
 * sequence holds the last three rows of [history; x]. */
ORACLE_EXPORT void gdn_oracle_causal_conv1d(const uint16_t* x, const uint16_t* w,
                                            uint16_t* state, const int32_t* cu, int32_t nseq,
                                            int64_t channels, int32_t use_state,
                                            uint16_t* out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int32_t s = 0; s < nseq; ++s) {
    for (int64_t c = 0; c < channels; ++c) {
      float h[3];
      for (int i = 0; i < 3; ++i)
        h[i] = use_state ? bf16_to_f32(state[((int64_t)s * 3 + i) * channels + c]) : 0.0f;
      const float w0 = bf16_to_f32(w[c]), w1 = bf16_to_f32(w[channels + c]);
      const float w2 = bf16_to_f32(w[2 * channels + c]), w3 = bf16_to_f32(w[3 * channels + c]);
      for (int64_t t = cu[s]; t < cu[s + 1]; ++t) {
        const float xt = bf16_to_f32(x[t * channels + c]);
        float acc = w0 * h[0];
        acc = fmaf(w1, h[1], acc);
        acc = fmaf(w2, h[2], acc);
        acc = fmaf(w3, xt, acc);
        out[t * channels + c] = f32_to_bf16(acc / (1.0f + expf(-acc)));
        h[0] = h[1];
        h[1] = h[2];
        h[2] = xt;
      }
      for (int i = 0; i < 3; ++i)
        state[((int64_t)s * 3 + i) * channels + c] = f32_to_bf16(h[i]);
    }
  }
}

/* ------------------------------------------------------ synthetic inputs -- */

/* Seeded benchmark inputs, the same generator as the product library's
 * gdn_b200_fill_synthetic (so the CPU baseline never needs that library):
 * a SplitMix64 counter keyed by (seed, tensor id) gives two 53-bit uniforms
 * per element; distribution 0 = normal p0 + p1 * N(0,1) (Box-Muller,
 * cosine branch), 1 = uniform [p0, p1), 2 = log of uniform (p0, p1].
 * dtype 1 = bf16 (round to nearest even), 2 = f32.  Computed in double with
 * the C library's sqrt/log/cos and no fused multiply-add (ISO C mode,
 * -ffp-contract=off), so both builds give the same bits (a CPU test compares
 * them). */
static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

ORACLE_EXPORT int32_t gdn_oracle_fill_synthetic(uint64_t seed, uint64_t tensor_id,
                                                uint64_t count, int32_t distribution,
                                                float p0, float p1, int32_t out_dtype,
                                                void* out) {
  if ((out == NULL && count > 0) || distribution < 0 || distribution > 2 ||
      (out_dtype != 1 && out_dtype != 2))
    return 1;
  const uint64_t key = splitmix64(splitmix64(seed) ^ (tensor_id * 0xD1B54A32D192ED03ull));
  const double two_pi = 6.283185307179586476925286766559;
  /* The product evaluates p0 + p1 * sqrt(..) * cos(..) left to right in
   * double, and (p1 - p0) in float: the same order here. */
  const double p0d = (double)p0, p1d = (double)p1, span = (double)(float)(p1 - p0);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)count; ++i) {
    const uint64_t r1 = splitmix64(key + 2 * (uint64_t)i);
    const uint64_t r2 = splitmix64(key + 2 * (uint64_t)i + 1);
    const double u1 = ((double)(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(r2 >> 11) * (1.0 / 9007199254740992.0);
    double val;
    if (distribution == 0) {
      const double scaled = p1d * sqrt(-2.0 * log(u1));
      val = p0d + scaled * cos(two_pi * u2);
    } else if (distribution == 1) {
      val = p0d + span * u2;
    } else {
      val = log(p0d + span * u1);
    }
    if (out_dtype == 1)
      ((uint16_t*)out)[i] = f32_to_bf16((float)val);
    else
      ((float*)out)[i] = (float)val;
  }
  return 0;
}
