// ORACLE — test infrastructure only. Never linked into, loaded by, or called
// from the product library (librnet_b200.so). Only tests/, the smoke check
// and bench.py's cpu_baseline leg may use it, and only as the checker.
//
// Scalar C++17 + OpenMP restatement of the reference's fp32 layer math
// (KristianPilatovich/resonance-net). Storage is fp32 exactly where the
// reference stores fp32; dot products / reductions accumulate in double.
// Each function cites the reference file:line whose behaviour it restates.
//
// Build: see oracle/Makefile (liboracle.so, -O3 -fopenmp).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// Byte-identical to the reference's ModelConfig (include/config.h:7-18): the
// first 40 bytes of a checkpoint.
struct OrcConfig {
  int d_model, n_layers, d_ff, n_heads, gru_dim, n_slots, slot_top_k, vocab_size, seq_len;
  float rms_eps;
};

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"

namespace {

// C[m,n] (+)= sum_k A[m*K+k] * B[n*K+k]   (both K-contiguous), double accumulate.
void gemm_nt(int M, int N, int K, const float* A, const float* B, float* C, bool accumulate) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < M; ++m) {
    const float* a = A + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const float* b = B + (size_t)n * K;
      double acc = 0.0;
#pragma omp simd reduction(+ : acc)
      for (int k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
      float* c = C + (size_t)m * N + n;
      *c = accumulate ? (float)((double)*c + acc) : (float)acc;
    }
  }
}

// out[c*R + r] = in[r*Cn + c]
std::vector<float> transpose(const float* in, int R, int Cn) {
  std::vector<float> out((size_t)R * Cn);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < R; ++r)
    for (int c = 0; c < Cn; ++c) out[(size_t)c * R + r] = in[(size_t)r * Cn + c];
  return out;
}

// y = x W^T with W [out, in] row-major (cuBLAS OP_T calls of the reference).
void linear(const float* x, const float* W, float* y, int N, int out, int in, bool acc = false) {
  gemm_nt(N, out, in, x, W, y, acc);
}

// dx (+)= dy W, W [out, in]: dx[n,i] = sum_o dy[n,o] W[o,i].
void linear_dx(const float* dy, const float* W, float* dx, int N, int out, int in, bool acc) {
  std::vector<float> Wt = transpose(W, out, in);  // [in, out]
  gemm_nt(N, in, out, dy, Wt.data(), dx, acc);
}

// dW[o,i] += sum_n dy[n,o] x[n,i].
void linear_dw(const float* dy, const float* x, float* dW, int N, int out, int in) {
  std::vector<float> dyT = transpose(dy, N, out);  // [out, N]
  std::vector<float> xT = transpose(x, N, in);     // [in, N]
  gemm_nt(out, in, N, dyT.data(), xT.data(), dW, true);
}

inline float sigmoid_ref(float v) { return 1.0f / (1.0f + std::exp(-v)); }

}  // namespace

extern "C" {

// ---------------------------------------------------------------- RMSNorm
// src/rms_norm.cu:8-40 — rinv = rsqrt(sum(x^2)/D + eps); y = x * rinv * w.
void orc_rms_norm_fwd(const float* x, const float* w, float* y, float* rinv, int N, int D,
                      float eps) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; ++r) {
    const float* xr = x + (size_t)r * D;
    double ss = 0.0;
    for (int i = 0; i < D; ++i) ss += (double)xr[i] * xr[i];
    const float ri = (float)(1.0 / std::sqrt(ss / D + (double)eps));
    if (rinv) rinv[r] = ri;
    for (int i = 0; i < D; ++i) y[(size_t)r * D + i] = xr[i] * ri * w[i];
  }
}

// src/rms_norm.cu:52-83 — dx = rinv*(dy*w - x*rinv*dot/D) (overwrite),
// dw += dy * x * rinv (accumulate over rows).
void orc_rms_norm_bwd(const float* dy, const float* x, const float* w, const float* rinv,
                      float* dx, float* dw, int N, int D) {
  std::vector<double> dwacc((size_t)D, 0.0);
#pragma omp parallel
  {
    std::vector<double> local((size_t)D, 0.0);
#pragma omp for schedule(static)
    for (int r = 0; r < N; ++r) {
      const float* dyr = dy + (size_t)r * D;
      const float* xr = x + (size_t)r * D;
      const float ri = rinv[r];
      double dot = 0.0;
      for (int i = 0; i < D; ++i) dot += (double)dyr[i] * w[i] * xr[i] * ri;
      const double sdot = dot / D;
      for (int i = 0; i < D; ++i) {
        const double nx = (double)xr[i] * ri;
        dx[(size_t)r * D + i] = (float)(ri * ((double)dyr[i] * w[i] - nx * sdot));
        local[i] += (double)dyr[i] * nx;
      }
    }
#pragma omp critical
    for (int i = 0; i < D; ++i) dwacc[i] += local[i];
  }
  for (int i = 0; i < D; ++i) dw[i] = (float)((double)dw[i] + dwacc[i]);
}

// ---------------------------------------------------------------- causal conv
// src/causal_conv.cu:9-30 depthwise causal conv (zero left pad within each
// sequence), :45-80 forward: c3/c7/c15, S = c3 + c7 + c15 stored over c3,
// y = S mix^T. conv_buf layout [3, N, D] = {S, c7, c15}.
void orc_conv_fwd(const float* x, float* y, const float* w3, const float* w7, const float* w15,
                  const float* mix, float* conv_buf, int B, int T, int D) {
  const size_t NE = (size_t)B * T * D;
  float* c3 = conv_buf;
  float* c7 = conv_buf + NE;
  float* c15 = conv_buf + 2 * NE;
  const float* ws[3] = {w3, w7, w15};
  float* cs[3] = {c3, c7, c15};
  const int ks[3] = {3, 7, 15};
  for (int s = 0; s < 3; ++s) {
    const int K = ks[s];
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
      for (int t = 0; t < T; ++t)
        for (int d = 0; d < D; ++d) {
          double acc = 0.0;
          for (int k = 0; k < K; ++k) {
            const int st = t - (K - 1) + k;
            if (st >= 0) acc += (double)x[((size_t)b * T + st) * D + d] * ws[s][k * D + d];
          }
          cs[s][((size_t)b * T + t) * D + d] = (float)acc;
        }
  }
  for (size_t i = 0; i < NE; ++i) c3[i] = c3[i] + c7[i] + c15[i];  // sum3_kernel, in place
  linear(c3, mix, y, B * T, D, D);
}

// src/causal_conv.cu:85-190. dS = dy mix; dmix += Sm^T dy where Sm is the
// re-summed buffer (quirk=1: S + c7 + c15 exactly as the reference's sum3 over
// the cached buffer, causal_conv.cu:155-168; quirk=0: S); dx += sum_K conv_K^T(dS);
// dw_K[k,d] += sum_{b,t} x[t-(K-1)+k] dS[t].
void orc_conv_bwd(const float* dy, const float* x, const float* w3, const float* w7,
                  const float* w15, const float* mix, const float* conv_buf, float* dx,
                  float* dw3, float* dw7, float* dw15, float* dmix, int B, int T, int D,
                  int quirk) {
  const int N = B * T;
  const size_t NE = (size_t)N * D;
  std::vector<float> dS(NE);
  linear_dx(dy, mix, dS.data(), N, D, D, false);
  std::vector<float> Sm(NE);
  for (size_t i = 0; i < NE; ++i)
    Sm[i] = quirk ? conv_buf[i] + conv_buf[NE + i] + conv_buf[2 * NE + i] : conv_buf[i];
  // dmix[i,j] += sum_n dy[n,i] * Sm[n,j]   (mix is [out=i, in=j])
  linear_dw(dy, Sm.data(), dmix, N, D, D);
  const float* ws[3] = {w3, w7, w15};
  float* dws[3] = {dw3, dw7, dw15};
  const int ks[3] = {3, 7, 15};
  std::vector<double> dxacc(NE, 0.0);
  for (int s = 0; s < 3; ++s) {
    const int K = ks[s];
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
      for (int t = 0; t < T; ++t)
        for (int d = 0; d < D; ++d) {
          double acc = 0.0;
          for (int k = 0; k < K; ++k) {
            const int ot = t + (K - 1) - k;
            if (ot < T) acc += (double)ws[s][k * D + d] * dS[((size_t)b * T + ot) * D + d];
          }
          dxacc[((size_t)b * T + t) * D + d] += acc;
        }
#pragma omp parallel for schedule(static)
    for (int kd = 0; kd < K * D; ++kd) {
      const int k = kd / D, d = kd % D;
      double acc = 0.0;
      for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) {
          const int st = t - (K - 1) + k;
          if (st >= 0) acc += (double)x[((size_t)b * T + st) * D + d] * dS[((size_t)b * T + t) * D + d];
        }
      dws[s][kd] = (float)((double)dws[s][kd] + acc);
    }
  }
  for (size_t i = 0; i < NE; ++i) dx[i] = (float)((double)dx[i] + dxacc[i]);
}

// ---------------------------------------------------------------- MinGRU
// src/min_gru.cu:20-84: pz = x Wz^T, ph = x Wh^T; z = sigmoid(pz+bz),
// h~ = ph + bh, h_t = (1-z) h_{t-1} + z h~, h_{-1} = 0 per sequence; y = h.
void orc_gru_fwd(const float* x, float* y, const float* Wz, const float* Wh, const float* bz,
                 const float* bh, float* zc, float* hc, int B, int T, int D) {
  const int N = B * T;
  std::vector<float> pz((size_t)N * D), ph((size_t)N * D);
  linear(x, Wz, pz.data(), N, D, D);
  linear(x, Wh, ph.data(), N, D, D);
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int d = 0; d < D; ++d) {
      float h = 0.0f;
      for (int t = 0; t < T; ++t) {
        const size_t i = ((size_t)b * T + t) * D + d;
        const float z = sigmoid_ref(pz[i] + bz[d]);
        const float ht = ph[i] + bh[d];
        h = (1.0f - z) * h + z * ht;
        zc[i] = z;
        hc[i] = h;
        y[i] = h;
      }
    }
}

// src/min_gru.cu:87-191: recompute h~; reverse scan dh += dy;
// dz = dh (h~ - h_prev) z (1-z); dh~ = dh z; dh *= (1-z);
// dx += dz Wz + dh~ Wh; dWz += dz^T x; dWh += dh~^T x; dbz += sum dz; dbh += sum dh~.
void orc_gru_bwd(const float* dy, const float* x, const float* Wz, const float* Wh,
                 const float* bz, const float* bh, const float* zc, const float* hc, float* dx,
                 float* dWz, float* dWh, float* dbz, float* dbh, int B, int T, int D) {
  (void)bz;
  const int N = B * T;
  const size_t NE = (size_t)N * D;
  std::vector<float> ht(NE), dz(NE), dht(NE);
  linear(x, Wh, ht.data(), N, D, D);
  for (size_t i = 0; i < NE; ++i) ht[i] += bh[i % D];
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int d = 0; d < D; ++d) {
      float dh = 0.0f;
      for (int t = T - 1; t >= 0; --t) {
        const size_t i = ((size_t)b * T + t) * D + d;
        dh += dy[i];
        const float z = zc[i];
        const float hp = t > 0 ? hc[i - D] : 0.0f;
        dz[i] = dh * (ht[i] - hp) * z * (1.0f - z);
        dht[i] = dh * z;
        dh = dh * (1.0f - z);
      }
    }
  linear_dx(dz.data(), Wz, dx, N, D, D, true);
  linear_dw(dz.data(), x, dWz, N, D, D);
  linear_dx(dht.data(), Wh, dx, N, D, D, true);
  linear_dw(dht.data(), x, dWh, N, D, D);
  for (int d = 0; d < D; ++d) {
    double a = 0.0, c = 0.0;
    for (int n = 0; n < N; ++n) {
      a += dz[(size_t)n * D + d];
      c += dht[(size_t)n * D + d];
    }
    dbz[d] = (float)((double)dbz[d] + a);
    dbh[d] = (float)((double)dbh[d] + c);
  }
}

// ---------------------------------------------------------------- slot memory
// src/slot_memory.cu:14-77 top-k selection + softmax + gather, exactly the
// reference's sequential scan: held = (-1e30, idx 0) x k; for each slot i in
// order, m = first index of the smallest held value; replace if v > held[m].
// `margin` (optional) receives the selection margin: the smaller of the gap
// between the k-th and (k+1)-th largest score and the smallest gap among the
// selected k (ties there decide the positional order).
static void topk_row(const float* sr, int S, int k, int* idx, float* w, float* margin = nullptr) {
  float val[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int id[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j = 0; j < k; ++j) { val[j] = -1e30f; id[j] = 0; }
  for (int i = 0; i < S; ++i) {
    const float v = sr[i];
    int mk = 0;
    for (int j = 1; j < k; ++j)
      if (val[j] < val[mk]) mk = j;
    if (v > val[mk]) { val[mk] = v; id[mk] = i; }
  }
  if (margin) {
    float kth = val[0];
    for (int j = 1; j < k; ++j) kth = std::fmin(kth, val[j]);
    float next = -INFINITY;
    for (int i = 0; i < S; ++i) {
      bool sel = false;
      for (int j = 0; j < k; ++j) sel = sel || id[j] == i;
      if (!sel) next = std::fmax(next, sr[i]);
    }
    float m = kth - next;
    for (int a = 0; a < k; ++a)
      for (int b = a + 1; b < k; ++b) m = std::fmin(m, std::fabs(val[a] - val[b]));
    *margin = m;
  }
  float mx = val[0];
  for (int j = 1; j < k; ++j) mx = std::fmax(mx, val[j]);
  double sum = 0.0;
  double e[8];
  for (int j = 0; j < k; ++j) { e[j] = std::exp((double)val[j] - mx); sum += e[j]; }
  for (int j = 0; j < k; ++j) { idx[j] = id[j]; w[j] = (float)(e[j] / sum); }
}

// src/slot_memory.cu:79-119: q = x proj_q^T; scores = q K (K [D,S]);
// top-k; r[d] = sum_j w_j V[d, idx_j]; y = r proj_out^T.
//
// `forced` (optional, [N, k]): on rows whose selection margin is below `tau`
// and whose selected set differs from forced's, the forced slots are used
// instead (softmax over their scores, in forced order); `n_forced` counts
// them. Test infrastructure: lets a parity test give the oracle the same
// discrete slot choices as the implementation under test on near-ties.
static void slot_fwd_impl(const float* x, float* y, const float* keys, const float* values,
                          const float* pq, const float* pout, float* q, float* scores, int* idx,
                          float* tw, int B, int T, int D, int S, int k, const int* forced,
                          float tau, int* n_forced) {
  const int N = B * T;
  linear(x, pq, q, N, D, D);
  std::vector<float> Kt = transpose(keys, D, S);  // [S, D]
  gemm_nt(N, S, D, q, Kt.data(), scores, false);
  std::vector<float> r((size_t)N * D);
  int nf = 0;
#pragma omp parallel for schedule(static) reduction(+ : nf)
  for (int n = 0; n < N; ++n) {
    float margin = 0.0f;
    topk_row(scores + (size_t)n * S, S, k, idx + (size_t)n * k, tw + (size_t)n * k,
             forced ? &margin : nullptr);
    if (forced && margin < tau) {
      const int* fr = forced + (size_t)n * k;
      bool same = true;
      for (int a = 0; a < k; ++a) {
        bool found = false;
        for (int b = 0; b < k; ++b) found = found || fr[a] == idx[(size_t)n * k + b];
        same = same && found;
      }
      if (!same) {
        ++nf;
        const float* sr = scores + (size_t)n * S;
        float mx = sr[fr[0]];
        for (int j = 1; j < k; ++j) mx = std::fmax(mx, sr[fr[j]]);
        double e[8], sum = 0.0;
        for (int j = 0; j < k; ++j) { e[j] = std::exp((double)sr[fr[j]] - mx); sum += e[j]; }
        for (int j = 0; j < k; ++j) {
          idx[(size_t)n * k + j] = fr[j];
          tw[(size_t)n * k + j] = (float)(e[j] / sum);
        }
      }
    }
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int j = 0; j < k; ++j)
        acc += (double)tw[(size_t)n * k + j] * values[(size_t)d * S + idx[(size_t)n * k + j]];
      r[(size_t)n * D + d] = (float)acc;
    }
  }
  linear(r.data(), pout, y, N, D, D);
  if (n_forced) *n_forced += nf;
}

void orc_slot_fwd(const float* x, float* y, const float* keys, const float* values,
                  const float* pq, const float* pout, float* q, float* scores, int* idx,
                  float* tw, int B, int T, int D, int S, int k) {
  slot_fwd_impl(x, y, keys, values, pq, pout, q, scores, idx, tw, B, T, D, S, k, nullptr, 0.0f,
                nullptr);
}

// src/slot_memory.cu:122-244: dr = dy proj_out; dproj_out += r^T dy (r
// recomputed from the cached top-k); dV[d,idx] += w dr; dw_j = <dr, V[:,idx_j]>;
// dscore_j = w_j (dw_j - sum w dw); dq = dscore K^T; dK += q^T dscore;
// dx += dq proj_q; dproj_q += x^T dq. The dense d_scores matrix of the
// reference is sparse with k nonzeros per row; the sums are identical.
void orc_slot_bwd(const float* dy, const float* x, const float* keys, const float* values,
                  const float* pq, const float* pout, const float* q, const int* idx,
                  const float* tw, float* dx, float* dkeys, float* dvalues, float* dpq,
                  float* dpout, int B, int T, int D, int S, int k) {
  const int N = B * T;
  const size_t NE = (size_t)N * D;
  std::vector<float> dr(NE), r(NE), dq(NE);
  linear_dx(dy, pout, dr.data(), N, D, D, false);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int j = 0; j < k; ++j)
        acc += (double)tw[(size_t)n * k + j] * values[(size_t)d * S + idx[(size_t)n * k + j]];
      r[(size_t)n * D + d] = (float)acc;
    }
  linear_dw(dy, r.data(), dpout, N, D, D);
  std::vector<double> dV((size_t)D * S, 0.0), dK((size_t)D * S, 0.0);
  std::vector<float> dsc((size_t)N * k);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    double dwj[8];
    for (int j = 0; j < k; ++j) {
      const int s = idx[(size_t)n * k + j];
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)dr[(size_t)n * D + d] * values[(size_t)d * S + s];
      dwj[j] = acc;
    }
    double dot = 0.0;
    for (int j = 0; j < k; ++j) dot += (double)tw[(size_t)n * k + j] * dwj[j];
    for (int j = 0; j < k; ++j) dsc[(size_t)n * k + j] = (float)(tw[(size_t)n * k + j] * (dwj[j] - dot));
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int j = 0; j < k; ++j)
        acc += (double)dsc[(size_t)n * k + j] * keys[(size_t)d * S + idx[(size_t)n * k + j]];
      dq[(size_t)n * D + d] = (float)acc;
    }
  }
  // Scatter (serial for determinism: reference uses atomics)
  for (int n = 0; n < N; ++n)
    for (int j = 0; j < k; ++j) {
      const int s = idx[(size_t)n * k + j];
      const double w = tw[(size_t)n * k + j], ds = dsc[(size_t)n * k + j];
      for (int d = 0; d < D; ++d) {
        dV[(size_t)d * S + s] += w * dr[(size_t)n * D + d];
        dK[(size_t)d * S + s] += ds * q[(size_t)n * D + d];
      }
    }
  for (size_t i = 0; i < (size_t)D * S; ++i) {
    dvalues[i] = (float)((double)dvalues[i] + dV[i]);
    dkeys[i] = (float)((double)dkeys[i] + dK[i]);
  }
  linear_dx(dq.data(), pq, dx, N, D, D, true);
  linear_dw(dq.data(), x, dpq, N, D, D);
}

// ---------------------------------------------------------------- SwiGLU
// src/swiglu_ffn.cu:11-60 (gate, up [F,D]; down [D,F] row-major):
// g = x gate^T, u = x up^T, h = g sigmoid(g) u, y = h down^T.
void orc_swiglu_fwd(const float* x, float* y, const float* gate, const float* up,
                    const float* down, float* gc, float* uc, int N, int D, int F) {
  linear(x, gate, gc, N, F, D);
  linear(x, up, uc, N, F, D);
  std::vector<float> h((size_t)N * F);
  for (size_t i = 0; i < h.size(); ++i) h[i] = gc[i] / (1.0f + std::exp(-gc[i])) * uc[i];
  linear(h.data(), down, y, N, D, F);
}

// src/swiglu_ffn.cu:71-152.
void orc_swiglu_bwd(const float* dy, const float* x, const float* gate, const float* up,
                    const float* down, const float* gc, const float* uc, float* dx, float* dgate,
                    float* dup, float* ddown, int N, int D, int F) {
  const size_t NF = (size_t)N * F;
  std::vector<float> h(NF), dh(NF), dg(NF), du(NF);
  for (size_t i = 0; i < NF; ++i) h[i] = gc[i] / (1.0f + std::exp(-gc[i])) * uc[i];
  linear_dx(dy, down, dh.data(), N, D, F, false);
  linear_dw(dy, h.data(), ddown, N, D, F);
  for (size_t i = 0; i < NF; ++i) {
    const float g = gc[i];
    const float sig = 1.0f / (1.0f + std::exp(-g));
    const float dsilu = sig + g * sig * (1.0f - sig);
    dg[i] = dh[i] * uc[i] * dsilu;
    du[i] = dh[i] * (g * sig);
  }
  linear_dx(dg.data(), gate, dx, N, F, D, true);
  linear_dw(dg.data(), x, dgate, N, F, D);
  linear_dx(du.data(), up, dx, N, F, D, true);
  linear_dw(du.data(), x, dup, N, F, D);
}

// ---------------------------------------------------------------- embedding / head / loss
// src/embedding.cu:6-47
void orc_embed_fwd(const int* tok, const float* table, float* out, int N, int D) {
  for (int n = 0; n < N; ++n)
    std::memcpy(out + (size_t)n * D, table + (size_t)tok[n] * D, sizeof(float) * D);
}
void orc_embed_bwd(const float* dout, const int* tok, float* dtable, int N, int V, int D) {
  std::vector<double> acc((size_t)V * D, 0.0);
  for (int n = 0; n < N; ++n)
    for (int d = 0; d < D; ++d) acc[(size_t)tok[n] * D + d] += dout[(size_t)n * D + d];
  for (size_t i = 0; i < acc.size(); ++i) dtable[i] = (float)((double)dtable[i] + acc[i]);
}
// src/embedding.cu:50-68 — out[M,N] = in[M,K] W[N,K]^T
void orc_linear(const float* in, const float* W, float* out, int M, int N, int K) {
  linear(in, W, out, M, N, K);
}
// src/embedding.cu:97-162 — loss = sum_n -(l[t] - max - log sum exp) (overwrites
// *loss), dlogits = softmax - onehot.
void orc_cross_entropy(const float* logits, const int* tgt, float* loss, float* dl, int N,
                       int V) {
  double total = 0.0;
#pragma omp parallel for reduction(+ : total) schedule(static)
  for (int n = 0; n < N; ++n) {
    const float* l = logits + (size_t)n * V;
    double mx = -1e300;
    for (int i = 0; i < V; ++i) mx = std::fmax(mx, (double)l[i]);
    double s = 0.0;
    for (int i = 0; i < V; ++i) s += std::exp((double)l[i] - mx);
    const double ls = std::log(s);
    total += -((double)l[tgt[n]] - mx - ls);
    for (int i = 0; i < V; ++i)
      dl[(size_t)n * V + i] = (float)(std::exp((double)l[i] - mx - ls) - (i == tgt[n] ? 1.0 : 0.0));
  }
  *loss = (float)total;
}

// ---------------------------------------------------------------- whole model
// Flat parameter layout = checkpoint tensor order (src/resonance_net.cpp:759-778).
size_t orc_param_count(const OrcConfig* c) {
  const size_t D = c->d_model, V = c->vocab_size, F = c->d_ff, S = c->n_slots;
  const size_t per = 4 * D + 25 * D + D * D + 2 * D * D + 2 * D + 2 * D * S + 2 * D * D + 3 * D * F;
  return 2 * V * D + D + per * c->n_layers;
}

}  // extern "C"

namespace {

struct LayerP {
  float *n1, *n2, *n3, *n4, *c3, *c7, *c15, *mix, *Wz, *Wh, *bz, *bh, *keys, *vals, *pq, *pout,
      *gate, *up, *down;
};
struct ModelP {
  float *embed, *out, *fnorm;
  std::vector<LayerP> L;
};

ModelP bind(const OrcConfig* c, float* base) {
  const size_t D = c->d_model, V = c->vocab_size, F = c->d_ff, S = c->n_slots;
  ModelP m;
  float* p = base;
  auto take = [&](size_t n) { float* r = p; p += n; return r; };
  m.embed = take(V * D);
  m.out = take(V * D);
  m.fnorm = take(D);
  for (int l = 0; l < c->n_layers; ++l) {
    LayerP q;
    q.n1 = take(D); q.n2 = take(D); q.n3 = take(D); q.n4 = take(D);
    q.c3 = take(3 * D); q.c7 = take(7 * D); q.c15 = take(15 * D); q.mix = take(D * D);
    q.Wz = take(D * D); q.Wh = take(D * D); q.bz = take(D); q.bh = take(D);
    q.keys = take(D * S); q.vals = take(D * S); q.pq = take(D * D); q.pout = take(D * D);
    q.gate = take(F * D); q.up = take(F * D); q.down = take(D * F);
    m.L.push_back(q);
  }
  return m;
}

struct LayerCache {
  std::vector<float> xin, r1, r2, r3, n1, n2, n3, n4, rms1, rms2, rms3, rms4, convbuf, z, h, q,
      scores, tw, gc, uc;
  std::vector<int> idx;
};

}  // namespace

extern "C" {

// Forward of the whole model (src/resonance_net.cpp:218-343, training path
// with caches). If `cache_out` is null the caches are discarded. Returns
// logits [B*T, V]. `topk_out` (optional) receives the per-layer top-k indices
// [L, B*T, k] and `topw_out` the weights.
void orc_model_forward(const OrcConfig* c, const float* params, const int* tokens, int B, int T,
                       float* logits, int* topk_out, float* topw_out);

// One full training step exactly as src/main.cpp:136-152 + ResonanceNet::step
// (src/resonance_net.cpp:551-663) with world_size = `world` (grads are assumed
// already summed over ranks when world > 1, so lr /= world and the clip
// threshold applies to ||g||/world). params updated in place; grads (flat,
// checkpoint order) returned; loss_sum = sum over tokens (not mean).
void orc_train_step(const OrcConfig* c, float* params, float* grads, const int* tokens,
                    const int* targets, int B, int T, float lr, float clip, int quirk,
                    float* loss_sum, int* topk_out, float* topw_out, float* logits_out);

void orc_train_step_forced(const OrcConfig* c, float* params, float* grads, const int* tokens,
                           const int* targets, int B, int T, float lr, float clip, int quirk,
                           float* loss_sum, int* topk_out, float* topw_out, float* logits_out,
                           const int* forced, float tau, int* n_forced);

// Backward only (no update): grads = d(loss_sum/N)/d params.
void orc_grads(const OrcConfig* c, const float* params, float* grads, const int* tokens,
               const int* targets, int B, int T, int quirk, float* loss_sum);

// SGD with global-norm clip (src/resonance_net.cpp:588-662).
void orc_sgd_step(const OrcConfig* c, float* params, const float* grads, float lr, float clip,
                  int world);

}  // extern "C"

namespace {

void model_fwd_impl(const OrcConfig* c, const ModelP& P, const int* tokens, int B, int T,
                    float* logits, std::vector<LayerCache>* caches, std::vector<float>* hidden_out,
                    std::vector<float>* fnormed, std::vector<float>* frms,
                    const int* forced = nullptr, float tau = 0.0f, int* n_forced = nullptr) {
  const int D = c->d_model, F = c->d_ff, S = c->n_slots, V = c->vocab_size, k = c->slot_top_k;
  const int N = B * T;
  const size_t NE = (size_t)N * D;
  std::vector<float> x(NE), tmp(NE), normed(NE);
  orc_embed_fwd(tokens, P.embed, x.data(), N, D);
  if (caches) caches->assign(c->n_layers, LayerCache());
  for (int l = 0; l < c->n_layers; ++l) {
    const LayerP& W = P.L[l];
    LayerCache lc;
    LayerCache& C = caches ? (*caches)[l] : lc;
    C.xin = x;
    C.n1.resize(NE); C.rms1.resize(N); C.convbuf.resize(3 * NE);
    orc_rms_norm_fwd(x.data(), W.n1, C.n1.data(), C.rms1.data(), N, D, c->rms_eps);
    orc_conv_fwd(C.n1.data(), tmp.data(), W.c3, W.c7, W.c15, W.mix, C.convbuf.data(), B, T, D);
    for (size_t i = 0; i < NE; ++i) x[i] += tmp[i];
    C.r1 = x;
    C.n2.resize(NE); C.rms2.resize(N); C.z.resize(NE); C.h.resize(NE);
    orc_rms_norm_fwd(x.data(), W.n2, C.n2.data(), C.rms2.data(), N, D, c->rms_eps);
    orc_gru_fwd(C.n2.data(), tmp.data(), W.Wz, W.Wh, W.bz, W.bh, C.z.data(), C.h.data(), B, T, D);
    for (size_t i = 0; i < NE; ++i) x[i] += tmp[i];
    C.r2 = x;
    C.n3.resize(NE); C.rms3.resize(N); C.q.resize(NE); C.scores.resize((size_t)N * S);
    C.idx.resize((size_t)N * k); C.tw.resize((size_t)N * k);
    orc_rms_norm_fwd(x.data(), W.n3, C.n3.data(), C.rms3.data(), N, D, c->rms_eps);
    slot_fwd_impl(C.n3.data(), tmp.data(), W.keys, W.vals, W.pq, W.pout, C.q.data(),
                  C.scores.data(), C.idx.data(), C.tw.data(), B, T, D, S, k,
                  forced ? forced + (size_t)l * N * k : nullptr, tau, n_forced);
    for (size_t i = 0; i < NE; ++i) x[i] += tmp[i];
    C.r3 = x;
    C.n4.resize(NE); C.rms4.resize(N); C.gc.resize((size_t)N * F); C.uc.resize((size_t)N * F);
    orc_rms_norm_fwd(x.data(), W.n4, C.n4.data(), C.rms4.data(), N, D, c->rms_eps);
    orc_swiglu_fwd(C.n4.data(), tmp.data(), W.gate, W.up, W.down, C.gc.data(), C.uc.data(), N, D, F);
    for (size_t i = 0; i < NE; ++i) x[i] += tmp[i];
    if (!caches) C.scores.clear();
  }
  std::vector<float> fr(N);
  orc_rms_norm_fwd(x.data(), P.fnorm, normed.data(), fr.data(), N, D, c->rms_eps);
  orc_linear(normed.data(), P.out, logits, N, V, D);
  if (hidden_out) *hidden_out = x;
  if (fnormed) *fnormed = normed;
  if (frms) *frms = fr;
}

void model_bwd_impl(const OrcConfig* c, const ModelP& P, ModelP& G, const int* tokens, int B,
                    int T, const float* dlogits, std::vector<LayerCache>& caches,
                    const std::vector<float>& hidden, const std::vector<float>& fnormed,
                    const std::vector<float>& frms, int quirk) {
  const int D = c->d_model, F = c->d_ff, S = c->n_slots, V = c->vocab_size, k = c->slot_top_k;
  const int N = B * T;
  const size_t NE = (size_t)N * D;
  std::vector<float> dnormed(NE), dh(NE), dsub(NE), dxn(NE);
  // src/resonance_net.cpp:428-442
  linear_dx(dlogits, P.out, dnormed.data(), N, V, D, false);
  linear_dw(dlogits, fnormed.data(), G.out, N, V, D);
  orc_rms_norm_bwd(dnormed.data(), hidden.data(), P.fnorm, frms.data(), dh.data(), G.fnorm, N, D);
  for (int l = c->n_layers - 1; l >= 0; --l) {
    const LayerP& W = P.L[l];
    LayerP& g = G.L[l];
    LayerCache& C = caches[l];
    // src/resonance_net.cpp:468-545
    std::fill(dsub.begin(), dsub.end(), 0.0f);
    orc_swiglu_bwd(dh.data(), C.n4.data(), W.gate, W.up, W.down, C.gc.data(), C.uc.data(),
                   dsub.data(), g.gate, g.up, g.down, N, D, F);
    orc_rms_norm_bwd(dsub.data(), C.r3.data(), W.n4, C.rms4.data(), dxn.data(), g.n4, N, D);
    for (size_t i = 0; i < NE; ++i) dh[i] += dxn[i];
    std::fill(dsub.begin(), dsub.end(), 0.0f);
    orc_slot_bwd(dh.data(), C.n3.data(), W.keys, W.vals, W.pq, W.pout, C.q.data(), C.idx.data(),
                 C.tw.data(), dsub.data(), g.keys, g.vals, g.pq, g.pout, B, T, D, S, k);
    orc_rms_norm_bwd(dsub.data(), C.r2.data(), W.n3, C.rms3.data(), dxn.data(), g.n3, N, D);
    for (size_t i = 0; i < NE; ++i) dh[i] += dxn[i];
    std::fill(dsub.begin(), dsub.end(), 0.0f);
    orc_gru_bwd(dh.data(), C.n2.data(), W.Wz, W.Wh, W.bz, W.bh, C.z.data(), C.h.data(),
                dsub.data(), g.Wz, g.Wh, g.bz, g.bh, B, T, D);
    orc_rms_norm_bwd(dsub.data(), C.r1.data(), W.n2, C.rms2.data(), dxn.data(), g.n2, N, D);
    for (size_t i = 0; i < NE; ++i) dh[i] += dxn[i];
    std::fill(dsub.begin(), dsub.end(), 0.0f);
    orc_conv_bwd(dh.data(), C.n1.data(), W.c3, W.c7, W.c15, W.mix, C.convbuf.data(), dsub.data(),
                 g.c3, g.c7, g.c15, g.mix, B, T, D, quirk);
    orc_rms_norm_bwd(dsub.data(), C.xin.data(), W.n1, C.rms1.data(), dxn.data(), g.n1, N, D);
    for (size_t i = 0; i < NE; ++i) dh[i] += dxn[i];
  }
  orc_embed_bwd(dh.data(), tokens, G.embed, N, V, D);
}

void copy_topk(const OrcConfig* c, const std::vector<LayerCache>& caches, int N, int* topk_out,
               float* topw_out) {
  const int k = c->slot_top_k;
  for (int l = 0; l < c->n_layers; ++l) {
    if (topk_out) std::memcpy(topk_out + (size_t)l * N * k, caches[l].idx.data(), sizeof(int) * N * k);
    if (topw_out) std::memcpy(topw_out + (size_t)l * N * k, caches[l].tw.data(), sizeof(float) * N * k);
  }
}

}  // namespace

extern "C" {

// Row-wise top-k + softmax on a given score matrix (the reference's selection
// rule, src/slot_memory.cu:32-62), for known-answer tests of tie handling.
void orc_topk_rows(const float* scores, int N, int S, int k, int* idx, float* w) {
  for (int n = 0; n < N; ++n)
    topk_row(scores + (size_t)n * S, S, k, idx + (size_t)n * k, w + (size_t)n * k);
}

// Per-layer top-k selection margins [L, B*T] of a forward pass (see topk_row).
void orc_topk_margins(const OrcConfig* c, const float* params, const int* tokens, int B, int T,
                      float* margins) {
  ModelP P = bind(c, const_cast<float*>(params));
  const int N = B * T;
  std::vector<float> logits((size_t)N * c->vocab_size);
  std::vector<LayerCache> caches;
  // forward with caches, then re-run the selection on each layer's scores
  model_fwd_impl(c, P, tokens, B, T, logits.data(), &caches, nullptr, nullptr, nullptr);
  for (int l = 0; l < c->n_layers; ++l) {
    std::vector<int> idx((size_t)N * c->slot_top_k);
    std::vector<float> w((size_t)N * c->slot_top_k);
    for (int n = 0; n < N; ++n)
      topk_row(caches[l].scores.data() + (size_t)n * c->n_slots, c->n_slots, c->slot_top_k,
               idx.data() + (size_t)n * c->slot_top_k, w.data() + (size_t)n * c->slot_top_k,
               margins + (size_t)l * N + n);
  }
}

void orc_model_forward(const OrcConfig* c, const float* params, const int* tokens, int B, int T,
                       float* logits, int* topk_out, float* topw_out) {
  ModelP P = bind(c, const_cast<float*>(params));
  std::vector<LayerCache> caches;
  model_fwd_impl(c, P, tokens, B, T, logits, (topk_out || topw_out) ? &caches : nullptr, nullptr,
                 nullptr, nullptr);
  if (topk_out || topw_out) copy_topk(c, caches, B * T, topk_out, topw_out);
}

void orc_grads(const OrcConfig* c, const float* params, float* grads, const int* tokens,
               const int* targets, int B, int T, int quirk, float* loss_sum) {
  const int N = B * T, V = c->vocab_size;
  ModelP P = bind(c, const_cast<float*>(params));
  std::memset(grads, 0, sizeof(float) * orc_param_count(c));
  ModelP G = bind(c, grads);
  std::vector<LayerCache> caches;
  std::vector<float> hidden, fnormed, frms, logits((size_t)N * V), dl((size_t)N * V);
  model_fwd_impl(c, P, tokens, B, T, logits.data(), &caches, &hidden, &fnormed, &frms);
  float loss = 0.0f;
  orc_cross_entropy(logits.data(), targets, &loss, dl.data(), N, V);
  if (loss_sum) *loss_sum = loss;
  const float sc = 1.0f / (float)N;  // src/main.cpp:146
  for (auto& v : dl) v *= sc;
  model_bwd_impl(c, P, G, tokens, B, T, dl.data(), caches, hidden, fnormed, frms, quirk);
}

void orc_sgd_step(const OrcConfig* c, float* params, const float* grads, float lr, float clip,
                  int world) {
  const size_t P = orc_param_count(c);
  if (world > 1) lr /= (float)world;
  double ss = 0.0;
#pragma omp parallel for reduction(+ : ss) schedule(static)
  for (size_t i = 0; i < P; ++i) ss += (double)grads[i] * grads[i];
  const double norm = std::sqrt(ss) / (world > 1 ? world : 1);
  if (clip > 0 && norm > clip) lr = (float)(lr * (clip / norm));
  const float neg = -lr;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < P; ++i) params[i] = params[i] + neg * grads[i];
}

void orc_train_step(const OrcConfig* c, float* params, float* grads, const int* tokens,
                    const int* targets, int B, int T, float lr, float clip, int quirk,
                    float* loss_sum, int* topk_out, float* topw_out, float* logits_out) {
  orc_train_step_forced(c, params, grads, tokens, targets, B, T, lr, clip, quirk, loss_sum,
                        topk_out, topw_out, logits_out, nullptr, 0.0f, nullptr);
}

// orc_train_step with near-tie slot choices taken from `forced` [L, N, k]
// (see slot_fwd_impl); n_forced receives how many rows were overridden.
void orc_train_step_forced(const OrcConfig* c, float* params, float* grads, const int* tokens,
                           const int* targets, int B, int T, float lr, float clip, int quirk,
                           float* loss_sum, int* topk_out, float* topw_out, float* logits_out,
                           const int* forced, float tau, int* n_forced) {
  const int N = B * T, V = c->vocab_size;
  if (n_forced) *n_forced = 0;
  ModelP P = bind(c, params);
  std::memset(grads, 0, sizeof(float) * orc_param_count(c));
  ModelP G = bind(c, grads);
  std::vector<LayerCache> caches;
  std::vector<float> hidden, fnormed, frms, logits((size_t)N * V), dl((size_t)N * V);
  model_fwd_impl(c, P, tokens, B, T, logits.data(), &caches, &hidden, &fnormed, &frms, forced,
                 tau, n_forced);
  if (logits_out) std::memcpy(logits_out, logits.data(), sizeof(float) * logits.size());
  copy_topk(c, caches, N, topk_out, topw_out);
  float loss = 0.0f;
  orc_cross_entropy(logits.data(), targets, &loss, dl.data(), N, V);
  if (loss_sum) *loss_sum = loss;
  const float sc = 1.0f / (float)N;
  for (auto& v : dl) v *= sc;
  model_bwd_impl(c, P, G, tokens, B, T, dl.data(), caches, hidden, fnormed, frms, quirk);
  orc_sgd_step(c, params, grads, lr, clip, 1);
}

}  // extern "C"
