/*
 * C port of the OrthoSSM Cheby-RKV forward (TEST ORACLE / CPU BASELINE ONLY).
 *
 * Restates, in fp32 with OpenMP threads, the BASELINE-semantics forward that
 * oracle/cheby_ref.py states in float64:
 *   softsign (sdpc_kernel.py:1078-1085), degree-K Clenshaw (:1147-1156),
 *   gamma_h damping (:1041), clamped tanh (:1160-1164), and the per-step
 *   clamped lambda-EMA (:1176-1203; per-head form of
 *   chimera_experiment/chimera_v2_ssm.py:75-98) with the optional per-token
 *   decay lam_h + scale*(sigmoid(W_h x_t + b_h) - 0.5) clamped to [lo, hi].
 * Used by bench.py as the timed CPU path of the reference algorithm and
 * checked against the numpy oracle in tests/.  Not part of the product.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float load_x(const void* x, int bf16, size_t i) {
  return bf16 ? bf16_to_f32(((const uint16_t*)x)[i]) : ((const float*)x)[i];
}

int ossm_ref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* lam_tok[b,t,h] for the dynamic-decay gate. */
static void gate_decay(int B, int S, int H, int D, const void* x, int x_bf16, const float* W,
                       const float* bias, const float* lam_h, float scale, float lo, float hi,
                       float* lam_tok) {
  const long long ntok = (long long)B * S;
#pragma omp parallel for schedule(static)
  for (long long tok = 0; tok < ntok; ++tok) {
    float acc[64];
    for (int h = 0; h < H; ++h) acc[h] = bias[h];
    for (int c = 0; c < D; ++c) {
      const float xv = load_x(x, x_bf16, (size_t)tok * D + c);
      for (int h = 0; h < H; ++h) acc[h] += W[(size_t)h * D + c] * xv;
    }
    for (int h = 0; h < H; ++h) {
      const float g = 1.0f / (1.0f + expf(-acc[h]));
      float l = lam_h[h] + scale * (g - 0.5f);
      l = l < lo ? lo : (l > hi ? hi : l);
      lam_tok[(size_t)tok * H + h] = l;
    }
  }
}

/*
 * x: [B,S,D] contiguous (fp32 or bf16 when x_bf16); coeffs [B,H,K,HD];
 * lam_h [H] or NULL (scalar momentum); gate_w [H,D] / gate_b [H] or NULL;
 * init [B,D] or NULL; out [B,S,D] (fp32, or bf16 when out_bf16); fin [B,D] or NULL.
 * nthreads <= 0: OpenMP default.  Returns 0, or -1 on a bad argument.
 */
int ossm_ref_fwd(int B, int S, int H, int HD, int K, const void* x, int x_bf16, const float* coeffs,
                 const float* lam_h, float momentum, const float* gate_w, const float* gate_b,
                 float gate_scale, float gate_lo, float gate_hi, const float* init, void* out,
                 int out_bf16, float* fin, int nthreads) {
  if (B < 1 || S < 1 || H < 1 || HD < 1 || K < 1 || K > 8 || H > 64) return -1;
  if (gate_w && (!gate_b || !lam_h)) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  const int D = H * HD;
  float* lam_tok = NULL;
  if (gate_w) {
    lam_tok = (float*)malloc((size_t)B * S * H * sizeof(float));
    if (!lam_tok) return -1;
    gate_decay(B, S, H, D, x, x_bf16, gate_w, gate_b, lam_h, gate_scale, gate_lo, gate_hi, lam_tok);
  }
  enum { CB = 16 }; /* channels per work item */
  const int nblk = (D + CB - 1) / CB;
#pragma omp parallel for schedule(static)
  for (int item = 0; item < B * nblk; ++item) {
    const int b = item / nblk;
    const int c0 = (item % nblk) * CB;
    const int cn = (D - c0) < CB ? (D - c0) : CB;
    float cf[CB][8], gam[CB], s[CB], lamc[CB];
    int hh[CB];
    for (int q = 0; q < cn; ++q) {
      const int ch = c0 + q, h = ch / HD, j = ch % HD;
      hh[q] = h;
      gam[q] = 0.98f - 0.06f * (float)h / (float)H;
      for (int k = 0; k < 8; ++k)
        cf[q][k] = k < K ? coeffs[(((size_t)b * H + h) * K + k) * HD + j] : 0.0f;
      s[q] = init ? init[(size_t)b * D + ch] : 0.0f;
      lamc[q] = lam_h ? lam_h[h] : momentum;
    }
    for (int t = 0; t < S; ++t) {
      const size_t row = ((size_t)b * S + t) * D;
      for (int q = 0; q < cn; ++q) {
        const float xv = load_x(x, x_bf16, row + c0 + q);
        const int isnan_ = xv != xv;
        const float xs = isnan_ ? 0.0f : xv;
        float m = fabsf(xs);
        m = m > 1e-7f ? m : 1e-7f;
        const float xa = m / (1.0f + m);
        const float xn = xs >= 0.0f ? xa : -xa;
        const float x2 = 2.0f * xn;
        float u1 = cf[q][7], u2 = 0.0f;
        for (int k = 6; k >= 1; --k) {
          const float tt = x2 * u1 - u2 + cf[q][k];
          u2 = u1;
          u1 = tt;
        }
        float z = (xn * u1 - u2 + cf[q][0]) * gam[q];
        z = z > 4.0f ? 4.0f : (z < -4.0f ? -4.0f : z);
        const float u = isnan_ ? 0.0f : tanhf(z);
        const float lam = lam_tok ? lam_tok[((size_t)b * S + t) * H + hh[q]] : lamc[q];
        float sv = lam * s[q] + (1.0f - lam) * u;
        sv = sv > 1.0f ? 1.0f : (sv < -1.0f ? -1.0f : sv);
        s[q] = sv;
        if (out_bf16)
          ((uint16_t*)out)[row + c0 + q] = f32_to_bf16(sv);
        else
          ((float*)out)[row + c0 + q] = sv;
      }
    }
    if (fin)
      for (int q = 0; q < cn; ++q) fin[(size_t)b * D + c0 + q] = s[q];
  }
  free(lam_tok);
  return 0;
}
