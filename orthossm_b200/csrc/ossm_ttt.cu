// BASELINE-mode test-time training step (no
// counterpart kernel in the reference, whose TTT is the local gated-error
// Lion step of _ortho_megakernel, sdpc_kernel.py:2126-2287).
//
// For one chunk of L tokens, after the forward (states s_t, fp32) and the two
// W_pred products done by the caller (cuBLAS):
//
//   gs_t  = dL/ds_t = (2/N) W_pred^T (W_pred s_t - x_{t+1}),  t < L-1;  gs_{L-1} = 0
//   adj_t = gs_t + a_{t+1} adj_{t+1}           (reverse EMA adjoint, adj_L = 0)
//   dy_t  = (1 - a_t) adj_t (1 - u_t^2) gamma_h [|gamma_h y_t| < 4]   (0 where x is NaN)
//   g_k   = sum_t dy_t T_k(xn_t) / (k+1)^p
//   Adam:  m <- b1 m + (1-b1) g,  v <- b2 v + (1-b2) g^2,
//          c <- lam_h c - lr mhat / (sqrt(vhat) + eps)   (lam_h = 1 without the forget gate)
//
// The reverse scan is split into 32-token sub-chunks, as the forward is:
//   ttt_rev_agg_kernel    warp per (b, h, sub-chunk): the sub-chunk's adjoint at
//                         its first token from a zero right carry, and the decay
//                         product that multiplies the right carry;
//   ttt_rev_carry_kernel  warp per (b, h): the adjoint entering each sub-chunk
//                         from the right, in a fixed order;
//   ttt_grad_kernel       warp per (b, h, sub-chunk): recomputes xn, y, u, the
//                         adjoint and dy, and sums dy T_k over its 32 tokens;
//   ttt_adam_kernel       thread per coefficient: sums the sub-chunk partials in
//                         a fixed order, scales, and applies Adam.
// Every sum has a fixed order: the step is bitwise reproducible.
#include <math.h>

#include "ossm_common.cuh"

namespace ossm {
namespace ttt {

constexpr int kL = 32;  // tokens per sub-chunk (lane = 2 channels of one head)
constexpr int kMaxK = 8;

struct Params {
  int B, L, H, HD, K, nq;
  const void* x;
  int x_bf16;
  long long xsb, xss;
  float* coeffs;  // [B,H,K,HD] in/out
  float* m;       // [B,H,K,HD] in/out
  float* v;       // [B,H,K,HD] in/out
  const float* lam_h;
  float momentum;
  const float* lam_tok;  // [B,L,H] or NULL
  const float* gs;       // [B,L-1,D] fp32 (contiguous)
  float lr, beta1, beta2, eps, bc1, bc2, spow;
  int forget;
  float* Rq;    // [B*H][nq][HD] sub-chunk adjoint at its first token, zero right carry
  float* Aq;    // [B*H][nq] decay product multiplying the right carry
  float* Cq;    // [B*H][nq][HD] adjoint entering each sub-chunk from the right
  float* part;  // [nq][B*H][K][HD] gradient partials
};

OSSM_DEV float xval(const Params& p, int b, int t, int ch) {
  if (p.x_bf16)
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.x)[(size_t)b * p.xsb + (size_t)t * p.xss + ch]);
  return reinterpret_cast<const float*>(p.x)[(size_t)b * p.xsb + (size_t)t * p.xss + ch];
}
// decay a_t of token t, head h (1 past the end, so nothing enters from there)
OSSM_DEV float decay(const Params& p, int b, int t, int h) {
  if (t >= p.L) return 1.f;
  if (p.lam_tok) return __ldg(p.lam_tok + ((size_t)b * p.L + t) * p.H + h);
  return p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
}
OSSM_DEV float gsval(const Params& p, int b, int t, int ch) {
  const int D = p.H * p.HD;
  return t < p.L - 1 ? __ldg(p.gs + ((size_t)b * (p.L - 1) + t) * D + ch) : 0.f;
}

// warp per (b, h, q); lane covers channels lane and lane + 32 of the head
// (head_dim 64) or lane only (head_dim 32); generic over HD <= 64.
__global__ void __launch_bounds__(256) ttt_rev_agg_kernel(const Params p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nch = p.B * p.H * p.nq;
  if (warp >= nch) return;
  const int q = warp % p.nq, bh = warp / p.nq, b = bh / p.H, h = bh % p.H;
  const int t0 = q * kL;
  float R[2] = {0.f, 0.f};
  float A = 1.f;
  for (int t = min(t0 + kL, p.L) - 1; t >= t0; --t) {
    const float an = decay(p, b, t + 1, h);  // a_{t+1}
    A *= an;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = lane + 32 * e;
      if (j < p.HD) R[e] = fmaf(an, R[e], gsval(p, b, t, h * p.HD + j));
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = lane + 32 * e;
    if (j < p.HD) p.Rq[((size_t)bh * p.nq + q) * p.HD + j] = R[e];
  }
  if (lane == 0) p.Aq[(size_t)bh * p.nq + q] = A;
}

// one warp per (b, h): C_q = R_q + A_q C_{q+1}, C_nq = 0 (the adjoint at the
// first token of sub-chunk q); Cq[q] stores C_{q+1}, the carry entering from the right.
__global__ void __launch_bounds__(32) ttt_rev_carry_kernel(const Params p) {
  const int bh = blockIdx.x, lane = threadIdx.x;
  float C[2] = {0.f, 0.f};
  for (int q = p.nq - 1; q >= 0; --q) {
    const float A = p.Aq[(size_t)bh * p.nq + q];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = lane + 32 * e;
      if (j < p.HD) {
        p.Cq[((size_t)bh * p.nq + q) * p.HD + j] = C[e];
        C[e] = fmaf(A, C[e], p.Rq[((size_t)bh * p.nq + q) * p.HD + j]);
      }
    }
  }
}

__global__ void __launch_bounds__(256) ttt_grad_kernel(const Params p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nch = p.B * p.H * p.nq;
  if (warp >= nch) return;
  const int q = warp % p.nq, bh = warp / p.nq, b = bh / p.H, h = bh % p.H;
  const int t0 = q * kL, t1 = min(t0 + kL, p.L);
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;
  float acc[2][kMaxK];
  float cf[2][kMaxK];
  float adj[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = lane + 32 * e;
    adj[e] = j < p.HD ? p.Cq[((size_t)bh * p.nq + q) * p.HD + j] : 0.f;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
      acc[e][k] = 0.f;
      cf[e][k] = (j < p.HD && k < p.K) ? p.coeffs[(((size_t)b * p.H + h) * p.K + k) * p.HD + j] : 0.f;
    }
  }
  for (int t = t1 - 1; t >= t0; --t) {
    const float an = decay(p, b, t + 1, h), at = decay(p, b, t, h);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = lane + 32 * e;
      if (j >= p.HD) continue;
      const int ch = h * p.HD + j;
      adj[e] = fmaf(an, adj[e], gsval(p, b, t, ch));
      const float x = xval(p, b, t, ch);
      if (x != x) continue;  // NaN input: u = 0, no gradient
      float xa, sg;
      const float xn = softsign<true>(x, false, xa, sg);
      // T_k(xn) and y = sum_k c_k T_k(xn) (the same basis feeds both)
      float T[kMaxK];
      T[0] = 1.f;
      T[1] = xn;
#pragma unroll
      for (int k = 2; k < kMaxK; ++k) T[k] = fmaf(2.f * xn, T[k - 1], -T[k - 2]);
      float y = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) y = fmaf(cf[e][k], T[k], y);
      const float z = gamma * y;
      if (!(fabsf(z) < 4.f)) continue;  // clamp: no gradient through the saturated branch
      const float u = tanhf(z);
      const float dy = (1.f - at) * adj[e] * (1.f - u * u) * gamma;
#pragma unroll
      for (int k = 0; k < kMaxK; ++k) acc[e][k] = fmaf(dy, T[k], acc[e][k]);
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = lane + 32 * e;
    if (j >= p.HD) continue;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k)
      if (k < p.K) p.part[(((size_t)q * p.B * p.H + bh) * p.K + k) * p.HD + j] = acc[e][k];
  }
}

__global__ void __launch_bounds__(256) ttt_adam_kernel(const Params p) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t per = (size_t)p.B * p.H * p.K * p.HD;
  if (i >= per) return;
  const int k = (int)((i / p.HD) % p.K), h = (int)((i / ((size_t)p.HD * p.K)) % p.H);
  float g = 0.f;
  for (int q = 0; q < p.nq; ++q) g += p.part[(size_t)q * per + i];
  g *= powf((float)(k + 1), -p.spow);
  const float m = fmaf(p.beta1, p.m[i], (1.f - p.beta1) * g);
  const float v = fmaf(p.beta2, p.v[i], (1.f - p.beta2) * g * g);
  p.m[i] = m;
  p.v[i] = v;
  const float mhat = m / p.bc1, vhat = v / p.bc2;
  const float fg = p.forget ? (p.lam_h ? __ldg(p.lam_h + h) : p.momentum) : 1.f;
  p.coeffs[i] = fg * p.coeffs[i] - p.lr * mhat / (sqrtf(vhat) + p.eps);
}

}  // namespace ttt
}  // namespace ossm

using namespace ossm;

namespace {
size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }
int ttt_validate(const ossm_ttt_args* a) {
  if (!a || a->B < 1 || a->L < 1 || a->H < 1 || a->head_dim < 1 || a->head_dim > 64 || a->degree < 1 ||
      a->degree > ttt::kMaxK)
    return OSSM_EINVAL;
  if (!a->x || !a->coeffs || !a->m || !a->v || (a->L > 1 && !a->gs)) return OSSM_EINVAL;
  if (a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) return OSSM_EINVAL;
  if (a->step < 1) return OSSM_EINVAL;
  return OSSM_OK;
}
}  // namespace

extern "C" size_t ossm_ttt_workspace_bytes(const ossm_ttt_args* a) {
  if (ttt_validate(a) != OSSM_OK) return 0;
  const size_t nq = (size_t)(a->L + ttt::kL - 1) / ttt::kL;
  const size_t BH = (size_t)a->B * a->H;
  return 2 * al256(BH * nq * a->head_dim * 4) + al256(BH * nq * 4) +
         al256(nq * BH * a->degree * a->head_dim * 4);
}

extern "C" int ossm_ttt_wpred_step(const ossm_ttt_args* a, void* workspace, size_t workspace_bytes,
                                   ossm_stream_t stream) {
  const int v = ttt_validate(a);
  if (v != OSSM_OK) return v;
  const size_t need = ossm_ttt_workspace_bytes(a);
  if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 256)) return OSSM_EWORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ttt::Params p;
  p.B = a->B;
  p.L = a->L;
  p.H = a->H;
  p.HD = a->head_dim;
  p.K = a->degree;
  p.nq = (a->L + ttt::kL - 1) / ttt::kL;
  p.x = a->x;
  p.x_bf16 = a->x_dtype == OSSM_BF16;
  p.xsb = a->x_stride_b;
  p.xss = a->x_stride_s;
  p.coeffs = a->coeffs;
  p.m = a->m;
  p.v = a->v;
  p.lam_h = a->lam_h;
  p.momentum = a->momentum;
  p.lam_tok = a->lam_tok;
  p.gs = a->gs;
  p.lr = a->lr;
  p.beta1 = a->beta1;
  p.beta2 = a->beta2;
  p.eps = a->eps;
  p.bc1 = 1.f - powf(a->beta1, (float)a->step);
  p.bc2 = 1.f - powf(a->beta2, (float)a->step);
  p.spow = a->spectral_pow;
  p.forget = a->forget;
  const size_t BH = (size_t)a->B * a->H;
  char* ws = static_cast<char*>(workspace);
  size_t off = 0;
  p.Rq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * p.HD * 4);
  p.Cq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * p.HD * 4);
  p.Aq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * 4);
  p.part = reinterpret_cast<float*>(ws + off);

  const size_t warps = BH * p.nq;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  ttt::ttt_rev_agg_kernel<<<blocks, 256, 0, st>>>(p);
  ttt::ttt_rev_carry_kernel<<<(unsigned)BH, 32, 0, st>>>(p);
  ttt::ttt_grad_kernel<<<blocks, 256, 0, st>>>(p);
  const size_t per = BH * p.K * p.HD;
  ttt::ttt_adam_kernel<<<(unsigned)((per + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
