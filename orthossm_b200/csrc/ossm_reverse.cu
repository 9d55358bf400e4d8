// Reverse mode of the Cheby-EMA forward: the backward of ossm_cheby_ema_fwd
// (gradients for x, the coefficients and the carried-in state) and the
// BASELINE-mode test-time training step built on the same adjoint.
//
// Forward (per channel): xn = softsign(x), y = sum_k c_k T_k(xn), z = gamma_h y,
// u = tanh(clamp(z, +-4)), s_t = a_t s_{t-1} + (1 - a_t) u_t (token 0 clamped).
// Given g_t = dL/ds_t (the incoming gradient; for TTT, W_pred^T of the
// prediction error):
//
//   adj_t = g_t + a_{t+1} adj_{t+1}                     (reverse EMA adjoint, adj_S = 0)
//   dy_t  = (1 - a_t) adj_t (1 - u_t^2) gamma_h [|z_t| < 4]   (0 where x is NaN)
//   dL/dc_k = sum_t dy_t T_k(xn_t)
//   dL/dx_t = dy_t y'(xn_t) / (1 + |x_t|)^2            (y' = sum_k c_k T_k')
//   dL/ds_{-1} = a_0 adj_0                               (the carried-in state)
// with the token-0 clamp passing no gradient where it bites.  A segmented
// backward (the reference's chunk loop: the EMA restarts from zero every
// `segment` tokens, each chunk with its own coefficients) cuts the adjoint at
// every restart and returns the gradient of segment 0's coefficients; the
// fast-path backward drops the tanh clamp and uses x.sign().  The decays are
// constants (no gradient through the gate), as in the reference's backward
// (FusedChebyRKVv10.backward, sdpc_kernel.py:2435-2515, which returns
// gradients for x and the coefficients only).
//
// TTT (the reference's TTT is instead the local
// gated-error Lion step, sdpc_kernel.py:2126-2287): g_t = (2/N) W_pred^T
// (W_pred s_t - x_{t+1}) for t < L-1, the gradient is scaled by 1/(k+1)^p and
// feeds Adam with the forget gate c <- lam_h c - lr mhat / (sqrt(vhat) + eps).
//
// The reverse scan is split into 32-token sub-chunks, as the forward is:
//   rev_agg_kernel    warp per (b, h, sub-chunk): its adjoint at the first token
//                     from a zero right carry, and the decay product that
//                     multiplies the right carry;
//   rev_carry_kernel  warp per (b, h): the adjoint entering each sub-chunk from
//                     the right, in a fixed order;
//   rev_grad_kernel   warp per (b, h, sub-chunk): recomputes xn, y, u, the
//                     adjoint and dy; dx per token, dy T_k summed per sub-chunk;
//   rev_reduce_kernel thread per coefficient: the sub-chunk partials in a fixed
//                     order, then (TTT) scaling and Adam.
// Every sum has a fixed order: both are bitwise reproducible.
#include <math.h>

#include "ossm_common.cuh"

namespace ossm {
namespace rev {

constexpr int kL = 32;  // tokens per sub-chunk
constexpr int kMaxK = 8;
constexpr int kB = 8;  // tokens (or sub-chunks) whose loads are issued together

struct Params {
  int B, L, H, HD, K, nq, ngrp;  // ngrp: 64-channel groups per head (one warp each)
  const void* x;
  int x_bf16;
  long long xsb, xss;
  float* coeffs;  // [B,H,K,HD] (TTT: updated in place)
  const float* lam_h;
  float momentum;
  const float* lam_tok;  // [B,L,H] or NULL
  // incoming gradient dL/ds_t: TTT: gs [B,L-1,D] fp32 contiguous (token L-1: 0);
  // backward: g with strides, fp32 or bf16, all L tokens
  int ttt;
  const void* g;
  int g_bf16;
  long long gsb, gss;
  // backward outputs
  void* gx;
  int gx_bf16;
  long long gxsb, gxss;
  float* gc;           // [B,H,K,HD]
  float* ginit;        // [B,D] or NULL
  const float* init;   // [B,D] or NULL (for the token-0 clamp)
  int seg;             // backward: the forward restarted its EMA every seg tokens (0: never)
  const float* cseg;   // [nseg][B,H,K,HD] coefficients per segment (NULL: coeffs)
  int fastpath;        // backward of the fast-path forward: unclamped tanh, sign(0) = 0
  // TTT optimizer
  float* m;
  float* v;
  float lr, beta1, beta2, eps, bc1, bc2, spow;
  int forget;
  // workspace
  float* Rq;    // [B*H][nq][HD]
  float* Aq;    // [B*H][nq]
  float* Cq;    // [B*H][nq][HD]
  float* part;  // [nq][B*H][K][HD]
};

OSSM_DEV float ld_any(const void* p, int bf16, size_t i) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}
OSSM_DEV float xval(const Params& p, int b, int t, int ch) {
  return ld_any(p.x, p.x_bf16, (size_t)b * p.xsb + (size_t)t * p.xss + ch);
}
OSSM_DEV float decay(const Params& p, int b, int t, int h) {  // 1 past the end: nothing enters from there
  if (t >= p.L) return 1.f;
  if (p.lam_tok) return __ldg(p.lam_tok + ((size_t)b * p.L + t) * p.H + h);
  return p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
}
// the decay that carries the adjoint from token t+1 back to token t: zero
// across a restart of the forward's EMA
OSSM_DEV float carry_decay(const Params& p, int b, int t1, int h) {
  if (p.seg > 0 && t1 % p.seg == 0) return 0.f;
  return decay(p, b, t1, h);
}
OSSM_DEV const float* coeffs_at(const Params& p, int t) {
  return (p.seg > 0 && p.cseg) ? p.cseg + (size_t)(t / p.seg) * ((size_t)p.B * p.H * p.K * p.HD) : p.coeffs;
}
OSSM_DEV float gval(const Params& p, int b, int t, int ch) {
  if (p.ttt) {
    const int D = p.H * p.HD;
    return t < p.L - 1 ? __ldg(reinterpret_cast<const float*>(p.g) + ((size_t)b * (p.L - 1) + t) * D + ch) : 0.f;
  }
  return ld_any(p.g, p.g_bf16, (size_t)b * p.gsb + (size_t)t * p.gss + ch);
}

// A warp covers one 64-channel group of a head; lane = channels
// grp*64 + lane and grp*64 + lane + 32.
__global__ void __launch_bounds__(256) rev_agg_kernel(const Params p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= p.B * p.H * p.ngrp * p.nq) return;
  const int q = warp % p.nq, grp = (warp / p.nq) % p.ngrp, bh = warp / (p.nq * p.ngrp), b = bh / p.H, h = bh % p.H;
  const int jb = grp * 64 + lane;
  const int t0 = q * kL;
  float R[2] = {0.f, 0.f};
  float A = 1.f;
  // tokens in batches of kB: the batch's loads first (independent), then the fold
  for (int tb = min(t0 + kL, p.L) - 1; tb >= t0; tb -= kB) {
    float anv[kB], gv[2][kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int t = tb - i;
      anv[i] = t >= t0 ? carry_decay(p, b, t + 1, h) : 1.f;  // a_{t+1}
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = jb + 32 * e;
        gv[e][i] = (t >= t0 && j < p.HD) ? gval(p, b, t, h * p.HD + j) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      if (tb - i < t0) break;
      A *= anv[i];
#pragma unroll
      for (int e = 0; e < 2; ++e) R[e] = fmaf(anv[i], R[e], gv[e][i]);
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = jb + 32 * e;
    if (j < p.HD) p.Rq[((size_t)bh * p.nq + q) * p.HD + j] = R[e];
  }
  if (lane == 0 && grp == 0) p.Aq[(size_t)bh * p.nq + q] = A;
}

// C_q = R_q + A_q C_{q+1}, C_nq = 0: the adjoint at sub-chunk q's first token;
// Cq[q] keeps C_{q+1}, the adjoint entering sub-chunk q from the right.
__global__ void __launch_bounds__(32) rev_carry_kernel(const Params p) {
  const int bh = blockIdx.x / p.ngrp, lane = threadIdx.x;
  const int jb = (blockIdx.x % p.ngrp) * 64 + lane;
  float C[2] = {0.f, 0.f};
  for (int qb = p.nq - 1; qb >= 0; qb -= kB) {  // kB sub-chunks' records first, then the fold
    float Av[kB], Rv[2][kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int q = qb - i;
      Av[i] = q >= 0 ? p.Aq[(size_t)bh * p.nq + q] : 1.f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = jb + 32 * e;
        Rv[e][i] = (q >= 0 && j < p.HD) ? p.Rq[((size_t)bh * p.nq + q) * p.HD + j] : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int q = qb - i;
      if (q < 0) break;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = jb + 32 * e;
        if (j < p.HD) {
          p.Cq[((size_t)bh * p.nq + q) * p.HD + j] = C[e];
          C[e] = fmaf(Av[i], C[e], Rv[e][i]);
        }
      }
    }
  }
}

// DX: the backward (input gradient, carried-in state gradient); without it
// (the TTT step) only the coefficient gradient is formed, so T_k', y' and the
// division for dx are not computed at all.
template <bool DX>
__global__ void __launch_bounds__(256) rev_grad_kernel(const Params p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= p.B * p.H * p.ngrp * p.nq) return;
  const int q = warp % p.nq, grp = (warp / p.nq) % p.ngrp, bh = warp / (p.nq * p.ngrp), b = bh / p.H, h = bh % p.H;
  const int jb = grp * 64 + lane;
  const int t0 = q * kL, t1 = min(t0 + kL, p.L);
  const int D = p.H * p.HD;
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;
  float acc[2][kMaxK];
  float cf[2][kMaxK];
  float adj[2];
  int cur_seg = -1;
  // the coefficients the forward used at token t (one set, or one per segment)
  auto load_cf = [&](int t) {
    const float* cb = coeffs_at(p, t);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = jb + 32 * e;
#pragma unroll
      for (int k = 0; k < kMaxK; ++k)
        cf[e][k] = (j < p.HD && k < p.K) ? cb[(((size_t)b * p.H + h) * p.K + k) * p.HD + j] : 0.f;
    }
  };
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = jb + 32 * e;
    adj[e] = j < p.HD ? p.Cq[((size_t)bh * p.nq + q) * p.HD + j] : 0.f;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) acc[e][k] = 0.f;
  }
  for (int t = t1 - 1; t >= t0; --t) {
    const int sg_t = p.seg > 0 ? t / p.seg : 0;
    if (sg_t != cur_seg) {
      cur_seg = sg_t;
      load_cf(t);
    }
    const float an = carry_decay(p, b, t + 1, h), at = decay(p, b, t, h);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = jb + 32 * e;
      if (j >= p.HD) continue;
      const int ch = h * p.HD + j;
      adj[e] = fmaf(an, adj[e], gval(p, b, t, ch));
      const float x = xval(p, b, t, ch);
      const bool nan = x != x;
      float dx = 0.f;
      // a NaN input: u = 0 in the fused forward (no gradient at all); xn = 0 in the fast path
      if (!nan || p.fastpath) {
        float xa, sg;
        // fused: sign(0) = +1; fast path: x.sign() (0 at 0) and NaN -> 0
        const float xn = nan ? 0.f : (p.fastpath && x == 0.f ? 0.f : softsign<true>(x, false, xa, sg));
        // T_k(xn), T_k'(xn); y = sum c_k T_k, y' = sum c_k T_k'
        float T[kMaxK], dT[kMaxK];
        T[0] = 1.f;
        T[1] = xn;
        dT[0] = 0.f;
        dT[1] = 1.f;
#pragma unroll
        for (int k = 2; k < kMaxK; ++k) {
          T[k] = fmaf(2.f * xn, T[k - 1], -T[k - 2]);
          if (DX) dT[k] = fmaf(2.f * xn, dT[k - 1], fmaf(2.f, T[k - 1], -dT[k - 2]));
        }
        float y = 0.f, yp = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxK; ++k) {
          y = fmaf(cf[e][k], T[k], y);
          if (DX) yp = fmaf(cf[e][k], dT[k], yp);
        }
        const float z = gamma * y;
        const bool live = p.fastpath || fabsf(z) < 4.f;  // the fused clamp passes no gradient where it bites
        const float u = p.fastpath ? tanhf(z) : tanhf(fminf(fmaxf(z, -4.f), 4.f));
        float w = 1.f - at;  // ds_t / du_t
        if (DX && t == 0 && !p.fastpath) {  // token 0: the carried-in state and its clamp
          const float iv = p.init ? p.init[(size_t)b * D + ch] : 0.f;
          const bool pass = fabsf(fmaf(at, iv, (1.f - at) * u)) <= 1.f;
          if (!pass) w = 0.f;
          if (p.ginit) p.ginit[(size_t)b * D + ch] = pass ? at * adj[e] : 0.f;
        }
        const float dy = live ? w * adj[e] * (1.f - u * u) * gamma : 0.f;
        if (p.seg == 0 || t < p.seg)  // segmented: the gradient of segment 0's coefficients
#pragma unroll
          for (int k = 0; k < kMaxK; ++k) acc[e][k] = fmaf(dy, T[k], acc[e][k]);
        if (DX) {
          const float d1 = 1.f + fabsf(x);
          // dxn/dx = 1/(1+|x|)^2 (the fast path's clamp of |x| at 1e-7 passes nothing below it)
          if (!nan && !(p.fastpath && fabsf(x) < 1e-7f)) dx = dy * yp / (d1 * d1);
        }
      } else if (DX && t == 0 && p.ginit) {  // fused, NaN at token 0: u = 0
        const float iv = p.init ? p.init[(size_t)b * D + ch] : 0.f;
        p.ginit[(size_t)b * D + ch] = fabsf(at * iv) <= 1.f ? at * adj[e] : 0.f;
      }
      if (DX) {
        const size_t o = (size_t)b * p.gxsb + (size_t)t * p.gxss + ch;
        if (p.gx_bf16)
          reinterpret_cast<__nv_bfloat16*>(p.gx)[o] = __float2bfloat16_rn(dx);
        else
          reinterpret_cast<float*>(p.gx)[o] = dx;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = jb + 32 * e;
    if (j >= p.HD) continue;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k)
      if (k < p.K) p.part[(((size_t)q * p.B * p.H + bh) * p.K + k) * p.HD + j] = acc[e][k];
  }
}

__global__ void __launch_bounds__(256) rev_reduce_kernel(const Params p) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t per = (size_t)p.B * p.H * p.K * p.HD;
  if (i >= per) return;
  float g = 0.f;
  for (int q = 0; q < p.nq; ++q) g += p.part[(size_t)q * per + i];
  if (!p.ttt) {
    p.gc[i] = g;
    return;
  }
  const int k = (int)((i / p.HD) % p.K), h = (int)((i / ((size_t)p.HD * p.K)) % p.H);
  g *= powf((float)(k + 1), -p.spow);
  const float m = fmaf(p.beta1, p.m[i], (1.f - p.beta1) * g);
  const float v = fmaf(p.beta2, p.v[i], (1.f - p.beta2) * g * g);
  p.m[i] = m;
  p.v[i] = v;
  const float mhat = m / p.bc1, vhat = v / p.bc2;
  const float fg = p.forget ? (p.lam_h ? __ldg(p.lam_h + h) : p.momentum) : 1.f;
  p.coeffs[i] = fg * p.coeffs[i] - p.lr * mhat / (sqrtf(vhat) + p.eps);
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

size_t workspace_bytes(int B, int L, int H, int HD, int K) {
  const size_t nq = (size_t)(L + kL - 1) / kL;
  const size_t BH = (size_t)B * H;
  return 2 * al256(BH * nq * HD * 4) + al256(BH * nq * 4) + al256(nq * BH * K * HD * 4);
}

int run(Params& p, char* ws, cudaStream_t st) {
  const size_t BH = (size_t)p.B * p.H;
  size_t off = 0;
  p.Rq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * p.HD * 4);
  p.Cq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * p.HD * 4);
  p.Aq = reinterpret_cast<float*>(ws + off);
  off += al256(BH * p.nq * 4);
  p.part = reinterpret_cast<float*>(ws + off);
  const size_t warps = BH * p.ngrp * p.nq;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  rev_agg_kernel<<<blocks, 256, 0, st>>>(p);
  rev_carry_kernel<<<(unsigned)(BH * p.ngrp), 32, 0, st>>>(p);
  if (p.ttt)
    rev_grad_kernel<false><<<blocks, 256, 0, st>>>(p);
  else
    rev_grad_kernel<true><<<blocks, 256, 0, st>>>(p);
  const size_t per = BH * p.K * p.HD;
  rev_reduce_kernel<<<(unsigned)((per + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

void common(Params& p, int B, int L, int H, int HD, int K, const void* x, int x_dtype, long long xsb, long long xss,
            float* coeffs, const float* lam_h, float momentum, const float* lam_tok) {
  p.B = B;
  p.L = L;
  p.H = H;
  p.HD = HD;
  p.K = K;
  p.nq = (L + kL - 1) / kL;
  p.ngrp = (HD + 63) / 64;
  p.x = x;
  p.x_bf16 = x_dtype == OSSM_BF16;
  p.xsb = xsb;
  p.xss = xss;
  p.coeffs = coeffs;
  p.lam_h = lam_h;
  p.momentum = momentum;
  p.lam_tok = lam_tok;
  p.g = nullptr;
  p.g_bf16 = 0;
  p.gsb = p.gss = 0;
  p.gx = nullptr;
  p.gx_bf16 = 0;
  p.gxsb = p.gxss = 0;
  p.gc = nullptr;
  p.ginit = nullptr;
  p.init = nullptr;
  p.seg = 0;
  p.cseg = nullptr;
  p.fastpath = 0;
  p.m = p.v = nullptr;
  p.lr = p.beta1 = p.beta2 = p.eps = p.spow = 0.f;
  p.bc1 = p.bc2 = 1.f;
  p.forget = 0;
}

}  // namespace rev
}  // namespace ossm

using namespace ossm;

namespace {
int ttt_validate(const ossm_ttt_args* a) {
  if (!a || a->B < 1 || a->L < 1 || a->H < 1 || a->head_dim < 1 || a->head_dim > 256 || a->degree < 1 ||
      a->degree > rev::kMaxK)
    return OSSM_EINVAL;
  if (!a->x || !a->coeffs || !a->m || !a->v || (a->L > 1 && !a->gs)) return OSSM_EINVAL;
  if (a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) return OSSM_EINVAL;
  if (a->step < 1) return OSSM_EINVAL;
  return OSSM_OK;
}
int bwd_validate(const ossm_bwd_args* a) {
  if (!a || a->B < 1 || a->S < 1 || a->H < 1 || a->head_dim < 1 || a->head_dim > 256 || a->degree < 1 ||
      a->degree > rev::kMaxK)
    return OSSM_EINVAL;
  if (!a->x || !a->coeffs || !a->grad_out || !a->grad_x || !a->grad_coeffs) return OSSM_EINVAL;
  if (a->segment < 0 || (a->segment > 0 && a->segment < a->S && !a->segment_coeffs)) return OSSM_EINVAL;
  for (int dt : {a->x_dtype, a->grad_out_dtype, a->grad_x_dtype})
    if (dt != OSSM_F32 && dt != OSSM_BF16) return OSSM_EINVAL;
  return OSSM_OK;
}
}  // namespace

extern "C" size_t ossm_ttt_workspace_bytes(const ossm_ttt_args* a) {
  if (ttt_validate(a) != OSSM_OK) return 0;
  return rev::workspace_bytes(a->B, a->L, a->H, a->head_dim, a->degree);
}

extern "C" int ossm_ttt_wpred_step(const ossm_ttt_args* a, void* workspace, size_t workspace_bytes,
                                   ossm_stream_t stream) {
  const int v = ttt_validate(a);
  if (v != OSSM_OK) return v;
  if (!workspace || workspace_bytes < ossm_ttt_workspace_bytes(a) || ((uintptr_t)workspace % 256))
    return OSSM_EWORKSPACE;
  rev::Params p;
  rev::common(p, a->B, a->L, a->H, a->head_dim, a->degree, a->x, a->x_dtype, a->x_stride_b, a->x_stride_s,
              a->coeffs, a->lam_h, a->momentum, a->lam_tok);
  p.ttt = 1;
  p.g = a->gs;
  p.m = a->m;
  p.v = a->v;
  p.lr = a->lr;
  p.beta1 = a->beta1;
  p.beta2 = a->beta2;
  p.eps = a->eps;
  p.bc1 = 1.f - powf(a->beta1, (float)a->step);
  p.bc2 = 1.f - powf(a->beta2, (float)a->step);
  p.spow = a->spectral_pow;
  p.forget = a->forget;
  return rev::run(p, static_cast<char*>(workspace), reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t ossm_bwd_workspace_bytes(const ossm_bwd_args* a) {
  if (bwd_validate(a) != OSSM_OK) return 0;
  return rev::workspace_bytes(a->B, a->S, a->H, a->head_dim, a->degree);
}

extern "C" int ossm_cheby_ema_bwd(const ossm_bwd_args* a, void* workspace, size_t workspace_bytes,
                                  ossm_stream_t stream) {
  const int v = bwd_validate(a);
  if (v != OSSM_OK) return v;
  if (!workspace || workspace_bytes < ossm_bwd_workspace_bytes(a) || ((uintptr_t)workspace % 256))
    return OSSM_EWORKSPACE;
  rev::Params p;
  rev::common(p, a->B, a->S, a->H, a->head_dim, a->degree, a->x, a->x_dtype, a->x_stride_b, a->x_stride_s,
              const_cast<float*>(a->coeffs), a->lam_h, a->momentum, a->lam_tok);
  p.ttt = 0;
  p.g = a->grad_out;
  p.g_bf16 = a->grad_out_dtype == OSSM_BF16;
  p.gsb = a->grad_out_stride_b;
  p.gss = a->grad_out_stride_s;
  p.gx = a->grad_x;
  p.gx_bf16 = a->grad_x_dtype == OSSM_BF16;
  p.gxsb = a->grad_x_stride_b;
  p.gxss = a->grad_x_stride_s;
  p.gc = a->grad_coeffs;
  p.ginit = a->grad_init;
  p.init = a->init_state;
  p.seg = a->segment > 0 && a->segment < a->S ? a->segment : 0;
  p.cseg = p.seg ? a->segment_coeffs : nullptr;
  p.fastpath = (a->flags & OSSM_F_FASTPATH) ? 1 : 0;
  return rev::run(p, static_cast<char*>(workspace), reinterpret_cast<cudaStream_t>(stream));
}
