// Reference-mode Cheby-RKV + Lion TTT over a whole sequence in one launch (sm_100a).
//
// Restates the full path of apply_cheby_rkv_v10 (sdpc_kernel.py:2574-2606): for
// each chunk of `chunk` tokens, FusedChebyRKVv10.forward (:2352-2433) launches
// _ortho_megakernel (:1889-2287), which runs the forward with the EMA reset to
// zero, accumulates the local gated-error TTT gradient and applies Lion; the
// updated coefficients feed the next chunk through a host loop.
//
// In that computation every channel (b, h, j) is independent: its gradient
// and Lion step use only its own coefficients, momentum and tokens.  So the
// chunk loop moves onto the device: a CTA owns a group of channels of one head
// and walks every chunk of the sequence, keeping coefficients and momentum in
// shared memory between chunks.  One launch replaces ceil(S/chunk) host-loop
// iterations, each of which (in the reference) cast x to bf16, cloned the state,
// allocated fp32 caches, launched, and cast the outputs back.
//
// Within a chunk the CTA processes passes of Lp tokens: thread = 4 channels x a
// run of 8 tokens; runs are combined per channel in shared memory and the pass
// carry stays in shared memory.
#include <math.h>

#include "ossm_common.cuh"

namespace ossm {

namespace lion {
constexpr int kNT = 256;
constexpr int kV = 4;
constexpr int kR = 8;
constexpr int kMaxG = 32;  // channels per CTA
}  // namespace lion

struct LionParams {
  int B, S, H, HD, K, chunk, G, P, RUNS, Lp, ngroups, D;
  const void* x;
  long long xsb, xss;
  float* coeffs;
  float* mom;
  const float* gate;
  const float* dyn;
  float mu, base_lr, beta1, beta2, wd;
  float ss[8];
  const float* lut;
  void* out;
  long long osb, oss;
  float* tanh_out;
  float* fin;
  float* trace;  // optional [nchunks][B,H,K,HD]: the coefficients each chunk starts from
  uint32_t flags;
};

// MULTI_SCALE_LAMBDA (sdpc_kernel.py:1416): per-head forget factor of Lion.
__constant__ float kLionLambda[8] = {0.9995f, 0.9995f, 0.997f, 0.997f, 0.995f, 0.995f, 0.97f, 0.95f};

// x.to(torch.bfloat16) of sdpc_kernel.py:2385, applied on load
template <typename XT>
OSSM_DEV float4 load4_bf16_rounded(const XT* p) {
  const float4 v = ld4(p);
  return make_float4(bf16_round(v.x), bf16_round(v.y), bf16_round(v.z), bf16_round(v.w));
}

OSSM_DEV float eval_one(uint32_t ev, const float* lut_s, int K, const float c[8], float xn, float xa,
                        float sgn) {
  if (ev == OSSM_EVAL_LUT) {
    // sdpc_kernel.py:2030-2069
    const float fidx = xa * 255.0f;
    int i0 = max((int)fidx, 0);
    if (i0 >= 255) i0 = 254;
    const float fr = fminf(fmaxf(fidx - (float)i0, 0.f), 1.f);
    float y = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < K) {
        const float ta = lut_s[k * 256 + i0];
        const float tb = lut_s[k * 256 + i0 + 1];
        float v = c[k] * (ta + fr * (tb - ta));
        if (k & 1) v *= sgn;
        y += v;
      }
    }
    return y;
  }
  // Clenshaw over zero-padded coefficients (exact degree K, or the
  // megakernel's c_0..c_3 truncation when the caller zeroed c_4..c_7)
  const float x2 = 2.f * xn;
  float u1 = c[7], u2 = 0.f;
#pragma unroll
  for (int k = 6; k >= 1; --k) {
    const float t = fmaf(x2, u1, c[k] - u2);
    u2 = u1;
    u1 = t;
  }
  return fmaf(xn, u1, c[0] - u2);
}

template <typename XT, typename OT>
__global__ void __launch_bounds__(lion::kNT, 1) lion_kernel(const LionParams p) {
  using namespace lion;
  extern __shared__ float smem[];
  float* red_s = smem;                 // [RUNS*G][8] gradient partials (8192)
  float* aggB_s = red_s + 8192;        // [RUNS][G] (1024)
  float* aggA_s = aggB_s + 1024;       // [RUNS] (128)
  float* carry_s = aggA_s + 128;       // [G] (32)
  float* csm = carry_s + 32;           // [8][G] coefficients
  float* msm = csm + 256;              // [8][G] Lion momentum
  float* lut_s = msm + 256;            // [8][256]

  const int tid = threadIdx.x;
  const int grp = blockIdx.x % p.ngroups;
  const int bh = blockIdx.x / p.ngroups;
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int G = p.G;
  const int pi = tid % p.P;
  const int run = tid / p.P;
  const int jl = pi * kV;             // channel within the group
  const int jh = grp * G + jl;        // channel within the head
  const int ch0 = h * p.HD + jh;      // channel within D
  const uint32_t ev = p.flags & OSSM_EVAL_MASK;
  const int Keff = ev == OSSM_EVAL_CLENSHAW_DEG4 ? min(p.K, 4) : p.K;

  // _get_lion_constants (:1423-1437) and the head/batch modulation of :2184-2200
  const float lam_h = h < 8 ? kLionLambda[h] : 0.995f;
  const float lr_scale = 1.0f + 0.25f * ((float)h - (float)p.H / 2.0f) / (float)max(p.H, 1);
  float lr = p.base_lr * lr_scale;
  float eff = lam_h;
  if (p.dyn) eff = fminf(fmaxf(lam_h + 0.008f * (__ldg(p.dyn + b) - 0.5f), 0.90f), 0.9999f);
  if (p.gate) lr = lr * __ldg(p.gate + b);
  const float decay = eff - lr * p.wd;
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;

  const size_t cbase = ((size_t)(b * p.H + h) * p.K) * p.HD + grp * G;
  for (int i = tid; i < 8 * G; i += kNT) {
    const int k = i / G, jj = i % G;
    csm[i] = k < p.K ? p.coeffs[cbase + (size_t)k * p.HD + jj] : 0.f;
    msm[i] = k < p.K ? p.mom[cbase + (size_t)k * p.HD + jj] : 0.f;
  }
  if (ev == OSSM_EVAL_LUT)
    for (int i = tid; i < 8 * 256; i += kNT) lut_s[i] = p.lut[i];
  __syncthreads();

  const XT* xb = reinterpret_cast<const XT*>(p.x) + (size_t)b * p.xsb + ch0;
  OT* ob = reinterpret_cast<OT*>(p.out) + (size_t)b * p.osb + ch0;
  const float mu = p.mu, oml = 1.f - p.mu;

  for (int cs = 0; cs < p.S; cs += p.chunk) {
    const int ce = min(cs + p.chunk, p.S);
    float cf[kV][8];
#pragma unroll
    for (int q = 0; q < kV; ++q)
#pragma unroll
      for (int k = 0; k < 8; ++k) cf[q][k] = k < Keff ? csm[k * G + jl + q] : 0.f;
    float g[kV][8];
#pragma unroll
    for (int q = 0; q < kV; ++q)
#pragma unroll
      for (int k = 0; k < 8; ++k) g[q][k] = 0.f;
    if (tid < G) carry_s[tid] = 0.f;  // EMA reset per chunk (:2398)
    if (p.trace && tid < 8 * G) {  // the chunk's starting coefficients, for the backward
      const int k = tid / G, jj = tid % G;
      if (k < p.K)
        p.trace[(size_t)(cs / p.chunk) * ((size_t)p.B * p.H * p.K * p.HD) + cbase + (size_t)k * p.HD + jj] =
            csm[k * G + jj];
    }
    __syncthreads();

    for (int ps = cs; ps < ce; ps += p.Lp) {
      const int tb = ps + run * kR;
      // -- phase 1: forward of the run from state 0
      float sl[kR][kV];
      float s[kV] = {0.f, 0.f, 0.f, 0.f};
      float Arun = 1.f;
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        const int t = tb + r;
        const bool valid = t < ce;
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) xv = load4_bf16_rounded(xb + (size_t)t * p.xss);
        const float xa4[kV] = {xv.x, xv.y, xv.z, xv.w};
        float u[kV];
#pragma unroll
        for (int q = 0; q < kV; ++q) {
          float xa, sg;
          const float xn = softsign<true>(xa4[q], false, xa, sg);
          const float y = eval_one(ev, lut_s, p.K, cf[q], xn, xa, sg) * gamma;
          const float yc = fminf(fmaxf(y, -4.f), 4.f);
          u[q] = (xa4[q] != xa4[q] || !valid) ? 0.f : tanhf(yc);
          if (valid) s[q] = fmaf(mu, s[q], oml * u[q]);
          sl[r][q] = s[q];
        }
        if (valid) Arun *= mu;
        if (p.tanh_out && valid)
          st4(p.tanh_out + (size_t)b * p.osb + (size_t)t * p.oss + ch0, make_float4(u[0], u[1], u[2], u[3]));
      }
      // -- phase 2: combine runs per channel, carry from the previous pass
#pragma unroll
      for (int q = 0; q < kV; ++q) aggB_s[run * G + jl + q] = s[q];
      if (pi == 0) aggA_s[run] = Arun;
      __syncthreads();
      if (tid < G) {
        float Bv = carry_s[tid];
        for (int q = 0; q < p.RUNS; ++q) {
          const float bq = aggB_s[q * G + tid];
          aggB_s[q * G + tid] = Bv;
          Bv = fmaf(aggA_s[q], Bv, bq);
        }
        carry_s[tid] = Bv;
      }
      __syncthreads();
      // -- phase 3: final states, outputs, TTT gradient
      float rc[kV];
#pragma unroll
      for (int q = 0; q < kV; ++q) rc[q] = aggB_s[run * G + jl + q];
      float xn_t[kV];
      if (tb < ce) {
        const float4 xv = load4_bf16_rounded(xb + (size_t)tb * p.xss);
        const float xa4[kV] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < kV; ++q) {
          float xa, sg;
          xn_t[q] = softsign<true>(xa4[q], false, xa, sg);
        }
      }
      float Acum = 1.f;
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        const int t = tb + r;
        if (t < ce) {
          Acum *= mu;
          float sf[kV];
#pragma unroll
          for (int q = 0; q < kV; ++q) sf[q] = clamp1(fmaf(Acum, rc[q], sl[r][q]));
          if (sizeof(OT) == 4)
            st4(ob + (size_t)t * p.oss,
                make_float4(bf16_round(sf[0]), bf16_round(sf[1]), bf16_round(sf[2]), bf16_round(sf[3])));
          else
            st4(ob + (size_t)t * p.oss, make_float4(sf[0], sf[1], sf[2], sf[3]));
          const bool has_next = t + 1 < ce;
          float xn_n[kV] = {0.f, 0.f, 0.f, 0.f};
          if (has_next) {
            const float4 xv = load4_bf16_rounded(xb + (size_t)(t + 1) * p.xss);
            const float xa4[kV] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int q = 0; q < kV; ++q) {
              float xa, sg;
              xn_n[q] = softsign<true>(xa4[q], false, xa, sg);
            }
          }
          // e = xn_{t+1} - s_t, weight sigmoid(3|e|), Chebyshev basis of xn_t (:2141-2169)
#pragma unroll
          for (int q = 0; q < kV; ++q) {
            const float e = has_next ? xn_n[q] - sf[q] : 0.f;
            const float w = 1.0f / (1.0f + expf(-3.0f * fabsf(e)));
            const float gv = e * w;
            const float xq = xn_t[q];
            float T0 = 1.f, T1 = xq;
            g[q][0] = fmaf(gv, T0, g[q][0]);
            g[q][1] = fmaf(gv, T1, g[q][1]);
#pragma unroll
            for (int k = 2; k < 8; ++k) {
              const float T2 = 2.0f * xq * T1 - T0;
              g[q][k] = fmaf(gv, T2, g[q][k]);
              T0 = T1;
              T1 = T2;
            }
            xn_t[q] = xn_n[q];
          }
        }
      }
      __syncthreads();  // aggB_s / carry reuse in the next pass
    }

    // -- chunk end: reduce the gradient over runs, Lion (:2179-2287)
#pragma unroll
    for (int q = 0; q < kV; ++q)
#pragma unroll
      for (int k = 0; k < 8; ++k) red_s[(run * G + jl + q) * 8 + k] = g[q][k];
    __syncthreads();
    if (tid < G * 8) {
      const int jj = tid >> 3, k = tid & 7;
      if (k < p.K) {
        float gs = 0.f;
        for (int q = 0; q < p.RUNS; ++q) gs += red_s[(q * G + jj) * 8 + k];
        const int Lc = ce - cs;
        // the reference divides by Lc - 1 (NaN for a 1-token chunk); a
        // 1-token chunk has no prediction pair and contributes no gradient.
        const float gr = Lc > 1 ? gs * (1.0f / (float)(Lc - 1)) : 0.f;
        const float m = msm[k * G + jj];
        const float c = csm[k * G + jj];
        const float interp = p.beta1 * m + (1.0f - p.beta1) * gr;
        const float sgn = interp > 0.f ? 1.f : (interp < 0.f ? -1.f : 0.f);
        msm[k * G + jj] = p.beta2 * m + (1.0f - p.beta2) * gr;
        csm[k * G + jj] = decay * c + lr * p.ss[k] * sgn;
      }
    }
    __syncthreads();
  }

  for (int i = tid; i < 8 * G; i += kNT) {
    const int k = i / G, jj = i % G;
    if (k < p.K) {
      p.coeffs[cbase + (size_t)k * p.HD + jj] = csm[i];
      p.mom[cbase + (size_t)k * p.HD + jj] = msm[i];
    }
  }
  if (p.fin && tid < G) p.fin[(size_t)b * p.D + h * p.HD + grp * G + tid] = carry_s[tid];
}

}  // namespace ossm

using namespace ossm;

namespace {
bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

template <typename XT, typename OT>
cudaError_t launch_lion(const LionParams& p, int grid, cudaStream_t st) {
  const size_t smem = (8192 + 1024 + 128 + 32 + 256 + 256 + 2048) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(lion_kernel<XT, OT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  lion_kernel<XT, OT><<<grid, lion::kNT, smem, st>>>(p);
  return cudaGetLastError();
}
}  // namespace

extern "C" int ossm_cheby_rkv_lion(const ossm_lion_args* a, ossm_stream_t stream) {
  if (!a || a->B < 1 || a->S < 1 || a->H < 1 || a->degree < 1 || a->degree > 8 || a->chunk < 1)
    return OSSM_EINVAL;
  if (!pow2(a->head_dim) || a->head_dim < 8 || a->head_dim > 256) return OSSM_EINVAL;
  if (!a->x || !a->coeffs || !a->momentum || !a->out) return OSSM_EINVAL;
  if ((a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) || (a->out_dtype != OSSM_F32 && a->out_dtype != OSSM_BF16))
    return OSSM_EINVAL;
  const uint32_t ev = a->flags & OSSM_EVAL_MASK;
  if (ev == 3u || (ev == OSSM_EVAL_LUT && !a->lut)) return OSSM_EINVAL;
  const long long D = (long long)a->H * a->head_dim;
  if (a->x_stride_s < D || a->out_stride_s < D) return OSSM_EINVAL;
  const int xel = a->x_dtype == OSSM_F32 ? 4 : 2, oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  if (((uintptr_t)a->x % (4 * xel)) || (a->x_stride_s % 4) || (a->x_stride_b % 4)) return OSSM_EINVAL;
  if (((uintptr_t)a->out % (4 * oel)) || (a->out_stride_s % 4) || (a->out_stride_b % 4)) return OSSM_EINVAL;
  if (a->tanh_out && ((uintptr_t)a->tanh_out % 16)) return OSSM_EINVAL;

  LionParams p;
  p.B = a->B;
  p.S = a->S;
  p.H = a->H;
  p.HD = a->head_dim;
  p.K = a->degree;
  p.chunk = a->chunk;
  p.G = a->head_dim < lion::kMaxG ? a->head_dim : lion::kMaxG;
  p.P = p.G / lion::kV;
  p.RUNS = lion::kNT / p.P;
  p.Lp = p.RUNS * lion::kR;
  p.ngroups = a->head_dim / p.G;
  p.D = (int)D;
  p.x = a->x;
  p.xsb = a->x_stride_b;
  p.xss = a->x_stride_s;
  p.coeffs = a->coeffs;
  p.mom = a->momentum;
  p.gate = a->gate_global;
  p.dyn = a->dynamic_lambda;
  p.mu = a->ema_momentum;
  p.base_lr = a->base_lr;
  p.beta1 = a->beta1;
  p.beta2 = a->beta2;
  p.wd = a->weight_decay;
  for (int k = 0; k < 8; ++k) p.ss[k] = (float)(1.0 / pow((double)k + 1.0, 1.5));  // (k+1)^-1.5 (:1433)
  p.lut = a->lut;
  p.out = a->out;
  p.osb = a->out_stride_b;
  p.oss = a->out_stride_s;
  p.tanh_out = a->tanh_out;
  p.fin = a->final_state;
  p.flags = a->flags;
  p.trace = a->coeff_trace;
  const long long grid = (long long)a->B * a->H * p.ngroups;
  if (grid > 0x7fffffffLL) return OSSM_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (a->x_dtype == OSSM_F32)
    e = a->out_dtype == OSSM_F32 ? launch_lion<float, float>(p, (int)grid, st)
                                 : launch_lion<float, __nv_bfloat16>(p, (int)grid, st);
  else
    e = a->out_dtype == OSSM_F32 ? launch_lion<__nv_bfloat16, float>(p, (int)grid, st)
                                 : launch_lion<__nv_bfloat16, __nv_bfloat16>(p, (int)grid, st);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
