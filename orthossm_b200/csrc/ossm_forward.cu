// Fused softsign -> Chebyshev -> gamma_h -> tanh -> lambda-EMA forward (sm_100a).
//
// Restates the arithmetic of _fused_clenshaw_ema_kernel (sdpc_kernel.py:988-1209)
// with a different parallel decomposition: the reference walks the whole
// sequence serially in 128-token tiles per (batch, head, 32 channels); here the
// sequence is cut into chunks that run concurrently and are stitched together
// with a decoupled look-back over per-chunk EMA aggregates.
//
// Work decomposition
//   CTA     = (batch b, head h, chunk c of L tokens), 256 threads.
//   thread  = 4 consecutive channels x a run of R consecutive tokens.
//   A head row of head_dim channels is read by P = head_dim/4 threads, so a
//   CTA holds RUNS = 256/P runs and L = RUNS*R tokens (L*head_dim = 16384
//   elements per CTA for R = 16).
// Phases
//   1. load x (streaming), evaluate, scan the run locally from state 0;
//      keep the run's local states in registers.
//   2. per channel, combine the runs' (decay product, state) aggregates in
//      shared memory -> chunk aggregate; publish it; look back over earlier
//      chunks of the same (b, h) for the carry-in; publish the inclusive state.
//   3. out_t = local_t + (decay product up to t) * (run carry-in).
// The decay a_t depends only on (b, t, h), so decay products are per token and
// shared by all channels of the head.
//
// Look-back determinism: a CTA walks back to the nearest chunk with an
// inclusive state I_k, then folds forward I_{j} = fma(A_j, I_{j-1}, B_j) for
// j = k+1 .. c-1, which is the same arithmetic the chunks themselves use to
// publish I_j; results are therefore bitwise independent of timing.
#include <algorithm>

#include "ossm_common.cuh"

namespace ossm {

constexpr int kNT = 256;  // threads per CTA
constexpr int kV = 4;     // channels per thread
// tokens per thread: 16 for the fast (bf16-output) variants, 8 for the
// precise fp32 variants whose library tanhf / IEEE division need more
// registers; both keep the CTA within 128 registers per thread.
template <bool PRECISE>
__host__ __device__ constexpr int run_len() { return PRECISE ? 8 : 16; }

struct FwdParams {
  int B, S, H, HD, K, P, RUNS, L, nchunks, D;
  const void* x;
  long long xsb, xss;
  const float* coeffs;
  const float* lam_h;
  float momentum;
  const float* lam_tok;  // [B,S,H] per-token decay (gate kernel output) or null
  const float* init;
  float* fin;
  void* out;
  long long osb, oss;
  float* tanh_out;
  const float* lut;
  uint32_t flags;
  WsHeader* ws;
  uint32_t* lbflag;  // [N]
  float* aggA;       // [N]
  float* aggB;       // [N][HD]
  float* incB;       // [N][HD]
  uint32_t nctas;
};

OSSM_DEV float ev_clamp4(float v) {
  float r;
  asm("max.NaN.f32 %0, %1, 0fC0800000;\n\tmin.NaN.f32 %0, %0, 0f40800000;" : "=f"(r) : "f"(v));
  return r;
}

struct GateParams {
  int B, S, H, D;
  const void* x;
  long long xsb, xss;
  const float* W;
  const float* bias;
  const float* lam_h;
  float scale, lo, hi;
  float* lam_tok;
};

// ---------------------------------------------------------------------------
// per-token dynamic decay: lam_tok[b,t,h] = clamp(lam_h + scale*(sigmoid(W_h.x_t + b_h) - .5))
// One warp per token; lanes stride over channels in float4 groups.
// ---------------------------------------------------------------------------
template <typename XT>
__global__ void __launch_bounds__(256) gate_kernel(const GateParams g) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long ntok = (long long)g.B * g.S;
  for (long long tok = (long long)blockIdx.x * 8 + warp; tok < ntok; tok += (long long)gridDim.x * 8) {
    const int b = (int)(tok / g.S);
    const int t = (int)(tok % g.S);
    const XT* xr = reinterpret_cast<const XT*>(g.x) + b * g.xsb + t * g.xss;
    float acc[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) acc[h] = 0.f;
    for (int c0 = lane * 4; c0 < g.D; c0 += 128) {
      const float4 xv = ld4(xr + c0);
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        if (h < g.H) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(g.W + (size_t)h * g.D + c0));
          acc[h] = fmaf(w.x, xv.x, acc[h]);
          acc[h] = fmaf(w.y, xv.y, acc[h]);
          acc[h] = fmaf(w.z, xv.z, acc[h]);
          acc[h] = fmaf(w.w, xv.w, acc[h]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
    }
    float mine = 0.f;
#pragma unroll
    for (int h = 0; h < 16; ++h)
      if (h == lane) mine = acc[h];
    if (lane < g.H) {
      const float z = mine + g.bias[lane];
      const float sg = 1.0f / (1.0f + expf(-z));
      const float lam = fminf(fmaxf(g.lam_h[lane] + g.scale * (sg - 0.5f), g.lo), g.hi);
      g.lam_tok[tok * g.H + lane] = lam;
    }
  }
}

// ---------------------------------------------------------------------------
// evaluation of one 4-channel group
// ---------------------------------------------------------------------------
struct Coef {
  float c[8][kV];  // gamma-folded (fast) or raw (precise) coefficients, zero-padded to 8
};

// Clenshaw u_k = 2 x u_{k+1} - u_{k+2} + c_k, y = x u_1 - u_2 + c_0
// (sdpc_kernel.py:1147-1156) on two channels at a time with packed f32x2 math.
OSSM_DEV void clenshaw4(const Coef& cf, const float xn[kV], float y[kV]) {
#pragma unroll
  for (int q = 0; q < kV; q += 2) {
    const float2 x2 = make_float2(2.f * xn[q], 2.f * xn[q + 1]);
    float2 u1 = make_float2(cf.c[7][q], cf.c[7][q + 1]);
    float2 u2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 6; k >= 1; --k) {
      const float2 ck = make_float2(cf.c[k][q], cf.c[k][q + 1]);
      const float2 t = fma2(x2, u1, sub2(ck, u2));
      u2 = u1;
      u1 = t;
    }
    const float2 xh = make_float2(xn[q], xn[q + 1]);
    const float2 c0 = make_float2(cf.c[0][q], cf.c[0][q + 1]);
    const float2 yy = fma2(xh, u1, sub2(c0, u2));
    y[q] = yy.x;
    y[q + 1] = yy.y;
  }
}

// Half-table lookup with linear interpolation and parity reconstruction
// (sdpc_kernel.py:1098-1138).
OSSM_DEV float lut_eval1(const float* lut_s, int K, const float c[8], float xa, float sgn) {
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

// ---------------------------------------------------------------------------
// the scan kernel
// ---------------------------------------------------------------------------
template <typename XT, typename OT, bool PRECISE, bool GENERAL>
__global__ void __launch_bounds__(kNT, 2) fwd_scan_kernel(const FwdParams p) {
  constexpr int kR = run_len<PRECISE>();
  extern __shared__ float smem[];
  float* aggB_s = smem;               // [RUNS][HD] == 1024 floats
  float* aggA_s = aggB_s + 1024;      // [RUNS]
  float* exclA_s = aggA_s + 128;      // [RUNS]
  float* carry_s = exclA_s + 128;     // [HD]
  float* lam_s = carry_s + 256;       // [L]
  float* lut_s = lam_s + 2048;        // [8*256] (LUT mode)
  __shared__ uint32_t s_ticket, s_epoch;

  const int tid = threadIdx.x;
  if (tid == 0) {
    const uint32_t e = atomicAdd(&p.ws->epoch, 0u);
    __threadfence();
    const uint32_t t = atomicAdd(&p.ws->ticket, 1u);
    if (t == p.nctas - 1) {  // every ticket is out: reset for the next launch
      __threadfence();
      atomicExch(&p.ws->ticket, 0u);
      atomicExch(&p.ws->epoch, e + 1u);
    }
    s_ticket = t;
    s_epoch = e;
  }
  const uint32_t eval = p.flags & OSSM_EVAL_MASK;
  if (GENERAL && eval == OSSM_EVAL_LUT) {
    for (int i = tid; i < 8 * 256; i += kNT) lut_s[i] = p.lut[i];
  }
  __syncthreads();
  const uint32_t ticket = s_ticket;
  const uint32_t epoch = s_epoch;
  if (ticket >= p.nctas) {  // the header was not left by a launch of this kernel: report it, touch nothing
    if (tid == 0) atomicExch(&p.ws->status, (uint32_t)OSSM_EWORKSPACE);
    return;
  }
  const int BH = p.B * p.H;
  const int c = (int)(ticket / BH);
  const int rem = (int)(ticket % BH);
  const int b = rem / p.H;
  const int h = rem % p.H;
  const int pi = tid % p.P;
  const int run = tid / p.P;
  const int j0 = pi * kV;
  const int ch0 = h * p.HD + j0;
  const int tbase = c * p.L + run * kR;
  const bool fastpath = GENERAL && (p.flags & OSSM_F_FASTPATH);

  // gamma_h = 0.98 - 0.06 h / H  (sdpc_kernel.py:1041), in fp32
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;
  const int Keff = (eval == OSSM_EVAL_CLENSHAW_DEG4) ? min(p.K, 4) : p.K;
  Coef cf;
  {
    const float* cb = p.coeffs + ((size_t)(b * p.H + h) * p.K) * p.HD + j0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < Keff) v = __ldg(reinterpret_cast<const float4*>(cb + (size_t)k * p.HD));
      const float g = PRECISE ? 1.0f : gamma;
      cf.c[k][0] = v.x * g;
      cf.c[k][1] = v.y * g;
      cf.c[k][2] = v.z * g;
      cf.c[k][3] = v.w * g;
    }
  }
  const bool per_token = p.lam_tok != nullptr;
  const float lam_c = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;

  // ---- phase 1: evaluate + local scan --------------------------------------
  const XT* xb = reinterpret_cast<const XT*>(p.x) + (size_t)b * p.xsb + ch0;
  float sl[kR][kV];
  float s[kV] = {0.f, 0.f, 0.f, 0.f};
  float Arun = 1.f;
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const int t = tbase + r;
    const bool valid = t < p.S;
    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) xv = ld4(xb + (size_t)t * p.xss);
    float lam = 1.f;
    if (valid) lam = per_token ? __ldg(p.lam_tok + ((size_t)b * p.S + t) * p.H + h) : lam_c;
    float xv_[kV] = {xv.x, xv.y, xv.z, xv.w};
    float xn[kV], xa[kV], sg[kV], u[kV];
    bool isnan_[kV];
#pragma unroll
    for (int q = 0; q < kV; ++q) {
      isnan_[q] = xv_[q] != xv_[q];
      xn[q] = softsign<PRECISE>(xv_[q], fastpath, xa[q], sg[q]);
    }
    float y[kV];
    if (GENERAL && eval == OSSM_EVAL_LUT) {
#pragma unroll
      for (int q = 0; q < kV; ++q) {
        float cq[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) cq[k] = cf.c[k][q];
        y[q] = lut_eval1(lut_s, p.K, cq, xa[q], sg[q]);
      }
    } else {
      clenshaw4(cf, xn, y);
    }
#pragma unroll
    for (int q = 0; q < kV; ++q) {
      const float z = PRECISE ? y[q] * gamma : y[q];
      if (fastpath) {
        u[q] = tanhf(z);  // exact torch.tanh of the fast path (:1739)
      } else {
        const float zc = ev_clamp4(z);  // NaN-propagating, as the reference's clamp (:1160-1161)
        u[q] = PRECISE ? tanhf(zc) : tanh_fast(zc);
        if (isnan_[q]) u[q] = 0.f;  // NaN guard (:1164)
      }
      if (!valid) u[q] = 0.f;
    }
    if (p.tanh_out && valid) {
      st4(p.tanh_out + (size_t)b * p.osb + (size_t)t * p.oss + ch0, make_float4(u[0], u[1], u[2], u[3]));
    }
    const float oml = 1.f - lam;
    if (t == 0) {
      // first token of the sequence: fold the carried-in state with the
      // step's clamp, then the scan is linear (|s| stays <= 1).
      const float4 iv = p.init ? __ldg(reinterpret_cast<const float4*>(p.init + (size_t)b * p.D + ch0))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      const float iv_[kV] = {iv.x, iv.y, iv.z, iv.w};
#pragma unroll
      for (int q = 0; q < kV; ++q) s[q] = clamp1(fmaf(lam, iv_[q], oml * u[q]));
      Arun = 0.f;
      lam = 0.f;
    } else {
#pragma unroll
      for (int q = 0; q < kV; ++q) s[q] = fmaf(lam, s[q], oml * u[q]);
      Arun *= lam;
    }
#pragma unroll
    for (int q = 0; q < kV; ++q) sl[r][q] = s[q];
    if (pi == 0) lam_s[run * kR + r] = lam;
  }

  // ---- phase 2: combine runs, look back over chunks -------------------------
#pragma unroll
  for (int q = 0; q < kV; ++q) aggB_s[run * p.HD + j0 + q] = s[q];
  if (pi == 0) aggA_s[run] = Arun;
  __syncthreads();
  const size_t n = (size_t)(b * p.H + h) * p.nchunks + c;  // chain index of this chunk
  float chunkB = 0.f, chunkA = 1.f;
  if (tid < p.HD) {
    float Bv = 0.f, Av = 1.f;
    for (int q = 0; q < p.RUNS; ++q) {
      const float aq = aggA_s[q];
      const float bq = aggB_s[q * p.HD + tid];
      aggB_s[q * p.HD + tid] = Bv;  // exclusive prefix state of run q
      if (tid == 0) exclA_s[q] = Av;
      Bv = fmaf(aq, Bv, bq);
      Av *= aq;
    }
    chunkB = Bv;
    chunkA = Av;
    if (c > 0) {
      p.aggB[n * p.HD + tid] = chunkB;
      if (tid == 0) p.aggA[n] = chunkA;
    }
  }
  __syncthreads();
  // barrier + a gpu-scope release fence in the publishing thread order the
  // CTA's writes before the flag
  if (c > 0 && tid == 0) {
    __threadfence();
    st_release(p.lbflag + n, (epoch << 2) | 1u);
  }

  if (tid < p.HD) {
    float X = 0.f;  // state at the end of chunk c-1
    if (c > 0) {
      // walk back to the nearest inclusive state
      int k = c - 1;
      bool ok = true;
      while (true) {
        const uint32_t st = wait_flag(p.lbflag + (n - (c - k)), epoch);
        if (st == 0) {
          ok = false;
          break;
        }
        if (st == 2 || k == 0) break;
        --k;
      }
      if (ok) {
        X = __ldcg(p.incB + (n - (c - k)) * p.HD + tid);
        for (int j = k + 1; j < c; ++j) {
          const size_t nj = n - (c - j);
          X = fmaf(__ldcg(p.aggA + nj), X, __ldcg(p.aggB + nj * p.HD + tid));
        }
      } else {
        atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
        atomicAdd(&p.ws->timeouts, 1u);
        X = 0.f;
      }
    }
    carry_s[tid] = X;
    p.incB[n * p.HD + tid] = fmaf(chunkA, X, chunkB);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    st_release(p.lbflag + n, (epoch << 2) | 2u);
  }

  // ---- phase 3: apply carries, write ---------------------------------------
  float rc[kV];
  {
    const float ea = exclA_s[run];
#pragma unroll
    for (int q = 0; q < kV; ++q) rc[q] = fmaf(ea, carry_s[j0 + q], aggB_s[run * p.HD + j0 + q]);
  }
  OT* ob = reinterpret_cast<OT*>(p.out) + (size_t)b * p.osb + ch0;
  float Acum = 1.f;
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const int t = tbase + r;
    if (t < p.S) {
      Acum *= lam_s[run * kR + r];
      float o[kV];
#pragma unroll
      for (int q = 0; q < kV; ++q) o[q] = clamp1(fmaf(Acum, rc[q], sl[r][q]));
      st4(ob + (size_t)t * p.oss, make_float4(o[0], o[1], o[2], o[3]));
      if (t == p.S - 1 && p.fin) {
        *reinterpret_cast<float4*>(p.fin + (size_t)b * p.D + ch0) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

}  // namespace ossm

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace ossm;

bool ossm_p3_eligible(const ossm_fwd_args* a);
size_t ossm_p3_workspace_bytes(const ossm_fwd_args* a);
int ossm_p3_parked(const ossm_fwd_args* a);
bool ossm_grp_eligible(const ossm_fwd_args* a);
size_t ossm_grp_workspace_bytes(const ossm_fwd_args* a);
int ossm_grp_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st);
int ossm_p3_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st);
int ossm_p3_shard_front(const ossm_fwd_args* a, int starts_sequence, char* ws, float* shard_decay, float* shard_state,
                        cudaStream_t st);
int ossm_p3_shard_back(const ossm_fwd_args* a, int shard, const float* totals, const float* seq_init, char* ws,
                       cudaStream_t st);
int ossm_p3_shard_fold(int B, int H, int hd, int nshards, const float* totals, const float* init, float* state_out,
                       cudaStream_t st);

namespace {

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

struct FwdLayout {
  int P, RUNS, L, nchunks;
  size_t N, off_flag, off_aggA, off_aggB, off_incB, off_lam, total;
};

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

int validate_fwd(const ossm_fwd_args* a) {
  if (!a) return OSSM_EINVAL;
  if (a->B < 1 || a->S < 1 || a->H < 1 || a->degree < 1 || a->degree > 8) return OSSM_EINVAL;
  if (!is_pow2(a->head_dim) || a->head_dim < 8 || a->head_dim > 256) return OSSM_EINVAL;
  if (!a->x || !a->coeffs || !a->out) return OSSM_EINVAL;
  if ((a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) ||
      (a->out_dtype != OSSM_F32 && a->out_dtype != OSSM_BF16))
    return OSSM_EINVAL;
  const long long D = (long long)a->H * a->head_dim;
  if (a->x_stride_s < D || a->out_stride_s < D) return OSSM_EINVAL;
  if (a->B > 1 && (a->x_stride_b < (long long)a->S * a->x_stride_s && a->x_stride_b < D)) return OSSM_EINVAL;
  const int xel = a->x_dtype == OSSM_F32 ? 4 : 2;
  const int oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  // 4-channel vectors must be naturally aligned
  if (((uintptr_t)a->x % (4 * xel)) || (a->x_stride_s % 4) || (a->x_stride_b % 4)) return OSSM_EINVAL;
  if (((uintptr_t)a->out % (4 * oel)) || (a->out_stride_s % 4) || (a->out_stride_b % 4)) return OSSM_EINVAL;
  if (((uintptr_t)a->coeffs % 16) || (a->init_state && ((uintptr_t)a->init_state % 16)) ||
      (a->final_state && ((uintptr_t)a->final_state % 16)) || (a->tanh_out && ((uintptr_t)a->tanh_out % 16)))
    return OSSM_EINVAL;
  const uint32_t ev = a->flags & OSSM_EVAL_MASK;
  if (ev == 3u) return OSSM_EINVAL;
  if (ev == OSSM_EVAL_LUT && !a->lut) return OSSM_EINVAL;
  if (a->gate_w && (!a->gate_b || !a->lam_h || a->H > 16)) return OSSM_EINVAL;
  if (a->lam_tok && ((uintptr_t)a->lam_tok % 4)) return OSSM_EINVAL;
  if (a->gate_w && ((uintptr_t)a->gate_w % 16)) return OSSM_EINVAL;
  return OSSM_OK;
}

bool fwd_general(const ossm_fwd_args* a) {
  return ((a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_LUT) || (a->flags & OSSM_F_FASTPATH);
}
bool fwd_precise(const ossm_fwd_args* a) {
  return (a->out_dtype == OSSM_F32) || (a->flags & OSSM_F_PRECISE) || (a->flags & OSSM_F_FASTPATH);
}

FwdLayout fwd_layout(const ossm_fwd_args* a) {
  FwdLayout l;
  l.P = a->head_dim / kV;
  l.RUNS = kNT / l.P;
  l.L = l.RUNS * (fwd_precise(a) ? run_len<true>() : run_len<false>());
  l.nchunks = (a->S + l.L - 1) / l.L;
  l.N = (size_t)a->B * a->H * l.nchunks;
  size_t off = sizeof(WsHeader);
  l.off_flag = off;
  off = align256(off + l.N * 4);
  l.off_aggA = off;
  off = align256(off + l.N * 4);
  l.off_aggB = off;
  off = align256(off + l.N * a->head_dim * 4);
  l.off_incB = off;
  off = align256(off + l.N * a->head_dim * 4);
  l.off_lam = off;
  if (a->gate_w && !a->lam_tok) off = align256(off + (size_t)a->B * a->S * a->H * 4);
  l.total = off;
  if (ossm_p3_eligible(a))  // the bf16 fast paths
    l.total = ossm_grp_eligible(a) ? ossm_grp_workspace_bytes(a) : ossm_p3_workspace_bytes(a);
  return l;
}

template <typename XT, typename OT, bool PR, bool GEN>
cudaError_t launch_fwd(const FwdParams& p, cudaStream_t st) {
  const size_t smem = (1024 + 128 + 128 + 256 + 2048 + (GEN ? 2048 : 0)) * sizeof(float);
  fwd_scan_kernel<XT, OT, PR, GEN><<<p.nctas, kNT, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename XT, typename OT>
cudaError_t launch_fwd_dt(const FwdParams& p, bool precise, bool general, cudaStream_t st) {
  if (precise)
    return general ? launch_fwd<XT, OT, true, true>(p, st) : launch_fwd<XT, OT, true, false>(p, st);
  return general ? launch_fwd<XT, OT, false, true>(p, st) : launch_fwd<XT, OT, false, false>(p, st);
}

cudaError_t launch_gate(const ossm_fwd_args* a, float* lam_tok, cudaStream_t st) {
  GateParams g;
  g.B = a->B;
  g.S = a->S;
  g.H = a->H;
  g.D = a->H * a->head_dim;
  g.x = a->x;
  g.xsb = a->x_stride_b;
  g.xss = a->x_stride_s;
  g.W = a->gate_w;
  g.bias = a->gate_b;
  g.lam_h = a->lam_h;
  g.scale = a->gate_scale;
  g.lo = a->gate_lo;
  g.hi = a->gate_hi;
  g.lam_tok = lam_tok;
  const long long ntok = (long long)a->B * a->S;
  const int grid = (int)std::min<long long>((ntok + 7) / 8, 148LL * 16);
  if (a->x_dtype == OSSM_F32)
    gate_kernel<float><<<grid, 256, 0, st>>>(g);
  else
    gate_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(g);
  return cudaGetLastError();
}

}  // namespace

extern "C" size_t ossm_fwd_workspace_bytes(const ossm_fwd_args* a) {
  if (validate_fwd(a) != OSSM_OK) return 0;
  return fwd_layout(a).total;
}

extern "C" int ossm_fwd_path(const ossm_fwd_args* a) {
  if (validate_fwd(a) != OSSM_OK) return -1;
  if (!ossm_p3_eligible(a)) return OSSM_PATH_GENERIC;
  if (ossm_grp_eligible(a)) return OSSM_PATH_GROUPED;
  return ossm_p3_parked(a) ? OSSM_PATH_PARKED : OSSM_PATH_THREE_PASS;
}

// Library-internal: where the generic kernel's look-back flags sit in the
// workspace of these arguments ([offset, offset + bytes)), or 0 bytes when
// the call takes the bf16 fast path, which keeps no flags between launches.
// A workspace shared by calls of different shapes must have this region
// cleared before each generic launch: the flags of one shape can lie over
// another shape's aggregates, and a stale float with a flag's bit pattern
// would pass as a published record.
size_t ossm_fwd_flag_region(const ossm_fwd_args* a, size_t* offset) {
  if (validate_fwd(a) != OSSM_OK || ossm_p3_eligible(a)) return 0;
  const FwdLayout l = fwd_layout(a);
  if (offset) *offset = l.off_flag;
  return l.N * 4;
}

extern "C" int ossm_cheby_ema_fwd(const ossm_fwd_args* a, void* workspace, size_t workspace_bytes,
                                  ossm_stream_t stream) {
  const int v = validate_fwd(a);
  if (v != OSSM_OK) return v;
  const FwdLayout l = fwd_layout(a);
  if (!workspace || workspace_bytes < l.total || ((uintptr_t)workspace % 256)) return OSSM_EWORKSPACE;
  if (l.N >= 0x7fffffffull) return OSSM_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);

  FwdParams p;
  p.B = a->B;
  p.S = a->S;
  p.H = a->H;
  p.HD = a->head_dim;
  p.K = a->degree;
  p.P = l.P;
  p.RUNS = l.RUNS;
  p.L = l.L;
  p.nchunks = l.nchunks;
  p.D = a->H * a->head_dim;
  p.x = a->x;
  p.xsb = a->x_stride_b;
  p.xss = a->x_stride_s;
  p.coeffs = a->coeffs;
  p.lam_h = a->lam_h;
  p.momentum = a->momentum;
  p.lam_tok = a->lam_tok ? a->lam_tok : (a->gate_w ? reinterpret_cast<const float*>(ws + l.off_lam) : nullptr);
  p.init = a->init_state;
  p.fin = a->final_state;
  p.out = a->out;
  p.osb = a->out_stride_b;
  p.oss = a->out_stride_s;
  p.tanh_out = a->tanh_out;
  p.lut = a->lut;
  p.flags = a->flags;
  p.ws = reinterpret_cast<WsHeader*>(ws);
  p.lbflag = reinterpret_cast<uint32_t*>(ws + l.off_flag);
  p.aggA = reinterpret_cast<float*>(ws + l.off_aggA);
  p.aggB = reinterpret_cast<float*>(ws + l.off_aggB);
  p.incB = reinterpret_cast<float*>(ws + l.off_incB);
  p.nctas = (uint32_t)l.N;

  if (ossm_p3_eligible(a)) return ossm_grp_eligible(a) ? ossm_grp_launch(a, ws, st) : ossm_p3_launch(a, ws, st);

  if (a->gate_w && !a->lam_tok) {
    if (launch_gate(a, reinterpret_cast<float*>(ws + l.off_lam), st) != cudaSuccess) return OSSM_ELAUNCH;
  }

  const bool general = fwd_general(a);
  const bool precise = fwd_precise(a);
  cudaError_t e;
  if (a->x_dtype == OSSM_F32)
    e = a->out_dtype == OSSM_F32 ? launch_fwd_dt<float, float>(p, precise, general, st)
                                 : launch_fwd_dt<float, __nv_bfloat16>(p, precise, general, st);
  else
    e = a->out_dtype == OSSM_F32 ? launch_fwd_dt<__nv_bfloat16, float>(p, precise, general, st)
                                 : launch_fwd_dt<__nv_bfloat16, __nv_bfloat16>(p, precise, general, st);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

// Sequence-sharded forward (one shard of consecutive tokens per rank).  Only
// the bf16 fast path (8 heads x 64) supports it; the workspace is the one
// ossm_fwd_workspace_bytes gives for the shard's arguments.
namespace {
int shard_check(const ossm_fwd_args* a, void* workspace, size_t workspace_bytes) {
  const int v = validate_fwd(a);
  if (v != OSSM_OK) return v;
  if (!ossm_p3_eligible(a)) return OSSM_EINVAL;
  if (!workspace || workspace_bytes < ossm_p3_workspace_bytes(a) || ((uintptr_t)workspace % 256))
    return OSSM_EWORKSPACE;
  return OSSM_OK;
}
}  // namespace

extern "C" int ossm_fwd_shard_aggregate(const ossm_fwd_args* a, int starts_sequence, void* workspace,
                                        size_t workspace_bytes, float* shard_decay, float* shard_state,
                                        ossm_stream_t stream) {
  const int v = shard_check(a, workspace, workspace_bytes);
  if (v != OSSM_OK) return v;
  if (!shard_decay || !shard_state || ((uintptr_t)shard_state % 8)) return OSSM_EINVAL;
  return ossm_p3_shard_front(a, starts_sequence, static_cast<char*>(workspace), shard_decay, shard_state,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ossm_fwd_shard_output(const ossm_fwd_args* a, int shard, const float* totals, const float* seq_init,
                                     void* workspace, size_t workspace_bytes, ossm_stream_t stream) {
  const int v = shard_check(a, workspace, workspace_bytes);
  if (v != OSSM_OK) return v;
  if (shard < 0 || (shard > 0 && (!totals || ((uintptr_t)totals % 4)))) return OSSM_EINVAL;
  if (seq_init && ((uintptr_t)seq_init % 4)) return OSSM_EINVAL;
  return ossm_p3_shard_back(a, shard, totals, seq_init, static_cast<char*>(workspace),
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ossm_fwd_shard_fold(int32_t B, int32_t H, int32_t head_dim, int32_t nshards, const float* totals,
                                   const float* seq_init, float* state_out, ossm_stream_t stream) {
  if (B < 1 || H < 1 || head_dim < 1 || nshards < 0 || !state_out || (nshards > 0 && !totals)) return OSSM_EINVAL;
  if ((long long)B * H * head_dim > 0x7fffffffLL) return OSSM_EINVAL;
  return ossm_p3_shard_fold(B, H, head_dim, nshards, totals, seq_init, state_out,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ossm_gate_decay(const ossm_fwd_args* a, float* lam_tok, ossm_stream_t stream) {
  const int v = validate_fwd(a);
  if (v != OSSM_OK) return v;
  if (!a->gate_w || !lam_tok || ((uintptr_t)lam_tok % 4)) return OSSM_EINVAL;
  return launch_gate(a, lam_tok, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

extern "C" int ossm_workspace_status(void* workspace, int clear, ossm_stream_t stream, int32_t* status) {
  if (!workspace || !status) return OSSM_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  WsHeader* h = reinterpret_cast<WsHeader*>(workspace);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, &h->status, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return OSSM_ELAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return OSSM_ELAUNCH;
  *status = (int32_t)v;
  if (clear && v) {
    if (cudaMemsetAsync(&h->status, 0, 4, st) != cudaSuccess) return OSSM_ELAUNCH;
  }
  return OSSM_OK;
}
