// Forward fast path for bf16 activations with head_dim 64 (sm_100a):
// TMA-staged tiles, the per-token decay gate on tcgen05 tensor cores inside an
// H-CTA cluster, packed f32x2 arithmetic, decoupled look-back across chunks.
//
// Same arithmetic contract as fwd_scan_kernel in ossm_forward.cu (which
// restates _fused_clenshaw_ema_kernel, sdpc_kernel.py:988-1209); this file only
// changes how the work is mapped onto the B200:
//
//   cluster = the H heads of one (batch b, chunk c of 256 tokens); CTA = head h.
//   1. one thread issues a 3D TMA load of the [256 tokens x 64 channels] bf16
//      tile (128-byte swizzle) into shared memory;
//   2. gate (optional): the tile is also the A operand of a tcgen05 MMA,
//      D[256 x 16] = X[256 x 64] . Wsplit[16 x 64]^T, where Wsplit holds the
//      gate weights of this head's 64 channels for all H heads as bf16 hi and
//      bf16 lo halves (x is exact in bf16, so hi+lo keeps ~16 mantissa bits of
//      W).  Each CTA sends its per-token partial logits to the owning head's
//      CTA over distributed shared memory; after a cluster barrier every CTA
//      holds the full logits of its head and forms lambda_t;
//   3. meanwhile threads evaluate softsign -> Chebyshev -> tanh from shared
//      memory (lane = 2 channels, warp = a run of 32 tokens; a warp reads one
//      128-byte row per token), then scan locally;
//   4. runs are combined per channel, the chunk publishes its aggregate, a
//      warp-wide look-back window finds the nearest inclusive predecessor, the
//      carry is folded forward, outputs are written.
#include <cudaTypedefs.h>

#include <mutex>

#include "ossm_sm100.cuh"

namespace ossm {
namespace tc {

constexpr int kNT = 256;
constexpr int kHD = 64;      // channels per CTA (one head)
constexpr int kL = 256;      // tokens per CTA
constexpr int kR = 32;       // tokens per thread (one run per warp)
constexpr int kRUNS = 8;     // runs per CTA (a warp covers a 64-channel row)
constexpr int kMaxH = 8;

// shared memory layout (bytes from a 1024-aligned base)
constexpr int kOffX = 0;                               // [256][128 B] swizzled x tile
constexpr int kOffW = kOffX + kL * 128;                // [16][128 B] swizzled gate weights
constexpr int kOffAggB = kOffW + 16 * 128;             // [16 runs][64] f32
constexpr int kOffAggA = kOffAggB + kRUNS * kHD * 4;   // [16] f32
constexpr int kOffExclA = kOffAggA + 64;               // [16] f32
constexpr int kOffCarry = kOffExclA + 64;              // [64] f32
constexpr int kOffLam = kOffCarry + kHD * 4;           // [256] float4 (lam, lam, 1-lam, 1-lam)
constexpr int kOffPart = kOffLam + kL * 16;            // [8 src][256] f32 partial logits
constexpr int kOffBar = kOffPart + kMaxH * kL * 4;     // 2 mbarriers + scalars
constexpr int kSmemBytes = kOffBar + 64;
constexpr int kSmemAlloc = kSmemBytes + 1024;          // slack for 1024-byte alignment

struct Params {
  int B, S, H, K, nchunks, D;
  const float* coeffs;
  const float* lam_h;
  float momentum;
  const float* gate_w;
  const float* gate_b;
  float gate_scale, gate_lo, gate_hi;
  const float* lam_tok;
  const float* init;
  float* fin;
  void* out;
  long long osb, oss;
  WsHeader* ws;
  uint32_t* lbflag;
  float* aggA;
  float* aggB;
  float* incB;
  uint32_t nunits;  // tickets per launch (clusters with the gate, CTAs without)
};

OSSM_DEV float4 unpack_bf16x4(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

template <bool GATE, bool PRECISE, typename OT>
__global__ void __launch_bounds__(kNT, 2) fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap, const Params p) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = sm + kOffX;
  uint8_t* wsm = sm + kOffW;
  float* aggB_s = reinterpret_cast<float*>(sm + kOffAggB);
  float* aggA_s = reinterpret_cast<float*>(sm + kOffAggA);
  float* exclA_s = reinterpret_cast<float*>(sm + kOffExclA);
  float* carry_s = reinterpret_cast<float*>(sm + kOffCarry);
  float4* lam_s = reinterpret_cast<float4*>(sm + kOffLam);
  float* part_s = reinterpret_cast<float*>(sm + kOffPart);
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* mma_bar = tma_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffBar + 16);
  uint32_t* s_ticket = tmem_slot + 1;
  uint32_t* s_epoch = tmem_slot + 2;
  int* s_kincl = reinterpret_cast<int*>(tmem_slot + 3);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = GATE ? cluster_rank() : 0u;

  // ---- ticket (one per cluster / CTA), mbarrier init --------------------------
  if (tid == 0) {
    mbar_init(tma_bar, 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap);
  }
  if (GATE && warp == 1) tmem_alloc(tmem_slot, 32);
  if (tid == 0 && crank == 0) {
    const uint32_t e = atomicAdd(&p.ws->epoch, 0u);
    __threadfence();
    const uint32_t t = atomicAdd(&p.ws->ticket, 1u);
    if (t == p.nunits - 1) {  // every ticket is out: reset for the next launch
      __threadfence();
      atomicExch(&p.ws->ticket, 0u);
      atomicExch(&p.ws->epoch, e + 1u);
    }
    *s_ticket = t;
    *s_epoch = e;
  }
  uint32_t ticket, epoch;
  if (GATE) {
    cluster_sync();  // every CTA has started (DSMEM addressable) and rank 0 holds the ticket
    ticket = ld_cluster_u32(map_smem(s_ticket, 0));
    epoch = ld_cluster_u32(map_smem(s_epoch, 0));
  } else {
    __syncthreads();
    ticket = *s_ticket;
    epoch = *s_epoch;
  }
  int b, h, c;
  if (GATE) {
    c = (int)(ticket / p.B);
    b = (int)(ticket % p.B);
    h = (int)crank;
  } else {
    c = (int)(ticket / (p.B * p.H));
    const int rem = (int)(ticket % (p.B * p.H));
    b = rem / p.H;
    h = rem % p.H;
  }
  const int t0 = c * kL;

  // ---- 1. TMA load of the x tile --------------------------------------------
  if (tid == 0) {
    mbar_expect_tx(tma_bar, kL * 128);
    tma_load_3d(xs, &tmap, tma_bar, h * kHD, t0, b);
  }

  // ---- gate weights of this head's channels, bf16 hi/lo, swizzled ------------
  if (GATE) {
    const int n = tid >> 4;          // 0..15: rows 0-7 hi, 8-15 lo
    const int k0 = (tid & 15) * 4;   // channel within the head
    const int hh = n & 7;
    float w[4] = {0.f, 0.f, 0.f, 0.f};
    if (hh < p.H) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p.gate_w + (size_t)hh * p.D + h * kHD + k0));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
    uint16_t e16[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(w[q]);
      const float v = n < 8 ? w[q] : w[q] - __bfloat162float(hi);
      const __nv_bfloat16 o = n < 8 ? hi : __float2bfloat16_rn(v);
      e16[q] = *reinterpret_cast<const uint16_t*>(&o);
    }
    const int byte = k0 * 2;  // 8 bytes, inside one 16-byte chunk
    uint8_t* dst = wsm + n * 128 + ((((byte >> 4) ^ (n & 7))) << 4) + (byte & 15);
    *reinterpret_cast<uint2*>(dst) =
        make_uint2((uint32_t)e16[0] | ((uint32_t)e16[1] << 16), (uint32_t)e16[2] | ((uint32_t)e16[3] << 16));
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
  }

  // ---- coefficients (registers) -----------------------------------------------
  const int run = warp;       // 0..7: tokens run*32 .. run*32+31
  const int j0 = lane * 2;    // channel pair within the head
  const int ch0 = h * kHD + j0;
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;
  float2 cf[8];  // PRECISE: raw Chebyshev c_k; fast: gamma-folded monomial a_m
  {
    const float* cb = p.coeffs + ((size_t)(b * p.H + h) * p.K) * kHD + j0;
    float2 ck[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      ck[k] = make_float2(0.f, 0.f);
      if (k < p.K) ck[k] = __ldg(reinterpret_cast<const float2*>(cb + (size_t)k * kHD));
    }
    if (PRECISE) {
#pragma unroll
      for (int k = 0; k < 8; ++k) cf[k] = ck[k];
    } else {
      // T_0..T_7 in the monomial basis: sum_k c_k T_k(x) = sum_m a_m x^m
      const float2 g2 = make_float2(gamma, gamma);
      auto lin = [&](float w0, int k0, float w1, int k1, float w2, int k2, float w3, int k3) {
        float2 r = make_float2(0.f, 0.f);
        if (k0 >= 0) r = fma2(make_float2(w0, w0), ck[k0], r);
        if (k1 >= 0) r = fma2(make_float2(w1, w1), ck[k1], r);
        if (k2 >= 0) r = fma2(make_float2(w2, w2), ck[k2], r);
        if (k3 >= 0) r = fma2(make_float2(w3, w3), ck[k3], r);
        return mul2(r, g2);
      };
      cf[0] = lin(1.f, 0, -1.f, 2, 1.f, 4, -1.f, 6);
      cf[1] = lin(1.f, 1, -3.f, 3, 5.f, 5, -7.f, 7);
      cf[2] = lin(2.f, 2, -8.f, 4, 18.f, 6, 0.f, -1);
      cf[3] = lin(4.f, 3, -20.f, 5, 56.f, 7, 0.f, -1);
      cf[4] = lin(8.f, 4, -48.f, 6, 0.f, -1, 0.f, -1);
      cf[5] = lin(16.f, 5, -112.f, 7, 0.f, -1, 0.f, -1);
      cf[6] = lin(32.f, 6, 0.f, -1, 0.f, -1, 0.f, -1);
      cf[7] = lin(64.f, 7, 0.f, -1, 0.f, -1, 0.f, -1);
    }
  }
  if (GATE) {
    tc_fence_before();
    __syncthreads();  // wsm complete and the TMEM address visible before the MMA issue
  }

  // ---- wait for the tile ------------------------------------------------------
  bool ok_tma = mbar_wait(tma_bar, 0);

  // ---- 2. gate MMA issue (one thread) -----------------------------------------
  if (GATE) tc_fence_after();
  const uint32_t tmem = GATE ? *tmem_slot : 0u;
  if (GATE && tid == 0) {
    tc_fence_after();
    constexpr uint32_t idesc = umma_idesc_bf16(128, 16);
    const uint32_t xa = smem_u32(xs), wa = smem_u32(wsm);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + mt * 16, umma_desc_sw128(xa + mt * 128 * 128 + ks * 32), umma_desc_sw128(wa + ks * 32),
                  idesc, ks > 0 ? 1u : 0u);
    umma_commit(mma_bar);
  }

  // ---- 3a. evaluate u = tanh(gamma * y(xn)) into registers ---------------------
  float2 sl[kR];
  {
    const int cb16 = (lane >> 2), cofs = (lane & 3) * 4;  // 16-byte chunk, offset of this lane's pair
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int row = run * kR + r;
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(xs + row * 128 + ((cb16 ^ (row & 7)) << 4) + cofs);
      const float x0 = __uint_as_float(raw << 16), x1 = __uint_as_float(raw & 0xffff0000u);
      float2 xn;
      if (PRECISE) {
        float xa, sg;
        xn.x = softsign<true>(x0, false, xa, sg);
        xn.y = softsign<true>(x1, false, xa, sg);
      } else {
        xn = make_float2(x0 * rcp_fast(1.0f + fabsf(x0)), x1 * rcp_fast(1.0f + fabsf(x1)));  // x / (1 + |x|)
      }
      float2 y;
      if (PRECISE) {
        const float2 x2 = make_float2(2.f * xn.x, 2.f * xn.y);
        float2 u1 = cf[7], u2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 6; k >= 1; --k) {
          const float2 t = fma2(x2, u1, sub2(cf[k], u2));
          u2 = u1;
          u1 = t;
        }
        y = fma2(xn, u1, sub2(cf[0], u2));
        y = make_float2(y.x * gamma, y.y * gamma);
      } else {
        // Horner in the monomial basis, gamma already folded in
        y = cf[7];
#pragma unroll
        for (int m = 6; m >= 0; --m) y = fma2(y, xn, cf[m]);
      }
      const float z0 = fminf(fmaxf(y.x, -4.f), 4.f), z1 = fminf(fmaxf(y.y, -4.f), 4.f);
      const float u0 = PRECISE ? tanhf(z0) : tanh_fast(z0);
      const float u1v = PRECISE ? tanhf(z1) : tanh_fast(z1);
      sl[r] = make_float2(x0 == x0 ? u0 : 0.f, x1 == x1 ? u1v : 0.f);  // NaN input -> 0 (sdpc_kernel.py:1164)
    }
  }

  // ---- 2b. gate: partial logits -> owning CTA; lambda_t -------------------------
  const int tt = tid;  // token handled in the lambda fill
  const int tg = t0 + tt;
  if (GATE) {
    bool ok_mma = mbar_wait(mma_bar, 0);
    tc_fence_after();
    const int q4 = warp & 3, mt = warp >> 2;
    float v[16];
    tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + mt * 16, v);
    const int tok = mt * 128 + q4 * 32 + lane;
    for (int n = 0; n < p.H; ++n)
      st_cluster_f32(map_smem(part_s + crank * kL + tok, n), v[n] + v[n + 8]);
    if (!ok_mma) atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
    tc_fence_before();
    cluster_sync();  // all partials delivered
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 32);
    float logit = __ldg(p.gate_b + h);
    for (int s = 0; s < p.H; ++s) logit += part_s[s * kL + tt];
    const float sg = 1.0f / (1.0f + __expf(-logit));
    float lam = fminf(fmaxf(__ldg(p.lam_h + h) + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
    if (tg >= p.S) lam = 1.f;
    lam_s[tt] = tg >= p.S ? make_float4(1.f, 1.f, 0.f, 0.f) : make_float4(lam, lam, 1.f - lam, 1.f - lam);
  } else {
    float lam = p.lam_tok ? (tg < p.S ? __ldg(p.lam_tok + ((size_t)b * p.S + tg) * p.H + h) : 1.f)
                          : (p.lam_h ? __ldg(p.lam_h + h) : p.momentum);
    lam_s[tt] = tg >= p.S ? make_float4(1.f, 1.f, 0.f, 0.f) : make_float4(lam, lam, 1.f - lam, 1.f - lam);
  }
  if (!ok_tma && tid == 0) atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
  __syncthreads();

  // ---- 3b. local scan of each run -------------------------------------------------
  const int tbase = t0 + run * kR;
  float Arun = 1.f;
  {
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const float4 lm = lam_s[run * kR + r];
      if (tbase + r == 0) {
        // first token of the sequence: fold the carried-in state with its clamp
        const float2 iv = p.init ? __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * p.D + ch0))
                                 : make_float2(0.f, 0.f);
        s2 = make_float2(clamp1(fmaf(lm.x, iv.x, lm.z * sl[r].x)), clamp1(fmaf(lm.x, iv.y, lm.z * sl[r].y)));
        Arun = 0.f;
      } else {
        s2 = fma2(make_float2(lm.x, lm.y), s2, mul2(make_float2(lm.z, lm.w), sl[r]));
        Arun *= lm.x;
      }
      sl[r] = s2;
    }
    *reinterpret_cast<float2*>(aggB_s + run * kHD + j0) = s2;
    if (lane == 0) aggA_s[run] = Arun;
  }
  __syncthreads();

  // ---- 4. combine runs, publish, look back -------------------------------------------
  const size_t n = (size_t)(b * p.H + h) * p.nchunks + c;
  float chunkB = 0.f, chunkA = 1.f;
  if (tid < kHD) {
    float Bv = 0.f, Av = 1.f;
#pragma unroll
    for (int q = 0; q < kRUNS; ++q) {
      const float aq = aggA_s[q];
      const float bq = aggB_s[q * kHD + tid];
      aggB_s[q * kHD + tid] = Bv;
      if (tid == 0) exclA_s[q] = Av;
      Bv = fmaf(aq, Bv, bq);
      Av *= aq;
    }
    chunkB = Bv;
    chunkA = Av;
    if (c > 0) {
      p.aggB[n * kHD + tid] = chunkB;
      if (tid == 0) p.aggA[n] = chunkA;
    }
  }
  __syncthreads();
  // the CTA's writes are ordered before the flag by the barrier plus a
  // gpu-scope release fence in the publishing thread
  if (c > 0 && tid == 0) {
    __threadfence();
    st_release(p.lbflag + n, (epoch << 2) | 1u);
  }
  if (c > 0 && warp == 0) {
    // warp-wide window: lane i probes chunk (base - i); nearest inclusive wins
    int base = c - 1, kincl = -1;
    bool ok = true;
    while (kincl < 0) {
      const int j = base - lane;
      uint32_t st = 0;
      if (j >= 0) st = wait_flag(p.lbflag + (n - (size_t)(c - j)), epoch);
      if (__ballot_sync(0xffffffffu, j >= 0 && st == 0)) {
        ok = false;
        break;
      }
      const uint32_t m2 = __ballot_sync(0xffffffffu, j >= 0 && st == 2);
      if (m2) kincl = base - (__ffs(m2) - 1);
      else base -= 32;
    }
    if (lane == 0) *s_kincl = ok ? kincl : -1;
  }
  __syncthreads();
  if (tid < kHD) {
    float X = 0.f;
    if (c > 0) {
      const int k = *s_kincl;
      if (k >= 0) {
        X = __ldcg(p.incB + (n - (size_t)(c - k)) * kHD + tid);
        // fold forward 4 chunks at a time; the loads do not depend on X
        int j = k + 1;
        for (; j + 4 <= c; j += 4) {
          float aa[4], bb[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const size_t nj = n - (size_t)(c - (j + u));
            aa[u] = __ldcg(p.aggA + nj);
            bb[u] = __ldcg(p.aggB + nj * kHD + tid);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) X = fmaf(aa[u], X, bb[u]);
        }
        for (; j < c; ++j) {
          const size_t nj = n - (size_t)(c - j);
          X = fmaf(__ldcg(p.aggA + nj), X, __ldcg(p.aggB + nj * kHD + tid));
        }
      } else if (tid == 0) {
        atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
        atomicAdd(&p.ws->timeouts, 1u);
      }
    }
    carry_s[tid] = X;
    p.incB[n * kHD + tid] = fmaf(chunkA, X, chunkB);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    st_release(p.lbflag + n, (epoch << 2) | 2u);
  }

  // ---- 5. outputs -----------------------------------------------------------------
  {
    const float ea = exclA_s[run];
    const float2 cv = *reinterpret_cast<const float2*>(carry_s + j0);
    const float2 eb = *reinterpret_cast<const float2*>(aggB_s + run * kHD + j0);
    const float2 rc = make_float2(fmaf(ea, cv.x, eb.x), fmaf(ea, cv.y, eb.y));
    OT* ob = reinterpret_cast<OT*>(p.out) + (size_t)b * p.osb + ch0;
    float2 A2 = make_float2(1.f, 1.f);
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int t = tbase + r;
      const float4 lm = lam_s[run * kR + r];
      A2 = mul2(A2, make_float2(lm.x, lm.y));
      float2 o = fma2(A2, rc, sl[r]);
      if (sizeof(OT) == 4) o = make_float2(clamp1(o.x), clamp1(o.y));
      if (t < p.S) {
        st2(ob + (size_t)t * p.oss, o);
        if (t == p.S - 1 && p.fin)
          *reinterpret_cast<float2*>(p.fin + (size_t)b * p.D + ch0) = make_float2(clamp1(o.x), clamp1(o.y));
      }
    }
  }
  // Every DSMEM access (ticket broadcast, partial logits) precedes the second
  // cluster barrier above, so CTAs may leave independently.
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

template <bool GATE, bool PRECISE, typename OT>
cudaError_t launch(const CUtensorMap& map, const Params& p, int nctas, cudaStream_t st) {
  auto kern = fwd_tc_kernel<GATE, PRECISE, OT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nctas, 1, 1);
  cfg.blockDim = dim3(kNT, 1, 1);
  cfg.dynamicSmemBytes = kSmemAlloc;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = GATE ? p.H : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = GATE ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, map, p);
}

}  // namespace tc
}  // namespace ossm

using namespace ossm;

// Eligibility of the TMA / tcgen05 path for these arguments.
bool ossm_tc_eligible(const ossm_fwd_args* a) {
  if (a->x_dtype != OSSM_BF16 || a->head_dim != 64 || a->tanh_out) return false;
  if ((a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_LUT || (a->flags & (OSSM_F_FASTPATH | OSSM_F_GENERIC))) return false;
  if (((uintptr_t)a->x % 16) || (a->x_stride_s % 8) || (a->B > 1 && (a->x_stride_b % 8))) return false;
  if (a->gate_w && !a->lam_tok && a->H > tc::kMaxH) return false;
  if (a->S > (1 << 30)) return false;
  return tc::encode_fn() != nullptr;
}

// Launch of the TMA / tcgen05 path (same workspace layout as the generic path:
// header, flags[N], aggA[N], aggB[N][64], incB[N][64] with N = B*H*nchunks).
int ossm_tc_launch(const ossm_fwd_args* a, char* ws, size_t off_flag, size_t off_aggA, size_t off_aggB,
                   size_t off_incB, cudaStream_t st) {
  using namespace tc;
  Params p;
  p.B = a->B;
  p.S = a->S;
  p.H = a->H;
  p.K = a->degree;
  p.nchunks = (a->S + kL - 1) / kL;
  p.D = a->H * kHD;
  p.coeffs = a->coeffs;
  p.lam_h = a->lam_h;
  p.momentum = a->momentum;
  const bool gate = a->gate_w && !a->lam_tok;
  p.gate_w = a->gate_w;
  p.gate_b = a->gate_b;
  p.gate_scale = a->gate_scale;
  p.gate_lo = a->gate_lo;
  p.gate_hi = a->gate_hi;
  p.lam_tok = a->lam_tok;
  p.init = a->init_state;
  p.fin = a->final_state;
  p.out = a->out;
  p.osb = a->out_stride_b;
  p.oss = a->out_stride_s;
  p.ws = reinterpret_cast<WsHeader*>(ws);
  p.lbflag = reinterpret_cast<uint32_t*>(ws + off_flag);
  p.aggA = reinterpret_cast<float*>(ws + off_aggA);
  p.aggB = reinterpret_cast<float*>(ws + off_aggB);
  p.incB = reinterpret_cast<float*>(ws + off_incB);
  const long long nctas = (long long)a->B * a->H * p.nchunks;
  if (nctas > 0x7fffffffLL) return OSSM_EINVAL;
  p.nunits = (uint32_t)(gate ? (long long)a->B * p.nchunks : nctas);

  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)p.D, (cuuint64_t)a->S, (cuuint64_t)a->B};
  const long long sb = a->B > 1 ? a->x_stride_b : (long long)a->S * a->x_stride_s;
  cuuint64_t strides[2] = {(cuuint64_t)a->x_stride_s * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[3] = {(cuuint32_t)kHD, (cuuint32_t)kL, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a->x), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return OSSM_EINVAL;
  const bool precise = (a->out_dtype == OSSM_F32) || (a->flags & OSSM_F_PRECISE);
  cudaError_t e;
  if (a->out_dtype == OSSM_F32) {
    e = gate ? launch<true, true, float>(map, p, (int)nctas, st) : launch<false, true, float>(map, p, (int)nctas, st);
  } else if (precise) {
    e = gate ? launch<true, true, __nv_bfloat16>(map, p, (int)nctas, st)
             : launch<false, true, __nv_bfloat16>(map, p, (int)nctas, st);
  } else {
    e = gate ? launch<true, false, __nv_bfloat16>(map, p, (int)nctas, st)
             : launch<false, false, __nv_bfloat16>(map, p, (int)nctas, st);
  }
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
