// Device pieces shared by the bf16 fast-path forward kernels (three-pass and
// single-pass): softsign, the degree-<=8 evaluation, the EMA step and the
// tensor-core gate.  Arithmetic contract of _fused_clenshaw_ema_kernel,
// sdpc_kernel.py:988-1209.
#pragma once

#include "ossm_sm100.cuh"

namespace ossm {
namespace ev {

constexpr int kL = 32;  // tokens per chunk

OSSM_DEV float clamp4_nan(float v) {  // NaN-propagating clamp to [-4, 4]
  float r;
  asm("max.NaN.f32 %0, %1, 0fC0800000;\n\tmin.NaN.f32 %0, %0, 0f40800000;" : "=f"(r) : "f"(v));
  return r;
}
// z = 4 xn = x / (1/4 + |x|/4) with one flush-to-zero reciprocal (three
// instructions; 1/4 + |x|/4 stays below 2^126 for every bf16 or finite fp32
// input of interest, so the reciprocal is never flushed).  xn is the
// reference's softsign sign(x) (1 - 1/(1 + |x|)) (sdpc_kernel.py:1078-1085);
// its 1e-7 floor on |x| moves xn by < 2e-7.  NaN and +-inf come out as NaN, so
// they reach the per-chunk check.
OSSM_DEV float softsign4_fast(float x) { return x * rcp_fast(fmaf(fabsf(x), 0.25f, 0.25f)); }

// Chebyshev -> monomial coefficients with gamma folded in (T_0..T_7 written out).
OSSM_DEV void cheb_to_mono(const float2 (&ck)[8], float gamma, float2 (&a)[8]) {
  const float2 g2 = make_float2(gamma, gamma);
  auto w = [](float v) { return make_float2(v, v); };
  a[0] = mul2(fma2(w(-1.f), ck[6], fma2(w(1.f), ck[4], fma2(w(-1.f), ck[2], ck[0]))), g2);
  a[1] = mul2(fma2(w(-7.f), ck[7], fma2(w(5.f), ck[5], fma2(w(-3.f), ck[3], ck[1]))), g2);
  a[2] = mul2(fma2(w(18.f), ck[6], fma2(w(-8.f), ck[4], mul2(w(2.f), ck[2]))), g2);
  a[3] = mul2(fma2(w(56.f), ck[7], fma2(w(-20.f), ck[5], mul2(w(4.f), ck[3]))), g2);
  a[4] = mul2(fma2(w(-48.f), ck[6], mul2(w(8.f), ck[4])), g2);
  a[5] = mul2(fma2(w(-112.f), ck[7], mul2(w(16.f), ck[5])), g2);
  a[6] = mul2(mul2(w(32.f), ck[6]), g2);
  a[7] = mul2(mul2(w(64.f), ck[7]), g2);
}

// The lane's two channels (j0, j0+1 of head h; 8 heads of 64) of the
// coefficients [B,8,Kd,64] (Kd = the tensor's degree), of which the first K
// are used (K < Kd in the degree-4 truncation mode): raw (precise), or
// gamma-folded monomial scaled by
// 4^-k for Horner in z = 4 xn (power-of-two scaling: the same roundings as
// Horner in xn on the unscaled monomial coefficients).
// Held as (channel j0, channel j0+1) pairs, the operand layout of the packed
// fp32x2 Horner.
template <bool PRECISE>
OSSM_DEV void load_coeffs(const float* coeffs, int Kd, int K, int b, int h, int j0, float gamma, float2 (&m)[8]) {
  const float* cb = coeffs + ((size_t)(b * 8 + h) * Kd) * 64 + j0;
  float2 ck[8], cf[8];
#pragma unroll
  for (int q = 0; q < 8; ++q)
    ck[q] = q < K ? __ldg(reinterpret_cast<const float2*>(cb + q * 64)) : make_float2(0.f, 0.f);
  if (PRECISE) {
#pragma unroll
    for (int q = 0; q < 8; ++q) cf[q] = ck[q];
  } else {
    cheb_to_mono(ck, gamma, cf);
    float sc = 1.f;
#pragma unroll
    for (int q = 0; q < 8; ++q, sc *= 0.25f) cf[q] = make_float2(cf[q].x * sc, cf[q].y * sc);
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) m[q] = cf[q];
}

// u = tanh(clamp(gamma y(xn), +-4)) for one channel of one token.
// EXACT: the reference's semantics for every input (NaN -> u = 0,
// sdpc_kernel.py:1164; +-inf -> xn = +-1, :1078-1085).  Otherwise a NaN input
// comes out as NaN (caught per chunk); every other input takes the
// reference's formula either way.
template <bool PRECISE, bool EXACT>
OSSM_DEV float eval_u1(float x, const float2 (&m)[8], bool second, float gamma) {
  auto c = [&](int q) { return second ? m[q].y : m[q].x; };
  float xn;  // xn (precise) or z = 4 xn (fast coefficients)
  if (PRECISE || EXACT) {
    float xa, sg;
    xn = softsign<PRECISE>(x, false, xa, sg);
    if (!EXACT && x != x) xn = x;
    if (!PRECISE) xn *= 4.f;
  } else {
    xn = softsign4_fast(x);
  }
  float y;
  if (PRECISE) {  // Clenshaw on the raw coefficients, then gamma
    const float x2 = 2.f * xn;
    float u1 = c(7), u2 = 0.f;
#pragma unroll
    for (int q = 6; q >= 1; --q) {
      const float tt = fmaf(x2, u1, c(q) - u2);
      u2 = u1;
      u1 = tt;
    }
    y = fmaf(xn, u1, c(0) - u2) * gamma;
  } else {  // Horner in z = 4 xn on the gamma-folded, 4^-k-scaled monomial coefficients
    y = c(7);
#pragma unroll
    for (int q = 6; q >= 0; --q) y = fmaf(y, xn, c(q));
  }
  if (EXACT) {  // a NaN y (from the coefficients) stays NaN, as in the reference's clamp (:1160-1161)
    const float z = clamp4_nan(y);
    return x != x ? 0.f : (PRECISE ? tanhf(z) : tanh_fast(z));
  }
  const float z = clamp4_nan(y);
  return PRECISE ? tanhf(z) : tanh_fast(z);
}
// Both channels of one token.  The fast path runs its Horner on the channel
// pair with packed fp32x2 FMAs (one instruction per degree for two channels).
template <bool PRECISE, bool EXACT>
OSSM_DEV float2 eval_u(uint32_t raw, const float2 (&m)[8], float gamma) {
  const float x0 = __uint_as_float(raw << 16), x1 = __uint_as_float(raw & 0xffff0000u);
  if (!PRECISE && !EXACT) {
    const float2 z = mul2(make_float2(x0, x1), make_float2(rcp_fast(fmaf(fabsf(x0), 0.25f, 0.25f)),
                                                           rcp_fast(fmaf(fabsf(x1), 0.25f, 0.25f))));
    float2 y = m[7];
#pragma unroll
    for (int q = 6; q >= 0; --q) y = fma2(y, z, m[q]);
    return make_float2(tanh_fast(clamp4_nan(y.x)), tanh_fast(clamp4_nan(y.y)));
  }
  return make_float2(eval_u1<PRECISE, EXACT>(x0, m, false, gamma), eval_u1<PRECISE, EXACT>(x1, m, true, gamma));
}

OSSM_DEV float clamp1_nan(float v) {  // NaN-propagating clamp to [-1, 1]
  float r;
  asm("max.NaN.f32 %0, %1, 0fBF800000;\n\tmin.NaN.f32 %0, %0, 0f3F800000;" : "=f"(r) : "f"(v));
  return r;
}

// s <- l s + (1 - l) u; token 0 of the sequence (first) folds the carried-in
// state with the reference's clamp.  The clamp lets NaN through, so a NaN u
// of the fast evaluation still reaches the per-chunk check.
OSSM_DEV float2 ema_step(float2 s, float2 lm, float2 u, bool first) {  // lm = (l, 1 - l)
  if (first) return make_float2(clamp1_nan(fmaf(lm.x, s.x, lm.y * u.x)), clamp1_nan(fmaf(lm.x, s.y, lm.y * u.y)));
  return fma2(make_float2(lm.x, lm.x), s, mul2(make_float2(lm.y, lm.y), u));
}

// The 32-token EMA of one chunk from state s (decays lam[0..31]); RAW(t) gives
// the packed bf16 pair of token t, OUT(t, s) receives each state.
template <bool PRECISE, bool EXACT, typename RawF, typename OutF>
OSSM_DEV float2 ema_chunk(float2 s, const float2* lam, bool first, const float2 (&m)[8], float gamma, RawF raw,
                          OutF out) {
#pragma unroll
  for (int t = 0; t < kL; ++t) {
    s = ema_step(s, lam[t], eval_u<PRECISE, EXACT>(raw(t), m, gamma), t == 0 && first);
    out(t, s);
  }
  return s;
}
// The same with the reference's NaN / inf semantics as a rolled loop (the rare
// recompute of a chunk that held such inputs).
template <bool PRECISE, typename RawF, typename OutF>
OSSM_DEV float2 ema_chunk_exact(float2 s, const float2* lam, bool first, const float2 (&m)[8], float gamma, RawF raw,
                                OutF out) {
#pragma unroll 1
  for (int t = 0; t < kL; ++t) {
    s = ema_step(s, lam[t], eval_u<PRECISE, true>(raw(t), m, gamma), t == 0 && first);
    out(t, s);
  }
  return s;
}

// The same two loops, handing each token's u to U(t, u) as well (the
// aggregate pass parks u for the output pass).
template <bool PRECISE, bool EXACT, typename RawF, typename UF>
OSSM_DEV float2 ema_chunk_u(float2 s, const float2* lam, bool first, const float2 (&m)[8], float gamma, RawF raw,
                            UF uf) {
#pragma unroll
  for (int t = 0; t < kL; ++t) {
    const float2 u = eval_u<PRECISE, EXACT>(raw(t), m, gamma);
    uf(t, u);
    s = ema_step(s, lam[t], u, t == 0 && first);
  }
  return s;
}
template <bool PRECISE, typename RawF, typename UF>
OSSM_DEV float2 ema_chunk_u_exact(float2 s, const float2* lam, bool first, const float2 (&m)[8], float gamma,
                                  RawF raw, UF uf) {
#pragma unroll 1
  for (int t = 0; t < kL; ++t) {
    const float2 u = eval_u<PRECISE, true>(raw(t), m, gamma);
    uf(t, u);
    s = ema_step(s, lam[t], u, t == 0 && first);
  }
  return s;
}

OSSM_DEV void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
OSSM_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of (token t, 16-byte chunk j) in a head's 128-byte-swizzled box
OSSM_DEV uint32_t box_off(int t, int j) { return (uint32_t)(t * 128 + ((j ^ (t & 7)) << 4)); }

}  // namespace ev
}  // namespace ossm
