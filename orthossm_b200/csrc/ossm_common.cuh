// Device helpers shared by the orthossm_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "orthossm_b200.h"

#define OSSM_DEV __device__ __forceinline__

namespace ossm {

// ---------------------------------------------------------------------------
// vector I/O: 4 consecutive channels per thread
// ---------------------------------------------------------------------------
OSSM_DEV float4 ld4(const float* p) {  // streaming read, 16 B
  return __ldcs(reinterpret_cast<const float4*>(p));
}
OSSM_DEV float4 ld4(const __nv_bfloat16* p) {  // streaming read, 8 B
  uint2 u = __ldcs(reinterpret_cast<const uint2*>(p));
  float4 r;
  r.x = __uint_as_float(u.x << 16);
  r.y = __uint_as_float(u.x & 0xffff0000u);
  r.z = __uint_as_float(u.y << 16);
  r.w = __uint_as_float(u.y & 0xffff0000u);
  return r;
}
OSSM_DEV void st4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }
OSSM_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
OSSM_DEV void st4(__nv_bfloat16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  __stcs(reinterpret_cast<uint2*>(p), u);
}
OSSM_DEV void st2(float* p, float2 v) { __stcs(reinterpret_cast<float2*>(p), v); }
OSSM_DEV void st2(__nv_bfloat16* p, float2 v) {
  __stcs(reinterpret_cast<unsigned int*>(p), pack_bf16x2(v.x, v.y));
}
OSSM_DEV float bf16_round(float v) {  // round-to-nearest-even to bf16, as float
  return __bfloat162float(__float2bfloat16_rn(v));
}

OSSM_DEV float get(const float4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// ---------------------------------------------------------------------------
// elementwise math
// ---------------------------------------------------------------------------
// tanh.approx.f32 (one MUFU op; documented max relative error ~2^-11),
// used only where the result is rounded to bf16.
OSSM_DEV float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
OSSM_DEV float rcp_fast(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
OSSM_DEV float clamp1(float v) { return fminf(fmaxf(v, -1.0f), 1.0f); }

// Packed two-lane fp32 arithmetic of sm_100 (PTX .f32x2): one instruction for
// two channels, same round-to-nearest result as the scalar fmaf/__fsub_rn.
OSSM_DEV float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
OSSM_DEV float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
OSSM_DEV float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Softsign magnitude and sign of sdpc_kernel.py:1078-1085 ("fused"
// semantics: NaN treated as 0, sign(0) = +1) or :1722-1725 ("torch":
// sign(0) = 0, NaN -> 0).  Returns xn; writes |xn| and the sign.
template <bool PRECISE>
OSSM_DEV float softsign(float x, bool torch_sem, float& xa, float& sgn) {
  const bool nan = x != x;
  const float xs = nan ? 0.0f : x;
  // |x| is capped at 2^64, where m / (1 + m) is already 1 in fp32, so that
  // +-inf and the largest finite inputs give +-1 as the reference's form does.
  const float m = fminf(fmaxf(fabsf(xs), 1e-7f), 0x1p64f);
  // m / (1 + m) == 1 - 1/(1 + m) without the cancellation of the latter.
  xa = PRECISE ? __fdiv_rn(m, 1.0f + m) : m * rcp_fast(1.0f + m);
  sgn = xs >= 0.0f ? 1.0f : -1.0f;
  if (torch_sem && (xs == 0.0f)) sgn = 0.0f;
  return sgn * xa;
}

// ---------------------------------------------------------------------------
// bounded spin on a look-back flag
// ---------------------------------------------------------------------------
OSSM_DEV uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
OSSM_DEV void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Workspace header shared by the kernels that use decoupled look-back.
struct WsHeader {
  uint32_t ticket;  // CTA ticket counter; reset to 0 by the last CTA of a launch
  uint32_t epoch;   // launch counter tagging look-back flags; advanced by the last CTA
  uint32_t status;  // sticky error word (OSSM_ETIMEOUT), cleared by the host
  uint32_t timeouts;
  uint32_t exited;  // persistent units that have left (the last one resets ticket/epoch)
  uint32_t pad[59];
};
static_assert(sizeof(WsHeader) == 256, "header is one 256-byte block");

constexpr uint32_t kSpinLimit = 1u << 21;  // ~0.1-0.5 s with backoff, then give up

// Wait until flag carries `epoch` and a non-zero state; return the state
// (1 = aggregate, 2 = inclusive prefix) or 0 on timeout.
OSSM_DEV uint32_t wait_flag(const uint32_t* flag, uint32_t epoch) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    const uint32_t f = ld_acquire(flag);
    if ((f >> 2) == (epoch & 0x3fffffffu) && (f & 3u)) return f & 3u;
    if (it > 64) __nanosleep(it > 4096 ? 256 : 32);
  }
  return 0;
}

}  // namespace ossm
