// Forward fast path for bf16 activations, 8 heads x head_dim 64 (sm_100a).
//
// Same arithmetic contract as fwd_scan_kernel in ossm_forward.cu (which
// restates _fused_clenshaw_ema_kernel, sdpc_kernel.py:988-1209); this file only
// changes how the work is mapped onto the B200:
//
//   work item = (batch b, chunk c of 32 tokens, all 8 heads): eight TMA loads,
//     one [32 tokens x 64 channels] bf16 box per head (128-byte swizzle), into
//     a 32 KB [head][token] tile, double-buffered;
//   schedule = a persistent grid of (CTAs per SM x SMs) units; unit u takes items
//     u, u+G, u+2G, ... in order (items chunk-major), so an item's predecessor
//     in its (b, h) chain is always an earlier or concurrent item of a resident
//     unit;
//   warp w = head w, lane = 2 channels, 32 tokens per lane:
//     u = tanh(clamp(gamma y(xn), +-4)) with packed f32x2 Horner, local scan,
//     then a warp-local decoupled look-back over (value, tag) 64-bit records
//     (single-copy atomic: no fences, no CTA barrier), outputs;
//   gate (optional) = per item a [32 tokens x 512] . [512 x 8 heads] product on
//     the tensor cores (mma.sync m16n8k16, bf16 x exact, weights split into
//     bf16 hi + lo), each warp over its own head's 64 channels, summed across
//     warps in shared memory;
//   bf16 outputs are written into the consumed tile and leave by a TMA store.
//
// The carry fold order depends on how far back the nearest inclusive record
// is when an item looks, so results are reproducible to fp32 rounding of the
// carry, not bitwise; the generic kernel in ossm_forward.cu is bitwise
// reproducible.
#include <cudaTypedefs.h>

#include <mutex>

#include "ossm_sm100.cuh"

namespace ossm {
namespace fast {

constexpr int kNT = 256;
constexpr int kH = 8;        // heads (one warp each)
constexpr int kHD = 64;      // channels per head
constexpr int kD = kH * kHD;
constexpr int kL = 32;       // tokens per item
constexpr int kTile = kL * kH * 128;  // 32 KB: row = head*32 + token, 128 B per row
constexpr int kWRow = 520;            // gate-weight row pitch in bf16 (1040 B: conflict-free ldmatrix)

// shared memory (bytes from a 1024-aligned base)
constexpr int kOffX = 0;                                // 2 tiles
constexpr int kOffW = kOffX + 2 * kTile;                // [2 hi/lo][8][kWRow] bf16
constexpr int kOffLam = kOffW + 2 * kH * kWRow * 2;     // [8 heads][32 tokens] float4
constexpr int kOffPart = kOffLam + kH * kL * 16;        // [8 warps][32 tokens][8] f32
constexpr int kOffBar = kOffPart + kH * kL * kH * 4;    // mbarriers
constexpr int kSmemBytes = kOffBar + 64;
constexpr int kSmemAlloc = kSmemBytes + 1024;

struct Params {
  int B, S, K, nchunks;
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
  unsigned long long* inc;   // [N][64] (inclusive state | tag)
  unsigned long long* agg;   // [N][64] (chunk aggregate state | tag)
  unsigned long long* aggA;  // [N] (chunk decay product | tag)
  uint32_t nitems;
};

OSSM_DEV unsigned long long pack_rec(float v, uint32_t tag) {
  return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
OSSM_DEV void st_rec(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
OSSM_DEV unsigned long long ld_rec(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
OSSM_DEV uint32_t rec_tag(unsigned long long v) { return (uint32_t)(v >> 32); }
OSSM_DEV float rec_val(unsigned long long v) { return __uint_as_float((uint32_t)v); }

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

// byte offset of (token t, head h, 16-byte chunk j) in the tile: each head's
// [32 x 128 B] box is 128-byte swizzled (chunk ^= row & 7), so 8 consecutive
// tokens of one head fall in 8 different bank groups
OSSM_DEV uint32_t tile_off(int t, int h, int j) { return (uint32_t)((h * kL + t) * 128 + ((j ^ (t & 7)) << 4)); }

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

template <bool GATE, bool PRECISE, typename OT>
__global__ void __launch_bounds__(kNT, 2)
    fwd_fast_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_o,
                    const Params p) {
  using namespace sm100;
  constexpr bool kTmaOut = sizeof(OT) == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* wsm = reinterpret_cast<__nv_bfloat16*>(sm + kOffW);
  float4* lam_s = reinterpret_cast<float4*>(sm + kOffLam);
  float* part_s = reinterpret_cast<float*>(sm + kOffPart);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [2]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int h = warp;
  const int j0 = lane * 2;
  const int ch0 = h * kHD + j0;
  const float gamma = 0.98f - 0.06f * (float)h / (float)kH;
  const uint32_t G = gridDim.x;
  const uint32_t u = blockIdx.x;

  const uint32_t epoch = atomicAdd(&p.ws->epoch, 0u);  // advanced only after every unit has left
  const uint32_t tag_agg = (epoch << 2) | 1u, tag_inc = (epoch << 2) | 2u;

  auto issue_load = [&](uint32_t k, int buf) {
    const int c = (int)(k / p.B), b = (int)(k % p.B);
    mbar_expect_tx(bar + buf, kTile);
#pragma unroll
    for (int hh = 0; hh < kH; ++hh)
      tma_load_3d(sm + kOffX + buf * kTile + hh * (kL * 128), &tmap_x, bar + buf, hh * kHD, c * kL, b);
  };
  if (tid == 0) {
    mbar_init(bar + 0, 1);
    mbar_init(bar + 1, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    if (kTmaOut) prefetch_tmap(&tmap_o);
    if (u < p.nitems) issue_load(u, 0);
    if (u + G < p.nitems) issue_load(u + G, 1);
  }
  if (GATE) {
    // gate weights as bf16 hi / lo, rows = target head, pitch kWRow
    for (int i = tid; i < kH * kD; i += kNT) {
      const int n = i / kD, k = i % kD;
      const float w = __ldg(p.gate_w + (size_t)n * kD + k);
      const __nv_bfloat16 hi = __float2bfloat16_rn(w);
      wsm[n * kWRow + k] = hi;
      wsm[kH * kWRow + n * kWRow + k] = __float2bfloat16_rn(w - __bfloat162float(hi));
    }
  }
  __syncthreads();

  float2 cf[8];
  int cur_b = -1;
  bool ok = true;
  uint32_t pend_k = 0xffffffffu;  // item whose tile the previous iteration left to load
  const uint32_t wbase = smem_u32(wsm);

  for (uint32_t k = u, it = 0; k < p.nitems; k += G, ++it) {
    const int buf = (int)(it & 1u);
    uint8_t* xs = sm + kOffX + buf * kTile;
    const int c = (int)(k / p.B), b = (int)(k % p.B);
    const int t0 = c * kL;

    if (b != cur_b) {  // coefficients of (b, h): raw (precise) or gamma-folded monomial
      cur_b = b;
      const float* cb = p.coeffs + ((size_t)(b * kH + h) * p.K) * kHD + j0;
      float2 ck[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        ck[q] = q < p.K ? __ldg(reinterpret_cast<const float2*>(cb + q * kHD)) : make_float2(0.f, 0.f);
      if (PRECISE) {
#pragma unroll
        for (int q = 0; q < 8; ++q) cf[q] = ck[q];
      } else {
        cheb_to_mono(ck, gamma, cf);
      }
    }
    float lam_in = 1.f;  // caller's per-token decay for token (t0 + lane), head h
    if (!GATE) {
      const int tg = t0 + lane;
      lam_in = p.lam_tok ? (tg < p.S ? __ldg(p.lam_tok + ((size_t)b * p.S + tg) * kH + h) : 1.f)
                         : (p.lam_h ? __ldg(p.lam_h + h) : p.momentum);
    }

    ok &= mbar_wait(bar + buf, (it >> 1) & 1u);
    const uint32_t xa = smem_u32(xs);

    // ---- gate: partial logits of this head's 64 channels on the tensor cores ----
    if (GATE) {
      const int m = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t a[4], bw[4];
          // A: tokens mt*16 + (m&1)*8 + rr, channels ks*16 + (m>>1)*8 of head h
          ldmatrix_x4(xa + tile_off(mt * 16 + (m & 1) * 8 + rr, h, ks * 2 + (m >> 1)), a);
          // B: weight rows n = rr, channels h*64 + ks*16 + (m&1)*8; lanes 0-15 hi, 16-31 lo
          const int kk = h * kHD + ks * 16 + (m & 1) * 8;
          ldmatrix_x4(wbase + (uint32_t)(((m >> 1) * kH * kWRow + rr * kWRow + kk) * 2), bw);
          mma_bf16_16816(d, a, bw[0], bw[1]);
          mma_bf16_16816(d, a, bw[2], bw[3]);
        }
        const int gid = lane >> 2, tig = lane & 3;
        float* pw = part_s + h * (kL * kH);
        pw[(mt * 16 + gid) * kH + 2 * tig] = d[0];
        pw[(mt * 16 + gid) * kH + 2 * tig + 1] = d[1];
        pw[(mt * 16 + gid + 8) * kH + 2 * tig] = d[2];
        pw[(mt * 16 + gid + 8) * kH + 2 * tig + 1] = d[3];
      }
      __syncthreads();
      {
        const int t = tid >> 3, n = tid & 7;
        float logit = __ldg(p.gate_b + n);
#pragma unroll
        for (int g = 0; g < kH; ++g) logit += part_s[g * (kL * kH) + t * kH + n];
        const float sg = 1.0f / (1.0f + __expf(-logit));
        const float lam = fminf(fmaxf(__ldg(p.lam_h + n) + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
        lam_s[n * kL + t] =
            (t0 + t) < p.S ? make_float4(lam, lam, 1.f - lam, 1.f - lam) : make_float4(1.f, 1.f, 0.f, 0.f);
      }
      __syncthreads();
    } else {
      lam_s[h * kL + lane] = (t0 + lane) < p.S ? make_float4(lam_in, lam_in, 1.f - lam_in, 1.f - lam_in)
                                               : make_float4(1.f, 1.f, 0.f, 0.f);
      __syncwarp();
    }

    // ---- u for 32 tokens, local scan ----------------------------------------------
    float2 sl[kL];
#pragma unroll
    for (int t = 0; t < kL; ++t) {
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(xs + tile_off(t, h, lane >> 2) + (lane & 3) * 4);
      const float x0 = __uint_as_float(raw << 16), x1 = __uint_as_float(raw & 0xffff0000u);
      float2 xn;
      if (PRECISE) {
        float xa_, sg;
        xn.x = softsign<true>(x0, false, xa_, sg);
        xn.y = softsign<true>(x1, false, xa_, sg);
      } else {
        // x / (1 + |x|) with |x| capped at 2^64, so +-inf and |x| >= 2^126 give +-1
        // (NaN is zeroed below)
        const float m0 = fminf(fabsf(x0), 0x1p64f), m1 = fminf(fabsf(x1), 0x1p64f);
        xn = make_float2(copysignf(m0 * rcp_fast(1.0f + m0), x0), copysignf(m1 * rcp_fast(1.0f + m1), x1));
      }
      float2 y;
      if (PRECISE) {
        const float2 x2 = make_float2(2.f * xn.x, 2.f * xn.y);
        float2 u1 = cf[7], u2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 6; q >= 1; --q) {
          const float2 tt = fma2(x2, u1, sub2(cf[q], u2));
          u2 = u1;
          u1 = tt;
        }
        y = fma2(xn, u1, sub2(cf[0], u2));
        y = make_float2(y.x * gamma, y.y * gamma);
      } else {
        y = cf[7];
#pragma unroll
        for (int q = 6; q >= 0; --q) y = fma2(y, xn, cf[q]);
      }
      const float z0 = fminf(fmaxf(y.x, -4.f), 4.f), z1 = fminf(fmaxf(y.y, -4.f), 4.f);
      const float u0 = PRECISE ? tanhf(z0) : tanh_fast(z0);
      const float u1v = PRECISE ? tanhf(z1) : tanh_fast(z1);
      sl[t] = make_float2(x0 == x0 ? u0 : 0.f, x1 == x1 ? u1v : 0.f);  // NaN input -> 0 (sdpc_kernel.py:1164)
    }
    // the next tile into the other buffer, once the previous item's store has read it
    if (tid == 0 && pend_k < p.nitems) {
      if (kTmaOut) bulk_wait_read0();
      issue_load(pend_k, buf ^ 1);
    }
    // local scan: token 0 of the sequence folds the carried-in state (with its clamp)
    float2 s2;
    float A;
    {
      const float4 lm = lam_s[h * kL];
      if (t0 == 0) {
        const float2 iv = p.init ? __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + ch0))
                                 : make_float2(0.f, 0.f);
        s2 = make_float2(clamp1(fmaf(lm.x, iv.x, lm.z * sl[0].x)), clamp1(fmaf(lm.x, iv.y, lm.z * sl[0].y)));
        A = 0.f;
      } else {
        s2 = mul2(make_float2(lm.z, lm.w), sl[0]);
        A = lm.x;
      }
      sl[0] = s2;
    }
#pragma unroll
    for (int t = 1; t < kL; ++t) {
      const float4 lm = lam_s[h * kL + t];
      s2 = fma2(make_float2(lm.x, lm.y), s2, mul2(make_float2(lm.z, lm.w), sl[t]));
      A *= lm.x;
      sl[t] = s2;
    }

    // ---- publish the aggregate, look back, publish the inclusive state -----------
    const size_t n = (size_t)(b * kH + h) * p.nchunks + c;
    float2 X = make_float2(0.f, 0.f);
    if (c == 0) {
      st_rec(p.inc + n * kHD + j0, pack_rec(s2.x, tag_inc));
      st_rec(p.inc + n * kHD + j0 + 1, pack_rec(s2.y, tag_inc));
    } else {
      st_rec(p.agg + n * kHD + j0, pack_rec(s2.x, tag_agg));
      st_rec(p.agg + n * kHD + j0 + 1, pack_rec(s2.y, tag_agg));
      if (lane == 0) st_rec(p.aggA + n, pack_rec(A, tag_agg));
      float2 accB = make_float2(0.f, 0.f);
      float accA = 1.f;
      size_t nj = n - 1;
      uint32_t spins = 0;
      while (true) {
        const unsigned long long i0 = ld_rec(p.inc + nj * kHD + j0);
        const unsigned long long i1 = ld_rec(p.inc + nj * kHD + j0 + 1);
        const unsigned long long a0 = ld_rec(p.agg + nj * kHD + j0);
        const unsigned long long a1 = ld_rec(p.agg + nj * kHD + j0 + 1);
        const unsigned long long aa = ld_rec(p.aggA + nj);
        if (rec_tag(i0) == tag_inc && rec_tag(i1) == tag_inc) {
          X = make_float2(fmaf(accA, rec_val(i0), accB.x), fmaf(accA, rec_val(i1), accB.y));
          break;
        }
        if (rec_tag(a0) == tag_agg && rec_tag(a1) == tag_agg && rec_tag(aa) == tag_agg) {
          accB = make_float2(fmaf(accA, rec_val(a0), accB.x), fmaf(accA, rec_val(a1), accB.y));
          accA *= rec_val(aa);
          --nj;  // chunk 0 always publishes an inclusive record, so the walk stays in the chain
          continue;
        }
        if (++spins > kSpinLimit) {
          ok = false;
          break;
        }
        if (spins > 16) __nanosleep(64);
      }
      st_rec(p.inc + n * kHD + j0, pack_rec(fmaf(A, X.x, s2.x), tag_inc));
      st_rec(p.inc + n * kHD + j0 + 1, pack_rec(fmaf(A, X.y, s2.y), tag_inc));
    }

    // ---- outputs ----------------------------------------------------------------------
    {
      float2 A2 = make_float2(1.f, 1.f);
      if (kTmaOut) {  // into the consumed tile; the TMA store clips rows past S
#pragma unroll
        for (int t = 0; t < kL; ++t) {
          A2 = mul2(A2, make_float2(lam_s[h * kL + t].x, lam_s[h * kL + t].x));
          const float2 o = fma2(A2, X, sl[t]);
          *reinterpret_cast<uint32_t*>(xs + tile_off(t, h, lane >> 2) + (lane & 3) * 4) = pack_bf16x2(o.x, o.y);
        }
      } else {
        OT* ob = reinterpret_cast<OT*>(p.out) + (size_t)b * p.osb + (size_t)t0 * p.oss + ch0;
        const int nt = min(kL, p.S - t0);
#pragma unroll
        for (int t = 0; t < kL; ++t) {
          A2 = mul2(A2, make_float2(lam_s[h * kL + t].x, lam_s[h * kL + t].x));
          const float2 o = fma2(A2, X, sl[t]);
          if (t < nt) st2(ob + (size_t)t * p.oss, make_float2(clamp1(o.x), clamp1(o.y)));
        }
      }
      const int tl = p.S - 1 - t0;  // the sequence's last token falls in this item: final state
      if (p.fin && tl < kL) {
        float2 B2 = make_float2(1.f, 1.f), v = make_float2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < kL; ++t) {
          B2 = mul2(B2, make_float2(lam_s[h * kL + t].x, lam_s[h * kL + t].x));
          if (t == tl) v = fma2(B2, X, sl[t]);
        }
        *reinterpret_cast<float2*>(p.fin + (size_t)b * kD + ch0) = make_float2(clamp1(v.x), clamp1(v.y));
      }
    }
    if (kTmaOut) fence_proxy_async_smem();
    __syncthreads();  // tile complete; lam_s / part_s free for the next item
    if (tid == 0 && kTmaOut) {
#pragma unroll
      for (int hh = 0; hh < kH; ++hh) tma_store_3d(&tmap_o, xs + hh * (kL * 128), hh * kHD, t0, b);
      bulk_commit();
    }
    pend_k = k + 2 * G;  // loaded into this buffer during the next item
  }

  if (tid == 0 && kTmaOut) bulk_wait0();
  if (!ok) {
    atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
    atomicAdd(&p.ws->timeouts, 1u);
  }
  if (tid == 0) {
    // the last unit to leave advances the epoch that tags the records
    __threadfence();
    if (atomicAdd(&p.ws->exited, 1u) == G - 1) {
      atomicExch(&p.ws->exited, 0u);
      atomicExch(&p.ws->epoch, epoch + 1u);
    }
  }
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

// [B, S, 512] bf16 as a 3D map with a [1, 32, 64] box (one head), 128-byte swizzle.
bool encode_map(CUtensorMap* map, const void* base, int S, int B, long long ss, long long sb) {
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)S, (cuuint64_t)B};
  const long long sbb = B > 1 ? sb : (long long)S * ss;
  cuuint64_t strides[2] = {(cuuint64_t)ss * 2, (cuuint64_t)sbb * 2};
  cuuint32_t box[3] = {(cuuint32_t)kHD, (cuuint32_t)kL, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool GATE, bool PRECISE, typename OT>
cudaError_t launch(const CUtensorMap& mx, const CUtensorMap& mo, const Params& p, cudaStream_t st) {
  auto kern = fwd_fast_kernel<GATE, PRECISE, OT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0, per_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNT, kSmemAlloc)) != cudaSuccess) return e;
  // every unit must be resident at once (a unit waits on items of other units)
  uint32_t G = (uint32_t)((per_sm > 0 ? per_sm : 1) * nsm);
  if (G > p.nitems) G = p.nitems;
  kern<<<G, kNT, kSmemAlloc, st>>>(mx, mo, p);
  return cudaGetLastError();
}

}  // namespace fast
}  // namespace ossm

using namespace ossm;

bool ossm_tc_eligible(const ossm_fwd_args* a) {
  if (a->x_dtype != OSSM_BF16 || a->H != fast::kH || a->head_dim != fast::kHD || a->tanh_out) return false;
  if ((a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_LUT || (a->flags & (OSSM_F_FASTPATH | OSSM_F_GENERIC))) return false;
  if (((uintptr_t)a->x % 16) || (a->x_stride_s % 8) || (a->B > 1 && (a->x_stride_b % 8))) return false;
  if (a->out_dtype == OSSM_BF16 &&
      (((uintptr_t)a->out % 16) || (a->out_stride_s % 8) || (a->B > 1 && (a->out_stride_b % 8))))
    return false;
  if (a->S > (1 << 30)) return false;
  return fast::encode_fn() != nullptr;
}

// Workspace of the fast path: header, then inclusive / aggregate records.
size_t ossm_tc_workspace_bytes(const ossm_fwd_args* a) {
  const size_t nch = (size_t)(a->S + fast::kL - 1) / fast::kL;
  const size_t N = (size_t)a->B * fast::kH * nch;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  return al(sizeof(WsHeader)) + 2 * al(N * fast::kHD * 8) + al(N * 8);
}

int ossm_tc_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st) {
  using namespace fast;
  Params p;
  p.B = a->B;
  p.S = a->S;
  p.K = a->degree;
  p.nchunks = (a->S + kL - 1) / kL;
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
  const size_t N = (size_t)a->B * kH * p.nchunks;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  p.ws = reinterpret_cast<WsHeader*>(ws);
  size_t off = al(sizeof(WsHeader));
  p.inc = reinterpret_cast<unsigned long long*>(ws + off);
  off += al(N * kHD * 8);
  p.agg = reinterpret_cast<unsigned long long*>(ws + off);
  off += al(N * kHD * 8);
  p.aggA = reinterpret_cast<unsigned long long*>(ws + off);
  const long long items = (long long)a->B * p.nchunks;
  if (items > 0x7fffffffLL) return OSSM_EINVAL;
  p.nitems = (uint32_t)items;

  CUtensorMap mx, mo;
  if (!encode_map(&mx, a->x, a->S, a->B, a->x_stride_s, a->x_stride_b)) return OSSM_EINVAL;
  mo = mx;
  if (a->out_dtype == OSSM_BF16 && !encode_map(&mo, a->out, a->S, a->B, a->out_stride_s, a->out_stride_b))
    return OSSM_EINVAL;
  const bool precise = (a->out_dtype == OSSM_F32) || (a->flags & OSSM_F_PRECISE);
  cudaError_t e;
  if (a->out_dtype == OSSM_F32) {
    e = gate ? launch<true, true, float>(mx, mo, p, st) : launch<false, true, float>(mx, mo, p, st);
  } else if (precise) {
    e = gate ? launch<true, true, __nv_bfloat16>(mx, mo, p, st) : launch<false, true, __nv_bfloat16>(mx, mo, p, st);
  } else {
    e = gate ? launch<true, false, __nv_bfloat16>(mx, mo, p, st)
             : launch<false, false, __nv_bfloat16>(mx, mo, p, st);
  }
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
