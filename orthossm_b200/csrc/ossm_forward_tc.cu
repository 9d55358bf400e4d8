// Forward fast path for bf16 activations with head_dim 64 (sm_100a): a
// persistent, TMA-pipelined kernel with the per-token decay gate on tcgen05
// tensor cores inside an H-CTA cluster.
//
// Same arithmetic contract as fwd_scan_kernel in ossm_forward.cu (which
// restates _fused_clenshaw_ema_kernel, sdpc_kernel.py:988-1209); this file only
// changes how the work is mapped onto the B200.
//
// Work item = (batch b, head h, chunk c of 256 tokens).  Items are handed out
// in ticket order (chunk-major), so every item's predecessors in its (b, h)
// chain are already owned by running CTAs when it waits on them.  Two CTAs
// stay resident per SM and loop over items:
//
//   * the x tiles of the next two items are in flight by TMA (3D tensor map,
//     128-byte swizzle) while the current one is computed: double buffer;
//   * gate (optional): the cluster holds the H heads of one (b, c); the tile is
//     the A operand of a tcgen05 MMA D[256x16] = X[256x64] . Wsplit[16x64]^T,
//     Wsplit = this head's gate weights for all H heads as bf16 hi and lo
//     halves (x is exact in bf16, hi+lo keeps ~16 mantissa bits of W), with
//     the accumulator in TMEM.  Partial logits go to the owning head's CTA over
//     distributed shared memory; one cluster barrier per item;
//   * lane = 2 channels, warp = a run of 32 tokens: u = tanh(gamma y(xn)) in
//     registers (packed f32x2 Horner), local scan, per-channel run combine,
//     decoupled look-back (warp-wide window, deterministic forward fold);
//   * bf16 outputs are written into the consumed x buffer (same swizzle) and
//     leave by a TMA store; the buffer is refilled once the store has read it.
#include <cudaTypedefs.h>

#include <mutex>

#include "ossm_sm100.cuh"

namespace ossm {
namespace tc {

constexpr int kNT = 256;
constexpr int kHD = 64;      // channels per item (one head)
constexpr int kL = 256;      // tokens per item
constexpr int kR = 32;       // tokens per thread (one run per warp)
constexpr int kRUNS = 8;     // runs per item
constexpr int kMaxH = 8;

// shared memory layout (bytes from a 1024-aligned base)
constexpr int kTile = kL * 128;                        // one [256][128 B] bf16 tile
constexpr int kOffX = 0;                               // 2 swizzled x / output tiles
constexpr int kOffW = kOffX + 2 * kTile;               // [16][128 B] swizzled gate weights
constexpr int kOffAggB = kOffW + 16 * 128;             // [8 runs][64] f32
constexpr int kOffAggA = kOffAggB + kRUNS * kHD * 4;   // [8] f32
constexpr int kOffExclA = kOffAggA + 64;               // [8] f32
constexpr int kOffCarry = kOffExclA + 64;              // [64] f32
constexpr int kOffLam = kOffCarry + kHD * 4;           // [256] float4 (lam, lam, 1-lam, 1-lam)
constexpr int kOffPart = kOffLam + kL * 16;            // [2 items][8 src][256] f32 partial logits
constexpr int kOffCoef = kOffPart + 2 * kMaxH * kL * 4; // [2 items][8][64] f32 coefficients of (b, h)
constexpr int kOffBar = kOffCoef + 2 * 8 * kHD * 4;    // mbarriers + scalars
constexpr int kSmemBytes = kOffBar + 128;
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
  uint32_t nunits;  // items (one per cluster with the gate)
  uint32_t ngrid;   // persistent units in the grid (clusters with the gate, CTAs without)
};

// Chebyshev -> monomial coefficients, gamma folded in:
// sum_k c_k T_k(x) = sum_m a_m x^m with T_0..T_7 written out.
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

OSSM_DEV uint32_t xs_offset(int row, int lane) {  // this lane's 2 channels of `row`, 128-byte swizzle
  return row * 128 + ((((lane >> 2) ^ (row & 7))) << 4) + (lane & 3) * 4;
}

template <bool GATE, bool PRECISE, typename OT>
__global__ void __launch_bounds__(kNT, 2)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_o,
                  const Params p) {
  using namespace sm100;
  constexpr bool kTmaOut = sizeof(OT) == 2;  // bf16 outputs leave by TMA store
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wsm = sm + kOffW;
  float* aggB_s = reinterpret_cast<float*>(sm + kOffAggB);
  float* aggA_s = reinterpret_cast<float*>(sm + kOffAggA);
  float* exclA_s = reinterpret_cast<float*>(sm + kOffExclA);
  float* carry_s = reinterpret_cast<float*>(sm + kOffCarry);
  float4* lam_s = reinterpret_cast<float4*>(sm + kOffLam);
  float* part_s = reinterpret_cast<float*>(sm + kOffPart);
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [2]
  uint64_t* mma_bar = tma_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffBar + 32);
  uint32_t* tk_s = tmem_slot + 1;  // [3] ticket ring
  uint32_t* s_epoch = tmem_slot + 4;
  int* s_kincl = reinterpret_cast<int*>(tmem_slot + 5);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = GATE ? cluster_rank() : 0u;
  const bool leader = GATE ? (crank == 0) : true;  // takes the unit's tickets

  // ---- prologue ----------------------------------------------------------------
  if (tid == 0) {
    mbar_init(tma_bar + 0, 1);
    mbar_init(tma_bar + 1, 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    if (kTmaOut) prefetch_tmap(&tmap_o);
    if (leader) {
      const uint32_t e = atomicAdd(&p.ws->epoch, 0u);
      __threadfence();
      tk_s[0] = atomicAdd(&p.ws->ticket, 1u);
      tk_s[1] = atomicAdd(&p.ws->ticket, 1u);
      *s_epoch = e;
    }
  }
  if (GATE && warp == 1) tmem_alloc(tmem_slot, 32);
  if (GATE) {
    // gate weights of this CTA's head (the cluster rank), bf16 hi/lo, swizzled
    const int n = tid >> 4;         // rows 0-7 hi, 8-15 lo
    const int k0 = (tid & 15) * 4;  // channel within the head
    const int hh = n & 7;
    float w[4] = {0.f, 0.f, 0.f, 0.f};
    if (hh < p.H) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p.gate_w + (size_t)hh * p.D + crank * kHD + k0));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
    uint16_t e16[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(w[q]);
      const __nv_bfloat16 o = n < 8 ? hi : __float2bfloat16_rn(w[q] - __bfloat162float(hi));
      e16[q] = *reinterpret_cast<const uint16_t*>(&o);
    }
    const int byte = k0 * 2;
    *reinterpret_cast<uint2*>(wsm + n * 128 + ((((byte >> 4) ^ (n & 7))) << 4) + (byte & 15)) =
        make_uint2((uint32_t)e16[0] | ((uint32_t)e16[1] << 16), (uint32_t)e16[2] | ((uint32_t)e16[3] << 16));
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
    tc_fence_before();
    cluster_sync();  // every CTA started (DSMEM addressable); rank 0 holds the first tickets
    tc_fence_after();
    if (tid == 0) {
      tk_s[0] = ld_cluster_u32(map_smem(tk_s + 0, 0));
      tk_s[1] = ld_cluster_u32(map_smem(tk_s + 1, 0));
      *s_epoch = ld_cluster_u32(map_smem(s_epoch, 0));
    }
  }
  __syncthreads();
  const uint32_t epoch = *s_epoch;
  const uint32_t tmem = GATE ? *tmem_slot : 0u;

  auto decode = [&](uint32_t t, int& b, int& h, int& c) {
    if (GATE) {
      c = (int)(t / p.B);
      b = (int)(t % p.B);
      h = (int)crank;
    } else {
      c = (int)(t / (p.B * p.H));
      const int rem = (int)(t % (p.B * p.H));
      b = rem / p.H;
      h = rem % p.H;
    }
  };
  auto issue_load = [&](uint32_t t, int buf) {  // one thread: x tile + the (b, h) coefficients
    int b, h, c;
    decode(t, b, h, c);
    const uint32_t cbytes = (uint32_t)p.K * kHD * 4;
    mbar_expect_tx(tma_bar + buf, kTile + cbytes);
    tma_load_3d(sm + kOffX + buf * kTile, &tmap_x, tma_bar + buf, h * kHD, c * kL, b);
    bulk_load(sm + kOffCoef + buf * (8 * kHD * 4), p.coeffs + ((size_t)(b * p.H + h) * p.K) * kHD, cbytes,
              tma_bar + buf);
  };
  if (tid == 0) {
    if (tk_s[0] < p.nunits) issue_load(tk_s[0], 0);
    if (tk_s[1] < p.nunits) issue_load(tk_s[1], 1);
  }

  const int run = warp;     // tokens run*32 .. run*32+31 of the item
  const int j0 = lane * 2;  // channel pair within the head
  bool ok = true;

  // ---- item loop -----------------------------------------------------------------
  for (int i = 0;; ++i) {
    const uint32_t T = tk_s[i % 3];
    if (T >= p.nunits) break;
    int b, h, c;
    decode(T, b, h, c);
    const int buf = i & 1;
    uint8_t* xs = sm + kOffX + buf * kTile;
    const int t0 = c * kL;
    const int ch0 = h * kHD + j0;
    const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;

    // the ticket two items ahead: issued now, consumed after the evaluation
    uint32_t t_ahead = 0;
    if (tid == 0 && leader) t_ahead = atomicAdd(&p.ws->ticket, 1u);
    // per-token decay supplied by the caller: load early as well
    const int tg = t0 + tid;
    float lam_in = 1.f;
    if (!GATE) {
      lam_in = p.lam_tok ? (tg < p.S ? __ldg(p.lam_tok + ((size_t)b * p.S + tg) * p.H + h) : 1.f)
                         : (p.lam_h ? __ldg(p.lam_h + h) : p.momentum);
    }

    ok &= mbar_wait(tma_bar + buf, (uint32_t)(i >> 1) & 1u);

    // coefficients of (b, h) from the tile's transaction: raw Chebyshev
    // (precise) or gamma-folded monomial
    float2 cf[8];
    {
      const float* cs = reinterpret_cast<const float*>(sm + kOffCoef + buf * (8 * kHD * 4)) + j0;
      float2 ck[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) ck[k] = k < p.K ? *reinterpret_cast<const float2*>(cs + k * kHD) : make_float2(0.f, 0.f);
      if (PRECISE) {
#pragma unroll
        for (int k = 0; k < 8; ++k) cf[k] = ck[k];
      } else {
        cheb_to_mono(ck, gamma, cf);
      }
    }

    // gate MMA (one thread): D[tokens][16] in TMEM
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

    // u = tanh(clamp(gamma y(xn), +-4)) into registers
    float2 sl[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int row = run * kR + r;
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(xs + xs_offset(row, lane));
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
        y = cf[7];
#pragma unroll
        for (int m = 6; m >= 0; --m) y = fma2(y, xn, cf[m]);
      }
      const float z0 = fminf(fmaxf(y.x, -4.f), 4.f), z1 = fminf(fmaxf(y.y, -4.f), 4.f);
      const float u0 = PRECISE ? tanhf(z0) : tanh_fast(z0);
      const float u1v = PRECISE ? tanhf(z1) : tanh_fast(z1);
      sl[r] = make_float2(x0 == x0 ? u0 : 0.f, x1 == x1 ? u1v : 0.f);  // NaN input -> 0 (sdpc_kernel.py:1164)
    }

    // decay of each token; publish the ticket taken above
    if (GATE) {
      ok &= mbar_wait(mma_bar, (uint32_t)i & 1u);
      tc_fence_after();
      const int q4 = warp & 3, mt = warp >> 2;
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + mt * 16, v);
      const int tok = mt * 128 + q4 * 32 + lane;
      float* part_i = part_s + buf * (kMaxH * kL);
      for (int n = 0; n < p.H; ++n) st_cluster_f32(map_smem(part_i + crank * kL + tok, n), v[n] + v[n + 8]);
      if (tid == 0 && leader)
        for (int r = 0; r < p.H; ++r) st_cluster_u32(map_smem(tk_s + (i + 2) % 3, r), t_ahead);
      tc_fence_before();
      cluster_sync();  // partial logits and the ticket delivered
      tc_fence_after();
      float logit = __ldg(p.gate_b + h);
      for (int s = 0; s < p.H; ++s) logit += part_i[s * kL + tid];
      const float sg = 1.0f / (1.0f + __expf(-logit));
      const float lam = fminf(fmaxf(__ldg(p.lam_h + h) + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
      lam_s[tid] = tg >= p.S ? make_float4(1.f, 1.f, 0.f, 0.f) : make_float4(lam, lam, 1.f - lam, 1.f - lam);
    } else {
      if (tid == 0) tk_s[(i + 2) % 3] = t_ahead;
      lam_s[tid] = tg >= p.S ? make_float4(1.f, 1.f, 0.f, 0.f) : make_float4(lam_in, lam_in, 1.f - lam_in, 1.f - lam_in);
    }
    __syncthreads();

    // local scan of each run
    const int tbase = t0 + run * kR;
    {
      float2 s2 = make_float2(0.f, 0.f);
      float Arun = 1.f;
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

    // combine runs per channel, publish the chunk aggregate
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
    // the CTA's writes are ordered before the flag by the barrier and the
    // gpu-scope release store of the publishing thread
    if (c > 0 && tid == 32) st_release(p.lbflag + n, (epoch << 2) | 1u);  // warp 1: warp 0 looks back
    if (c > 0 && warp == 0) {
      // warp-wide window: lane i probes chunk (base - i); nearest inclusive wins
      int base = c - 1, kincl = -1;
      bool okw = true;
      while (kincl < 0) {
        const int j = base - lane;
        uint32_t st = 0;
        if (j >= 0) st = wait_flag(p.lbflag + (n - (size_t)(c - j)), epoch);
        if (__ballot_sync(0xffffffffu, j >= 0 && st == 0)) {
          okw = false;
          break;
        }
        const uint32_t m2 = __ballot_sync(0xffffffffu, j >= 0 && st == 2);
        if (m2) kincl = base - (__ffs(m2) - 1);
        else base -= 32;
      }
      if (lane == 0) *s_kincl = okw ? kincl : -1;
    }
    __syncthreads();
    if (tid < kHD) {
      float X = 0.f;
      if (c > 0) {
        const int k = *s_kincl;
        if (k >= 0) {
          X = __ldcg(p.incB + (n - (size_t)(c - k)) * kHD + tid);
          int j = k + 1;  // fold forward 4 chunks at a time; loads do not depend on X
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
        } else {
          ok = false;
        }
      }
      carry_s[tid] = X;
      p.incB[n * kHD + tid] = fmaf(chunkA, X, chunkB);
    }
    __syncthreads();
    if (tid == 32) st_release(p.lbflag + n, (epoch << 2) | 2u);

    // outputs
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
        const int row = run * kR + r;
        const float4 lm = lam_s[row];
        A2 = mul2(A2, make_float2(lm.x, lm.y));
        float2 o = fma2(A2, rc, sl[r]);
        if (kTmaOut) {
          *reinterpret_cast<uint32_t*>(xs + xs_offset(row, lane)) = pack_bf16x2(o.x, o.y);
        } else {
          o = make_float2(clamp1(o.x), clamp1(o.y));
          if (t < p.S) st2(ob + (size_t)t * p.oss, o);
        }
        if (t == p.S - 1 && p.fin)
          *reinterpret_cast<float2*>(p.fin + (size_t)b * p.D + ch0) = make_float2(clamp1(o.x), clamp1(o.y));
      }
      if (kTmaOut) fence_proxy_async_smem();
    }
    __syncthreads();
    if (tid == 0) {
      if (kTmaOut) {
        tma_store_3d(&tmap_o, xs, h * kHD, t0, b);
        bulk_commit();
      }
      const uint32_t t2 = tk_s[(i + 2) % 3];
      if (t2 < p.nunits) {
        if (kTmaOut) bulk_wait_read0();  // the store has read the buffer
        issue_load(t2, buf);
      }
    }
  }

  // ---- epilogue ------------------------------------------------------------------
  if (tid == 0 && kTmaOut) bulk_wait0();
  if (!ok) {
    atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
    atomicAdd(&p.ws->timeouts, 1u);
  }
  if (GATE) {
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 32);
  }
  if (tid == 0 && leader) {
    // the last unit to leave resets the ticket counter and advances the epoch
    __threadfence();
    if (atomicAdd(&p.ws->exited, 1u) == p.ngrid - 1) {
      atomicExch(&p.ws->ticket, 0u);
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

// [B, S, D] bf16 tensor as a 3D map with a [1, 256, 64] box (128-byte swizzle).
bool encode_tile_map(CUtensorMap* map, const void* base, int D, int S, int B, long long ss, long long sb) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)B};
  const long long sbb = B > 1 ? sb : (long long)S * ss;
  cuuint64_t strides[2] = {(cuuint64_t)ss * 2, (cuuint64_t)sbb * 2};
  cuuint32_t box[3] = {(cuuint32_t)kHD, (cuuint32_t)kL, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool GATE, bool PRECISE, typename OT>
cudaError_t launch(const CUtensorMap& mx, const CUtensorMap& mo, Params p, cudaStream_t st) {
  auto kern = fwd_tc_kernel<GATE, PRECISE, OT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kNT, 1, 1);
  cfg.dynamicSmemBytes = kSmemAlloc;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = GATE ? p.H : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Units = resident CTAs per SM x SMs (divided by the cluster size).  Units
  // that cannot be resident at once simply start later: a unit takes no
  // ticket before it runs, and it only ever waits on smaller tickets.
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNT, kSmemAlloc)) != cudaSuccess) return e;
  int units = (per_sm > 0 ? per_sm : 1) * nsm;
  if (GATE) units = units / p.H > 0 ? units / p.H : 1;
  if ((uint32_t)units > p.nunits) units = (int)p.nunits;
  p.ngrid = (uint32_t)units;
  cfg.gridDim = dim3(units * (GATE ? p.H : 1), 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, mx, mo, p);
}

}  // namespace tc
}  // namespace ossm

using namespace ossm;

// Eligibility of the TMA / tcgen05 path for these arguments.
bool ossm_tc_eligible(const ossm_fwd_args* a) {
  if (a->x_dtype != OSSM_BF16 || a->head_dim != 64 || a->tanh_out) return false;
  if ((a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_LUT || (a->flags & (OSSM_F_FASTPATH | OSSM_F_GENERIC))) return false;
  if (((uintptr_t)a->x % 16) || (a->x_stride_s % 8) || (a->B > 1 && (a->x_stride_b % 8))) return false;
  if (a->out_dtype == OSSM_BF16 &&
      (((uintptr_t)a->out % 16) || (a->out_stride_s % 8) || (a->B > 1 && (a->out_stride_b % 8))))
    return false;
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
  const long long items = (long long)a->B * a->H * p.nchunks;
  if (items > 0x7fffffffLL) return OSSM_EINVAL;
  p.nunits = (uint32_t)(gate ? (long long)a->B * p.nchunks : items);
  p.ngrid = 0;

  CUtensorMap mx, mo;
  if (!encode_tile_map(&mx, a->x, p.D, a->S, a->B, a->x_stride_s, a->x_stride_b)) return OSSM_EINVAL;
  mo = mx;  // unused unless the output is bf16
  if (a->out_dtype == OSSM_BF16 && !encode_tile_map(&mo, a->out, p.D, a->S, a->B, a->out_stride_s, a->out_stride_b))
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
