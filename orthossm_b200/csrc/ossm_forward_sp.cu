// Single-pass forward for bf16 activations, 8 heads x head_dim 64 (sm_100a),
// with the chunk carries relayed by dedicated warps.
//
// Same arithmetic contract as fwd_scan_kernel in ossm_forward.cu (which
// restates _fused_clenshaw_ema_kernel, sdpc_kernel.py:988-1209).  The EMA
// s_t = a_t s_{t-1} + (1 - a_t) u_t is split into 16-token chunks.  One
// cooperative launch holds two kinds of CTA of 768 threads, one per SM, all
// resident at once:
//
//   worker CTAs   three independent groups of 8 warps; a group takes (b, chunk)
//                 items, warp = head, lane = 2 channels x 16 tokens.
//                 A worker TMA-loads the [16 x 512] tile, forms the decays (the
//                 optional gate as a tensor-core product), evaluates u once and
//                 runs the EMA from a zero state, keeping the 16 local states in
//                 registers.  It publishes the chunk's end state and decay
//                 product, waits for the state entering the chunk, and writes
//                 out_t = local_t + (decay product to t) * carry.
//   relay CTAs    kRelayPerCta warps, one per (b, h) chain, on SMs of their own
//                 (sharing an SM with workers left them a few issue slots per
//                 step).  A relay warp folds the published chunk
//                 records in chunk order, carry_{k+1} = A_k carry_k + agg_k,
//                 and publishes each carry.  Records reach it through a
//                 cp.async ring in shared memory (kNB batches of kBat chunks in
//                 flight, completed in order), and it folds a whole batch per
//                 round, so a chunk costs it a few instructions once its record
//                 is out.  (Register-prefetched global loads measured no
//                 overlap here: every step paid a full round trip.)
//
// x is read once and every element is evaluated once.  Measured at config 2
// (B=8, S=16384, 1 x B200): 220 us per step gated, 132 us with constant
// decays, against 148 / 130 us for the three-pass kernel: every relay round
// pays the issue cost of its memory instructions on a serial chain of 1024
// chunks, and with the gate the eight heads of a worker group wait for the
// slowest relay at every item.  Kept as an opt-in path (OSSM_F_RELAY).
//
// Records are 64-bit words (f32 value | 32-bit tag), written and read whole,
// so no fences are needed: a reader polls until every word it needs carries
// the expected tag.  A waiting worker polls one word from one lane (the
// record's other words follow within a poll or two), which keeps the polling
// out of the way of the relay's loads in L2.  Records live in per-chain rings
// of kRing chunk slots that stay in L2.  A slot is reused only after its
// reader is done with it: worker group (unit) g keeps chain b = g mod B and
// takes chunks g/B, g/B + dC, ... (dC = units / B), so a unit reaches chunk
// c + dC only after finishing chunk c, and the relay passes chunk c + kRing
// only after that; kRing > dC + 1 is checked at launch.  Tags carry the launch
// epoch (advanced by the last CTA to leave) and the ring round, so records of
// earlier launches never match.
//
// Results are bitwise reproducible: every fold has a fixed order.
//
// NaN and +-inf inputs surface as a NaN state in the fast evaluation; the warp
// then redoes its chunk with the reference's semantics (u = 0 at NaN x,
// xn = +-1 at +-inf) in rolled loops: once for the chunk record, once more for
// the outputs when the carry has arrived (keeping the tile until then).
#include <cudaTypedefs.h>

#include <algorithm>

#include "ossm_eval.cuh"

namespace ossm {
namespace fast {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
}  // namespace fast

namespace sp {

using namespace ev;

constexpr int kT = 16;   // tokens per chunk
constexpr int kH = 8;    // heads (one warp each)
constexpr int kHD = 64;  // channels per head
constexpr int kD = kH * kHD;
constexpr int kGroupNT = 256;  // one worker group: 8 warps, one per head
constexpr int kGroups = 3;     // worker groups per CTA
constexpr int kNT = kGroups * kGroupNT;
// Relay warps per relay CTA.  A relay round is bound by how fast its SM
// issues the round's stores and cp.async copies; at config 2 (gated / constant
// decay, us per step) 16 per CTA measured 275 / 259, 8 per CTA 207 / 148 and
// 4 per CTA 220 / 132.
constexpr int kRelayPerCta = 4;
constexpr int kTile = kT * kD * 2;                        // 16 KB: [16 tokens][8 heads][128 B]
constexpr int kStages = 2;
constexpr int kOffW = kStages * kTile;                    // gate B fragments [8 warps][4 k-steps][32 lanes] uint4
constexpr int kOffPart = kOffW + kH * 4 * 32 * 16;        // [2][8 warps][16 tokens][8 heads] f32
constexpr int kOffTab = kOffPart + 2 * kH * kT * kH * 4;  // [8 warps][16 tokens] (a, 1 - a, P, -)
constexpr int kOffBar = kOffTab + kH * kT * 16;           // full[2] mbarriers, then left[2] counters
constexpr int kGroupSmem = (kOffBar + 32 + 1023) & ~1023;  // one group's region (its tiles 1024-byte aligned)
constexpr int kSmemAlloc = kGroups * kGroupSmem + 1024;    // + alignment slack
constexpr int kRingLog = 7;
constexpr int kRing = 1 << kRingLog;  // chunk slots per chain
constexpr int kBat = 4;               // relay: chunks per round
constexpr int kNB = 3;                // relay: rounds of records in flight
constexpr int kRelaySlot = 33;        // relay ring slot: 32 lanes' records + the decay word, 16 B each
static_assert(kRing % kBat == 0, "a relay round stays inside one ring round");
static_assert(kRelayPerCta * kNB * kBat * kRelaySlot * 16 + 1024 <= kSmemAlloc, "relay rings fit the CTA's shared memory");

struct Params {
  int B, S, K, nchunks;
  int nunits;  // worker groups, a multiple of B: group u of worker CTA u / 3
  int nwcta;   // worker CTAs; CTAs from nwcta on relay
  const float* coeffs;
  const float* lam_h;
  float momentum;
  const float* gate_w;
  const float* gate_b;
  float gate_scale, gate_lo, gate_hi;
  const float* lam_tok;  // caller's per-token decay [B,S,H] or NULL
  const float* init;
  float* fin;
  __nv_bfloat16* out;        // [B, S, 512], contiguous
  uint4* agg;                // [B*8 chains][kRing][32 lanes]: (end state | tag) x 2 channels
  uint4* arec;               // [B*8][kRing]: (decay product | tag), 16-byte slots
  uint4* inc;                // [B*8][kRing][32]: (state after the chunk | tag) x 2
  WsHeader* ws;
};

// Odd, so a zero-filled workspace never matches; 19 bits of epoch, 12 of ring round.
OSSM_DEV uint32_t tag_of(uint32_t epoch, int c) {
  return ((epoch & 0x7ffffu) << 13) | ((uint32_t)(c >> kRingLog) << 1) | 1u;
}

OSSM_DEV uint4 ld_rec(const uint4* p) {
  unsigned long long a, b;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
  return make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)b, (uint32_t)(b >> 32));
}
OSSM_DEV void st_rec(uint4* p, float2 v, uint32_t tag) {
  const unsigned long long a = (unsigned long long)__float_as_uint(v.x) | ((unsigned long long)tag << 32);
  const unsigned long long b = (unsigned long long)__float_as_uint(v.y) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
OSSM_DEV unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long a;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}
OSSM_DEV void st_word(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long a = (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
OSSM_DEV void cpa16(void* s, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(s)), "l"(g) : "memory");
}
OSSM_DEV void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
OSSM_DEV void cpa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
OSSM_DEV void group_sync(int grp) {  // the 256 threads of one worker group (named barrier 1 + grp)
  asm volatile("bar.sync %0, 256;" ::"r"(1 + grp) : "memory");
}
OSSM_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(sm100::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(sm100::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// u of the lane's two channels at one token: z = 4 xn = x / (1/4 + |x|/4),
// Horner on the gamma-folded monomial coefficients scaled by 4^-k (the same
// roundings as Horner in xn on the unscaled ones), tanh(clamp(y, +-4)).
// NaN and +-inf inputs come out as NaN.
OSSM_DEV float2 u_fast(uint32_t raw, const float2 (&m)[8]) {
  const float x0 = __uint_as_float(raw << 16), x1 = __uint_as_float(raw & 0xffff0000u);
  const float r0 = rcp_fast(fmaf(fabsf(x0), 0.25f, 0.25f)), r1 = rcp_fast(fmaf(fabsf(x1), 0.25f, 0.25f));
  const float2 z = mul2(make_float2(x0, x1), make_float2(r0, r1));
  float2 y = m[7];
#pragma unroll
  for (int q = 6; q >= 0; --q) y = fma2(y, z, m[q]);
  return make_float2(tanh_fast(clamp4_nan(y.x)), tanh_fast(clamp4_nan(y.y)));
}
// The reference's semantics for every input (sdpc_kernel.py:1078-1085, :1160-1164).
OSSM_DEV float u1_exact(float x, const float2 (&m)[8], bool second) {
  float xa, sg;
  const float z = 4.f * softsign<false>(x, false, xa, sg);
  float y = second ? m[7].y : m[7].x;
#pragma unroll
  for (int q = 6; q >= 0; --q) y = fmaf(y, z, second ? m[q].y : m[q].x);
  const float u = tanh_fast(clamp4_nan(y));
  return x != x ? 0.f : u;
}

// The chunk's EMA with the reference's semantics from state s (rolled; the rare
// chunk that holds NaN / inf inputs).  Writes the first nt states to op when
// given; returns the state after token 15.
OSSM_DEV float2 exact_run(const uint8_t* xrow, const float4* tab, const float2 (&m)[8], float2 s, bool first, int nt,
                          __nv_bfloat16* op = nullptr) {
#pragma unroll 1
  for (int t = 0; t < kT; ++t) {
    const uint32_t raw = *reinterpret_cast<const volatile uint32_t*>(xrow + t * (kH * 128));
    const float4 tb = tab[t];
    const float u0 = u1_exact(__uint_as_float(raw << 16), m, false);
    const float u1 = u1_exact(__uint_as_float(raw & 0xffff0000u), m, true);
    if (t == 0 && first)
      s = make_float2(clamp1(fmaf(tb.x, s.x, tb.y * u0)), clamp1(fmaf(tb.x, s.y, tb.y * u1)));
    else
      s = make_float2(fmaf(tb.x, s.x, tb.y * u0), fmaf(tb.x, s.y, tb.y * u1));
    if (op && t < nt) st2(op + (size_t)t * kD, s);
  }
  return s;
}

// ---------------------------------------------------------------------------
// relay warp: chain (b, h)
// ---------------------------------------------------------------------------
__device__ __noinline__ bool relay(const uint4* agg, const uint4* ar, uint4* inc, float* fin, int n, int b, int h,
                                   int lane, uint32_t epoch, uint4* rs) {
  const int chain = b * kH + h;
  agg += (size_t)chain * kRing * 32 + lane;
  ar += (size_t)chain * kRing;
  inc += (size_t)chain * kRing * 32 + lane;
  // round cb's records into ring rounds slotb .. slotb + kBat - 1 (an empty group past the end)
  auto fetch = [&](int slotb, int cb) {
#pragma unroll
    for (int q = 0; q < kBat; ++q) {
      const int c = cb + q;
      if (c < n) {
        const int sl = c & (kRing - 1);
        cpa16(rs + (slotb + q) * kRelaySlot + lane, agg + sl * 32);
        if (lane == 0) cpa16(rs + (slotb + q) * kRelaySlot + 32, ar + sl);
      }
    }
    cpa_commit();
  };
#pragma unroll
  for (int j = 0; j < kNB; ++j) fetch(j * kBat, j * kBat);
  bool ok = true;
  float2 X = make_float2(0.f, 0.f);
  int slotb = 0;
  for (int cb = 0; cb < n; cb += kBat) {
    cpa_wait<kNB - 1>();
    __syncwarp();
    const uint32_t tg = tag_of(epoch, cb);
    uint4 r[kBat], a[kBat];
    bool good = true;
#pragma unroll
    for (int q = 0; q < kBat; ++q) {
      r[q] = rs[(slotb + q) * kRelaySlot + lane];
      a[q] = rs[(slotb + q) * kRelaySlot + 32];
      if (cb + q < n) good = good && r[q].y == tg && r[q].w == tg && a[q].y == tg;
    }
    uint32_t spins = 0;
    while (ok && !__all_sync(0xffffffffu, good)) {  // not all out yet: poll the round from global memory
      if (++spins > kSpinLimit) {
        ok = false;
        break;
      }
      if (spins > 4) __nanosleep(32);
      good = true;
#pragma unroll
      for (int q = 0; q < kBat; ++q)
        if (cb + q < n) {
          const int sl = (cb + q) & (kRing - 1);
          r[q] = ld_rec(agg + sl * 32);
          a[q] = ld_rec(ar + sl);
          good = good && r[q].y == tg && r[q].w == tg && a[q].y == tg;
        }
    }
#pragma unroll
    for (int q = 0; q < kBat; ++q)
      if (cb + q < n) {
        const float A = __uint_as_float(a[q].x);
        X = make_float2(fmaf(A, X.x, __uint_as_float(r[q].x)), fmaf(A, X.y, __uint_as_float(r[q].z)));
        st_rec(inc + ((cb + q) & (kRing - 1)) * 32, X, tg);
      }
    __syncwarp();
    fetch(slotb, cb + kNB * kBat);
    slotb = slotb + kBat == kNB * kBat ? 0 : slotb + kBat;
  }
  cpa_wait<0>();
  if (fin)
    *reinterpret_cast<float2*>(fin + (size_t)b * kD + h * kHD + 2 * lane) = make_float2(clamp1(X.x), clamp1(X.y));
  return ok;
}

// The state entering chunk c (written by the relay after chunk c - 1).  The
// first look takes the whole record; while it is not out, lane 0 polls one
// word and the record is read again once its tag shows.
OSSM_DEV bool wait_carry(const uint4* ip, uint32_t tp, int lane, bool ok, float2& X) {
  uint4 r = ld_rec(ip);
  uint32_t spins = 0;
  while (ok && !__all_sync(0xffffffffu, r.y == tp && r.w == tp)) {
    if (++spins > kSpinLimit) return false;
    __nanosleep(spins > 64 ? 256 : 32);
    uint32_t seen = 0;
    if (lane == 0) seen = (uint32_t)(ld_word(reinterpret_cast<const unsigned long long*>(ip)) >> 32);
    if (__shfl_sync(0xffffffffu, seen, 0) == tp) r = ld_rec(ip);
  }
  X = make_float2(__uint_as_float(r.x), __uint_as_float(r.z));
  return ok;
}

// ---------------------------------------------------------------------------
// worker CTA
// ---------------------------------------------------------------------------
template <bool GATE>
OSSM_DEV bool work(const CUtensorMap* tmap, const Params& p, uint8_t* sm, int g, int grp, int h, int lane,
                   uint32_t epoch) {
  using namespace sm100;
  const int b = g % p.B;
  const int dC = p.nunits / p.B;
  const bool leader = h == 0 && lane == 0;
  const int chain = b * kH + h;
  const int j0 = 2 * lane;
  const float gamma = 0.98f - 0.06f * (float)h / (float)kH;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* left = reinterpret_cast<uint32_t*>(full + 2);  // warps done with each stage
  float* part = reinterpret_cast<float*>(sm + kOffPart);
  float4* tab = reinterpret_cast<float4*>(sm + kOffTab) + h * kT;
  uint4* wfr = reinterpret_cast<uint4*>(sm + kOffW) + h * 4 * 32 + lane;
  bool ok = true;

  auto issue = [&](int stage, int c) {
    mbar_expect_tx(full + stage, kTile);
    tma_load_4d(sm + stage * kTile, tmap, full + stage, 0, 0, c * kT, b);
  };
  const int cfirst = g / p.B;
  if (leader) {
    mbar_init(full + 0, 1);
    mbar_init(full + 1, 1);
    left[0] = left[1] = 0u;
    fence_mbar_init();
    prefetch_tmap(tmap);
    if (cfirst < p.nchunks) issue(0, cfirst);
    if (cfirst + dC < p.nchunks) issue(1, cfirst + dC);
  }
  // coefficients: gamma-folded monomial, scaled by 4^-k for z = 4 xn
  float2 m[8];
  {
    load_coeffs<false>(p.coeffs, p.K, b, h, j0, gamma, m);
  }
  const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  float bias_h = 0.f;
  if (GATE) {  // this warp's mma B fragments of W[gid][h*64 + ks*16 + ...], split into bf16 hi + lo
    const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float* wr = p.gate_w + (size_t)gid * kD + h * kHD + ks * 16 + 2 * tig;
      const float2 w01 = __ldg(reinterpret_cast<const float2*>(wr));
      const float2 w89 = __ldg(reinterpret_cast<const float2*>(wr + 8));
      const float hw[4] = {w01.x, w01.y, w89.x, w89.y};
      float hi[4], lo[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        hi[q] = bf16_round(hw[q]);
        lo[q] = bf16_round(hw[q] - hi[q]);
      }
      wfr[ks * 32] = make_uint4(pack_bf16x2(hi[0], hi[1]), pack_bf16x2(hi[2], hi[3]), pack_bf16x2(lo[0], lo[1]),
                                pack_bf16x2(lo[2], lo[3]));
    }
    bias_h = __ldg(p.gate_b + h);
  }
  float2 init2 = make_float2(0.f, 0.f);
  if (cfirst == 0 && p.init) init2 = __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + h * kHD + j0));
  // the lane's 4 bytes of token t: row (t, h) of the tile, 16-byte unit lane/4 swizzled by h
  const uint32_t xoff = (uint32_t)(h * 128 + (((lane >> 2) ^ h) << 4) + (lane & 3) * 4);
  group_sync(grp);

  int k = 0;
  for (int c = cfirst; c < p.nchunks; c += dC, ++k) {
    const int s = k & 1;
    const uint8_t* xs = sm + s * kTile;
    if (!mbar_wait(full + s, (uint32_t)(k >> 1) & 1u)) ok = false;
    const int t0 = c * kT;
    const bool first = c == 0;

    // ---- decays of tokens t0 .. t0+15 (lanes 0..15)
    float lam;
    if (GATE) {  // partial logits of this head's 64 channels for all 8 heads, then the sum
      const uint32_t xa = smem_u32(xs);
      const int mi = lane >> 3, rr = lane & 7, gid = lane >> 2, tig = lane & 3;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t af[4];
        const int t = (mi & 1) * 8 + rr, u16 = ks * 2 + (mi >> 1);
        ldmatrix_x4(xa + (uint32_t)((t * kH + h) * 128 + ((u16 ^ h) << 4)), af);
        const uint4 wf = wfr[ks * 32];
        mma_bf16_16816(d, af, wf.x, wf.y);
        mma_bf16_16816(d, af, wf.z, wf.w);
      }
      float* pw = part + (s * kH + h) * (kT * kH);
      *reinterpret_cast<float2*>(pw + gid * kH + 2 * tig) = make_float2(d[0], d[1]);
      *reinterpret_cast<float2*>(pw + (gid + 8) * kH + 2 * tig) = make_float2(d[2], d[3]);
      group_sync(grp);
      const float* ps = part + s * kH * (kT * kH) + (lane & 15) * kH + h;
      float logit = bias_h;
#pragma unroll
      for (int w = 0; w < kH; ++w) logit += ps[w * (kT * kH)];
      const float sg = 1.0f / (1.0f + __expf(-logit));
      lam = fminf(fmaxf(lam_base + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
    } else {
      const int tq = min(t0 + (lane & 15), p.S - 1);
      lam = p.lam_tok ? __ldg(p.lam_tok + ((size_t)b * p.S + tq) * kH + h) : lam_base;
    }
    if (t0 + (lane & 15) >= p.S) lam = 1.f;  // past the end: the state is carried unchanged
    // inclusive decay products within the chunk; token 0 of the sequence takes
    // the carried-in state itself, so nothing before it carries through
    float P = (first && (lane & 15) == 0) ? 0.f : lam;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      const float v = __shfl_up_sync(0xffffffffu, P, o, 16);
      if ((lane & 15) >= o) P *= v;
    }
    const float Achunk = __shfl_sync(0xffffffffu, P, 15);
    if (lane < kT) tab[lane] = make_float4(lam, 1.f - lam, P, 0.f);
    __syncwarp();

    // ---- evaluate once, EMA from zero (chunk 0: from the carried-in state)
    float2 st[kT];
    float2 s2 = first ? init2 : make_float2(0.f, 0.f);
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(xs + xoff + t * (kH * 128));
      const float4 tb = tab[t];
      const float2 u = u_fast(raw, m);
      if (t == 0 && first)  // a NaN u must survive the clamp to reach the check below
        s2 = make_float2(clamp1_nan(fmaf(tb.x, s2.x, tb.y * u.x)), clamp1_nan(fmaf(tb.x, s2.y, tb.y * u.y)));
      else
        s2 = fma2(make_float2(tb.x, tb.x), s2, mul2(make_float2(tb.y, tb.y), u));
      st[t] = s2;
    }
    // NaN / inf inputs: the chunk record with the reference's semantics
    const bool exact = __any_sync(0xffffffffu, s2.x != s2.x || s2.y != s2.y);
    if (exact) s2 = exact_run(xs + xoff, tab, m, first ? init2 : make_float2(0.f, 0.f), first, kT);
    // the last warp to leave a stage refills it with chunk c + 2 dC
    auto release = [&]() {
      __syncwarp();
      if (lane == 0 && atomicAdd(left + s, 1u) == kH - 1) {
        atomicExch(left + s, 0u);
        if (c + 2 * dC < p.nchunks) issue(s, c + 2 * dC);
      }
    };
    if (!exact) release();

    // ---- publish the chunk record
    const uint32_t tg = tag_of(epoch, c);
    const int slot = c & (kRing - 1);
    st_rec(p.agg + ((size_t)chain * kRing + slot) * 32 + lane, s2, tg);
    if (lane == 0) st_word(reinterpret_cast<unsigned long long*>(p.arec + (size_t)chain * kRing + slot), Achunk, tg);

    // ---- the state entering the chunk
    float2 X = make_float2(0.f, 0.f);
    if (!first) {
      const uint4* ip = p.inc + ((size_t)chain * kRing + ((c - 1) & (kRing - 1))) * 32 + lane;
      ok = wait_carry(ip, tag_of(epoch, c - 1), lane, ok, X);
    }

    // ---- outputs
    __nv_bfloat16* op = p.out + ((size_t)b * p.S + t0) * kD + h * kHD + j0;
    const int nt = min(kT, p.S - t0);
    if (exact) {
      exact_run(xs + xoff, tab, m, first ? init2 : X, first, nt, op);
      release();
    } else if (nt == kT) {
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        const float Pt = tab[t].z;
        st2(op + (size_t)t * kD, fma2(make_float2(Pt, Pt), X, st[t]));
      }
    } else {
#pragma unroll
      for (int t = 0; t < kT; ++t)
        if (t < nt) {
          const float Pt = tab[t].z;
          st2(op + (size_t)t * kD, fma2(make_float2(Pt, Pt), X, st[t]));
        }
    }
    __syncwarp();  // tab is rewritten by the next item
  }
  return ok;
}

template <bool GATE>
__global__ void __launch_bounds__(kNT, 1) sp_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&p.ws->epoch);  // advanced only after all CTAs left
  bool ok = true;
  if ((int)blockIdx.x >= p.nwcta) {
    const int rw = ((int)blockIdx.x - p.nwcta) * kRelayPerCta + w;
    if (w < kRelayPerCta && rw < p.B * kH)
      ok = relay(p.agg, p.arec, p.inc, p.fin, p.nchunks, rw / kH, rw % kH, lane, epoch,
                 reinterpret_cast<uint4*>(sm) + w * kNB * kBat * kRelaySlot);
  } else {
    const int grp = w / kH, unit = (int)blockIdx.x * kGroups + grp;
    if (unit < p.nunits) ok = work<GATE>(&tmap_x, p, sm + grp * kGroupSmem, unit, grp, w % kH, lane, epoch);
  }
  const int bad = __syncthreads_or(!ok);
  if (threadIdx.x == 0) {
    if (bad) {
      atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
      atomicAdd(&p.ws->timeouts, 1u);
    }
    __threadfence();
    if (atomicAdd(&p.ws->exited, 1u) == gridDim.x - 1) {  // the last CTA to leave advances the epoch
      atomicExch(&p.ws->exited, 0u);
      atomicExch(&p.ws->epoch, epoch + 1u);
    }
  }
}

// [B, S, 512] bf16 as a 4D map (64 channels, 8 heads, S tokens, B) with a
// [1, 16, 8, 64] box (one chunk, all heads), 128-byte swizzle.
bool encode_map4(CUtensorMap* map, const void* base, int S, int B, long long ss, long long sb) {
  cuuint64_t dims[4] = {(cuuint64_t)kHD, (cuuint64_t)kH, (cuuint64_t)S, (cuuint64_t)B};
  const long long sbb = B > 1 ? sb : (long long)S * ss;
  cuuint64_t strides[3] = {(cuuint64_t)kHD * 2, (cuuint64_t)ss * 2, (cuuint64_t)sbb * 2};
  cuuint32_t box[4] = {(cuuint32_t)kHD, (cuuint32_t)kH, (cuuint32_t)kT, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fast::encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t ring_bytes(int B) { return (size_t)B * kH * kRing * 32 * 16; }

}  // namespace sp
}  // namespace ossm

using namespace ossm;

bool ossm_tc_eligible(const ossm_fwd_args* a);

// The relay path: bf16 in and out (not precise), contiguous output, 4 to 32
// sequences, fewer than 2^19 chunks.
bool ossm_sp_eligible(const ossm_fwd_args* a) {
  if (!ossm_tc_eligible(a)) return false;
  if (a->out_dtype != OSSM_BF16 || (a->flags & OSSM_F_PRECISE)) return false;
  if (a->out_stride_s != sp::kD || (a->B > 1 && a->out_stride_b != (long long)a->S * sp::kD)) return false;
  if (a->B < 4 || a->B > 32) return false;
  const long long nch = ((long long)a->S + sp::kT - 1) / sp::kT;
  return nch < (1LL << 19);
}

size_t ossm_sp_workspace_bytes(const ossm_fwd_args* a) {
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  return al(sizeof(WsHeader)) + 2 * al(sp::ring_bytes(a->B)) + al((size_t)a->B * sp::kH * sp::kRing * 16);
}

int ossm_sp_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st) {
  using namespace sp;
  Params p;
  p.B = a->B;
  p.S = a->S;
  p.K = (a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_CLENSHAW_DEG4 ? (a->degree < 4 ? a->degree : 4) : a->degree;
  p.nchunks = (a->S + kT - 1) / kT;
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
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  size_t off = al(sizeof(WsHeader));
  p.ws = reinterpret_cast<WsHeader*>(ws);
  p.agg = reinterpret_cast<uint4*>(ws + off);
  off += al(ring_bytes(a->B));
  p.inc = reinterpret_cast<uint4*>(ws + off);
  off += al(ring_bytes(a->B));
  p.arec = reinterpret_cast<uint4*>(ws + off);

  CUtensorMap mx;
  if (!encode_map4(&mx, a->x, a->S, a->B, a->x_stride_s, a->x_stride_b)) return OSSM_EINVAL;
  void (*kern)(const CUtensorMap, const Params) = gate ? sp_kernel<true> : sp_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc) != cudaSuccess)
    return OSSM_ELAUNCH;
  int dev = 0, nsm = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNT, kSmemAlloc) != cudaSuccess)
    return OSSM_ELAUNCH;
  // every CTA must be resident at once (workers and relays wait on each other)
  const int nrc = (a->B * kH + kRelayPerCta - 1) / kRelayPerCta;
  const long long wslots = (long long)per_sm * nsm - nrc;
  long long nu = (wslots * kGroups / a->B) * a->B;
  nu = std::min<long long>(nu, (long long)a->B * p.nchunks);    // no more units than items
  nu = std::min<long long>(nu, (long long)(kRing - 2) * a->B);  // ring reuse: chunk stride dC <= kRing - 2
  if (nu < a->B) return OSSM_ELAUNCH;
  p.nunits = (int)nu;
  p.nwcta = (int)((nu + kGroups - 1) / kGroups);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.nwcta + nrc));
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = kSmemAlloc;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mx, p);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
