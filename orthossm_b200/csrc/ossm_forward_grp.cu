// Single-evaluation forward for bf16 activations, 8 heads x head_dim 64,
// bf16 output (sm_100a): a persistent grid of one CTA per SM, each sequence
// owned by a group of CTAs that exchange their tile aggregates through a ring
// in global memory.
//
// Same arithmetic contract as the three-pass path (ossm_forward_3p.cu) and the
// generic kernel (ossm_forward.cu), which restate _fused_clenshaw_ema_kernel
// (sdpc_kernel.py:988-1209): softsign, degree-8 Chebyshev (Horner on the
// gamma-folded monomial form), clamp, tanh, and the EMA
// s_t = a_t s_{t-1} + (1 - a_t) u_t with the per-token gate of BASELINE.json
// configs[1].
//
// Schedule.  The grid (cooperative launch: every CTA resident) is split into
// B groups; member m of group b (G_b members) takes tiles r * G_b + m of
// sequence b, a tile being 32 tokens x 512 channels, in rounds r.  In
// iteration r a CTA
//   1. evaluates tile r (warp = head, lane = channel pair, 32 tokens): the
//      tile was TMA-loaded two rounds ahead (three stages, CTA-local
//      destinations, no multicast); the decays come from the gate (an
//      mma.sync product with the weights split into bf16 hi + lo); every
//      element is evaluated ONCE and the EMA runs from a zero state, the local
//      states parked in tensor memory (tcgen05.st, three banks);
//   2. publishes tile r's aggregate (end state from zero per channel, decay
//      product per head) in the group's ring; its flag (tagged with the
//      launch epoch and the round) is released once the record is written;
//   3. folds round r - 2: its G_b records were bulk-loaded into shared memory
//      at the end of iteration r - 1, after their flags were seen, so the load
//      overlapped tile r's evaluation.  Every member folds the same records in
//      the same order from the state entering the round, so all agree bitwise
//      and nothing depends on timing: the carry of its tile r - 2 and the state
//      entering round r - 1;
//   4. writes tile r - 2's outputs: the parked states back (tcgen05.ld),
//      out = local + P_t * carry, coalesced bf16 stores;
// A ninth warp does the asynchronous work of every round: the x tiles' TMA
// loads, the flag release of the CTA's record, reading the group's flags and
// bulk-loading round r - 1's records into shared memory.  The 8 evaluation
// warps meet only mbarriers it feeds and one named barrier among themselves
// (the gate's partial sums), so the exchange latency stays off their path.
// x is read once and every element is evaluated once.
//
// Waits: every wait is bounded (mbarrier waits and flag polls give up, record
// OSSM_ETIMEOUT in the workspace header and the kernel finishes).
#include <cudaTypedefs.h>

#include <mutex>

#include "ossm_eval.cuh"

namespace ossm {
namespace fast {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
bool encode_map(CUtensorMap* map, const void* base, int S, int B, long long ss, long long sb, int rows);
}  // namespace fast
}  // namespace ossm

namespace ossm {
namespace grp {

using namespace ev;
using namespace sm100;

constexpr int kEW = 8;            // evaluation warps: one per head, all 32 tokens of the tile
constexpr int kNT = (kEW + 1) * 32;  // + one exchange warp
constexpr int kH = 8;             // heads
constexpr int kHD = 64;           // channels per head
constexpr int kD = kH * kHD;      // 512
constexpr int kT = kL;            // tokens per tile (32)
constexpr int kStages = 3;        // x stages
constexpr int kAhead = 2;         // rounds a load is issued ahead
constexpr int kBox = kT * 128;    // one head's [32 x 128 B] box
constexpr int kTile = kH * kBox;  // 32 KB
constexpr int kPartRow = kT + 4;  // gate partials [8 channel groups][8 outputs][32 + 4]
constexpr int kRec = kD + kH;     // aggregate record: 512 end states, 8 decay products (f32)
constexpr int kRecBytes = kRec * 4;
constexpr int kMaxG = 19;         // members per group at most (shared-memory staging)
constexpr int kRing = 6;          // rounds a group's ring holds
constexpr int kLag = 2;           // rounds between a tile's evaluation and its fold
// TMEM: warp w owns lanes 32 (w % 4) .. + 31 and columns 256 (w / 4) .. + 255:
// three 64-column banks of parked states (a channel pair per token), then 32
// columns of per-launch constants (the lane's monomial coefficients and gate
// fragments, reloaded every round so they hold no registers across the fold).
constexpr int kTmemCols = 512;
constexpr int kTmemConst = 192;
constexpr uint32_t kBarGate = 1;  // named barrier: the eight warps' gate partials

// shared memory map (from a 1024-byte aligned base: the swizzled TMA boxes)
constexpr int kOffX = 0;                                        // [kStages][kTile]
constexpr int kOffStage = kOffX + kStages * kTile;              // [2][kMaxG][kRec] a round's records
constexpr int kOffPart = kOffStage + 2 * kMaxG * kRecBytes;     // [2][8][8][kPartRow] gate partial logits
constexpr int kOffLam = kOffPart + 2 * kH * kH * kPartRow * 4;  // [kH][kT] float2 (l, 1 - l)
constexpr int kOffP = kOffLam + kH * kT * 8;                    // [3][kH][kT] decay products within the tile
constexpr int kOffBar = kOffP + 3 * kH * kT * 4;  // mbarriers: full[3], empty[3], rec[2], recfree[2], pub[4]
constexpr int kOffTmem = kOffBar + 14 * 8;        // TMEM base address
constexpr int kSmem = kOffTmem + 16 + 1024;       // + alignment slack
static_assert(kSmem <= 227 * 1024, "shared memory");
static_assert(kRecBytes % 16 == 0 && kOffStage % 16 == 0, "bulk copy alignment");

struct Params {
  int B, S, K, Kd, ntiles;  // K degrees used of the coefficient tensor's Kd
  const float* coeffs;
  const float* lam_h;
  float momentum;
  const float* gate_w;
  const float* gate_b;
  float gate_scale, gate_lo, gate_hi;
  const float* lam_in;  // caller's per-token decay [B,S,H] or NULL
  const float* init;
  float* fin;
  __nv_bfloat16* out;
  long long osb, oss;   // output batch / token strides (elements)
  WsHeader* ws;
  float* ring;          // [B][kRing][kMaxG][kRec] published aggregates
  unsigned long long* flags;  // [B][kRing][kMaxG] tag(epoch, round)
};

// A flag's value for round r of the launch with this epoch, salted so that
// no small integer or float pair left in the workspace by another kernel
// reads as one.
OSSM_DEV unsigned long long flag_tag(unsigned long long epoch, int r) {
  return ((epoch << 32) | (unsigned long long)(r + 1)) ^ 0x9E3779B97F4A7C15ull;
}

OSSM_DEV void split_bf16x2(float2 w, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(w.x, w.y);
  lo = pack_bf16x2(w.x - __uint_as_float(hi << 16), w.y - __uint_as_float(hi & 0xffff0000u));
}

// The lane's 4 bytes of token t in a head's 128-byte-swizzled [32 x 128 B]
// box: t*128 + ((lane/4 ^ t%8) * 16) + (lane%4)*4 = t*128 + (base ^ 16 (t%8)).
OSSM_DEV uint32_t box_lane(uint32_t base, int t) { return (uint32_t)(t * 128) + (base ^ (uint32_t)((t & 7) << 4)); }

// The 32-token EMA of one head's tile from state s: u evaluated once per
// element; the states are parked in TMEM (columns tcol .. tcol + 63, a pair
// of channels per token) eight tokens at a time.  After each eight tokens,
// part(i) runs: the caller's independent work (an older tile's outputs),
// which the scheduler overlaps with the evaluation's arithmetic.
template <bool EXACT, typename PartF>
OSSM_DEV float2 tile_scan(float2 s, const uint8_t* xs, uint32_t base, const float2* lam, bool first,
                          const float2 (&cm)[8], float gamma, uint32_t tcol, PartF part_done) {
#pragma unroll
  for (int part = 0; part < kT / 8; ++part) {
    // the eight tokens' u first (independent of each other and of the state,
    // so their evaluations interleave), then the EMA through them
    float2 u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      u[k] = eval_u<false, EXACT>(*reinterpret_cast<const uint32_t*>(xs + box_lane(base, part * 8 + k)), cm, gamma);
    uint32_t L[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int t = part * 8 + k;
      s = ema_step(s, lam[t], u[k], first && t == 0);
      L[2 * k] = __float_as_uint(s.x);
      L[2 * k + 1] = __float_as_uint(s.y);
    }
    tmem_st16(tcol + (uint32_t)(part * 16), L);
    part_done(part);
  }
  return s;
}

OSSM_DEV unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
OSSM_DEV void st_release64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
OSSM_DEV void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Lane q < G's view of member q's flag of round r (an acquire load issued
// ahead, so that its latency passes while the warp evaluates its tile).
OSSM_DEV unsigned long long peek_flag(const Params& p, int b, int G, int r, int lane) {
  if (lane >= G) return 0;
  return ld_acquire64(p.flags + ((size_t)b * kRing + (size_t)(r % kRing)) * kMaxG + lane);
}

// Lanes q < G of the calling warp wait (bounded) until member q's flag of
// round r is out (`seen`: the value peek_flag returned earlier), then
// bulk-load its record into the staging slot; lane 0 first arms the slot's
// mbarrier for all G records.  Returns false if a flag never came.
OSSM_DEV bool load_round(const Params& p, int b, int G, int r, unsigned long long epoch, int lane,
                         unsigned long long seen, float* slot, uint64_t* bar) {
  if (lane == 0) mbar_expect_tx(bar, (uint32_t)(G * kRecBytes));
  __syncwarp();
  bool ok = true;
  if (lane < G) {
    const size_t e = ((size_t)b * kRing + (size_t)(r % kRing)) * kMaxG + lane;
    const unsigned long long want = flag_tag(epoch, r);
    uint32_t it = 0;
    while (seen != want) {
      if (++it >= kSpinLimit) {
        ok = false;
        break;
      }
      if (it > 32) __nanosleep(it > 1024 ? 256 : 32);
      seen = ld_acquire64(p.flags + e);
    }
    if (ok) {
      fence_proxy_async_all();  // the acquired record is read by the async proxy
      bulk_load(slot + (size_t)lane * kRec, p.ring + e * kRec, kRecBytes, bar);
    }
  }
  return __all_sync(0xffffffffu, ok);
}

template <bool GATE>
__global__ void __launch_bounds__(kNT, 1) grp_fwd_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stage = reinterpret_cast<float*>(sm + kOffStage);
  float* part_s = reinterpret_cast<float*>(sm + kOffPart);
  float2* lam_s = reinterpret_cast<float2*>(sm + kOffLam);
  float* P_s = reinterpret_cast<float*>(sm + kOffP);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);  // x tile landed, per stage
  uint64_t* empty = full + kStages;                            // x tile consumed by the 8 evaluation warps
  uint64_t* recbar = empty + kStages;                          // a round's records landed, per staging slot
  uint64_t* recfree = recbar + 2;                              // a round's records folded by the 8 warps
  // the 8 warps' parts of a round's record, per round mod 4: a warp reaches
  // round q's record only after all 8 consumed tile q - 3 (the x stages), so
  // after every writer arrived for round q - 4
  uint64_t* pubbar = recfree + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffTmem);
  __shared__ unsigned long long s_epoch;

  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int h = w & 7;
  const int j0 = lane * 2, ch = h * kHD + j0;
  // group b = blockIdx % B, member m = blockIdx / B, G members
  const int b = (int)(blockIdx.x % (unsigned)p.B), m = (int)(blockIdx.x / (unsigned)p.B);
  const int G = ((int)gridDim.x - b + p.B - 1) / p.B;
  const int rounds = (p.ntiles + G - 1) / G;
  const float gamma = 0.98f - 0.06f * (float)h / (float)kH;

  if (tid == 0) {
    s_epoch = (unsigned long long)atomicAdd(&p.ws->epoch, 0u);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kEW);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&recbar[s], 1);
      mbar_init(&recfree[s], kEW);
    }
    for (int s = 0; s < 4; ++s) mbar_init(&pubbar[s], kEW);
    fence_mbar_init();
  }
  __syncwarp();  // warp 0 reconverges before the warp-collective allocation
  if (w == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned long long epoch = s_epoch;
  bool ok = true;

  if (w == kEW) {
    // ------------------------------------------------ the exchange warp
    // Round r: the x tile kAhead rounds on, round r - 1's records (their flags
    // were read a round earlier, so the read's latency has passed), round r's
    // flag once the 8 writers are done, and a first look at round r's flags.
    auto load_x = [&](int r) {  // round r's tile into its stage, once the 8 warps are done with it
      const int tile = r * G + m, st = r % kStages;
      if (tile >= p.ntiles) return;
      if (r >= kStages) ok = mbar_wait(&empty[st], (uint32_t)(((r - kStages) / kStages) & 1)) && ok;
      mbar_expect_tx(&full[st], kTile);
#pragma unroll
      for (int hh = 0; hh < kH; ++hh)
        tma_load_3d(sm + kOffX + st * kTile + hh * kBox, &tmap_x, &full[st], hh * kHD, tile * kT, b);
    };
    if (lane == 0)
      for (int r = 0; r < kAhead && r < rounds; ++r) load_x(r);
    unsigned long long seen = 0;
    for (int r = 0; r < rounds + kLag; ++r) {
      if (lane == 0 && r + kAhead < rounds) load_x(r + kAhead);
      __syncwarp();
      const int nr = r - kLag + 1;  // folded in iteration nr + kLag
      if (nr >= 0 && nr < rounds) {
        if (nr >= 2) ok = mbar_wait(&recfree[nr & 1], (uint32_t)(((nr - 2) >> 1) & 1)) && ok;
        ok = load_round(p, b, G, nr, epoch, lane, seen, stage + (size_t)(nr & 1) * kMaxG * kRec, &recbar[nr & 1]) &&
             ok;
      }
      if (r < rounds) {  // round r's record is written: release its flag
        ok = mbar_wait(&pubbar[r & 3], (uint32_t)((r >> 2) & 1)) && ok;
        if (lane == 0) {
          __threadfence();
          st_release64(p.flags + ((size_t)b * kRing + (size_t)(r % kRing)) * kMaxG + m, flag_tag(epoch, r));
        }
        __syncwarp();
      }
      const int nn = nr + 1;
      seen = (nn >= 0 && nn < rounds) ? peek_flag(p, b, G, nn, lane) : 0ull;
    }
  } else {
    // ------------------------------------------------ the 8 evaluation warps (warp = head)
    const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
    const float bias_h = GATE ? __ldg(p.gate_b + h) : 0.f;
    const uint32_t xbase = (uint32_t)(((lane >> 2) << 4) | ((lane & 3) * 4));  // box_lane's lane part
    const uint32_t tmem = *tmem_slot;
    // this warp's TMEM: lanes of quarter w % 4, column block w / 4
    const uint32_t tm_base = tmem + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)((w >> 2) * 256);
    const uint32_t tm_const = tm_base + (uint32_t)kTmemConst;
    {  // per-launch constants into TMEM: the lane's two channels' coefficients in
       // the fast path's form, the gate's weight fragments split bf16 hi + lo
      float2 cm[8];
      load_coeffs<false>(p.coeffs, p.Kd, p.K, b, h, j0, gamma, cm);
      uint32_t cv[16], fv[16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cv[2 * q] = __float_as_uint(cm[q].x);
        cv[2 * q + 1] = __float_as_uint(cm[q].y);
      }
      tmem_st16(tm_const, cv);
      if (GATE) {
        const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const float* wr = p.gate_w + (size_t)gid * kD + h * kHD + ks * 16 + 2 * tig;
          split_bf16x2(__ldg(reinterpret_cast<const float2*>(wr)), fv[4 * ks], fv[4 * ks + 2]);
          split_bf16x2(__ldg(reinterpret_cast<const float2*>(wr + 8)), fv[4 * ks + 1], fv[4 * ks + 3]);
        }
        tmem_st16(tm_const + 16u, fv);
      }
      tmem_wait_st();
    }

    float2 Z = make_float2(0.f, 0.f);  // state entering the round folded next
    __nv_bfloat16* const outp = p.out + (size_t)b * p.osb + ch;  // this lane's channel pair of sequence b

    // The decays of tile r (per-token gate or given) into lam_s, their
    // products within the tile into P_s bank r % 3; returns the tile's decay
    // product.  The tile's x must have landed.
    auto decays = [&](int r, const uint32_t (&fv)[16]) -> float {
      const int tile = r * G + m, st = r % kStages;
      const uint8_t* xs = sm + kOffX + st * kTile + h * kBox;
      const int tg = tile * kT + lane;  // this lane's token
      float lam;
      if (GATE) {  // this head's 64-channel partial logits of all 8 gate outputs, then the sums
        const uint32_t xa = smem_u32(xs);
        const int mm = lane >> 3, rr = lane & 7, gid = lane >> 2, tig = lane & 3;
        float* pw = part_s + (size_t)(r & 1) * (kH * kH * kPartRow) + h * (kH * kPartRow);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // hi and lo products apart
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            uint32_t av[4];
            ldmatrix_x4(xa + box_off(mt * 16 + (mm & 1) * 8 + rr, ks * 2 + (mm >> 1)), av);
            mma_bf16_16816(d, av, fv[4 * ks], fv[4 * ks + 1]);
            mma_bf16_16816(e, av, fv[4 * ks + 2], fv[4 * ks + 3]);
          }
          pw[(2 * tig) * kPartRow + mt * 16 + gid] = d[0] + e[0];
          pw[(2 * tig + 1) * kPartRow + mt * 16 + gid] = d[1] + e[1];
          pw[(2 * tig) * kPartRow + mt * 16 + gid + 8] = d[2] + e[2];
          pw[(2 * tig + 1) * kPartRow + mt * 16 + gid + 8] = d[3] + e[3];
        }
        named_sync(kBarGate, kEW * 32);  // all eight channel groups' partials
        const float* pr = part_s + (size_t)(r & 1) * (kH * kH * kPartRow) + h * kPartRow + lane;
        const float s0 = pr[0 * kH * kPartRow] + pr[1 * kH * kPartRow], s1 = pr[2 * kH * kPartRow] + pr[3 * kH * kPartRow];
        const float s2 = pr[4 * kH * kPartRow] + pr[5 * kH * kPartRow], s3 = pr[6 * kH * kPartRow] + pr[7 * kH * kPartRow];
        const float logit = bias_h + ((s0 + s1) + (s2 + s3));
        const float sg = 1.0f / (1.0f + __expf(-logit));
        lam = fminf(fmaxf(lam_base + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
        if (tg >= p.S) lam = 1.f;
      } else {
        lam = tg >= p.S ? 1.f : (p.lam_in ? __ldg(p.lam_in + ((size_t)b * p.S + tg) * kH + h) : lam_base);
      }
      float P = lam;  // decay products within the tile (inclusive)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float q = __shfl_up_sync(0xffffffffu, P, o);
        if (lane >= o) P *= q;
      }
      lam_s[h * kT + lane] = make_float2(lam, 1.f - lam);
      P_s[((r % 3) * kH + h) * kT + lane] = P;
      __syncwarp();
      return __shfl_sync(0xffffffffu, P, 31);
    };
    // Tile r's x has landed; the constants from TMEM (gate fragments only with
    // the gate).
    auto tile_ready = [&](int r, uint32_t (&cv)[16], uint32_t (&fv)[16]) {
      tmem_ld16_nowait(tm_const, cv);
      if (GATE) tmem_ld16_nowait(tm_const + 16u, fv);
      ok = mbar_wait(&full[r % kStages], (uint32_t)((r / kStages) & 1)) && ok;
      tmem_wait_ld();
    };

    float a_next = 1.f;  // the decay product of the tile evaluated next (its decays are ready)
    if (rounds > 0 && m < p.ntiles) {
      uint32_t cv[16], fv[16];
      tile_ready(0, cv, fv);
      a_next = decays(0, fv);
    }
    for (int r = 0; r < rounds + kLag; ++r) {
      const bool has_eval = r < rounds;
      const int tile = r * G + m;
      const bool valid = has_eval && tile < p.ntiles;

      // ---- 1. fold round r - kLag: that tile's carry and the next round's entry state
      float2 Xt = make_float2(0.f, 0.f);
      const int pr_ = r - kLag;
      if (pr_ >= 0) {
        const int slot = pr_ & 1;
        ok = mbar_wait(&recbar[slot], (uint32_t)((pr_ >> 1) & 1)) && ok;
        const float* A = stage + (size_t)slot * kMaxG * kRec;
        float2 X = Z;
        Xt = Z;
        for (int q = 0; q < G; ++q) {
          if (q == m) Xt = X;
          const float2 ev = *reinterpret_cast<const float2*>(A + (size_t)q * kRec + ch);
          const float aq = A[(size_t)q * kRec + kD + h];
          X = fma2(make_float2(aq, aq), X, ev);
        }
        Z = X;
        __syncwarp();
        if (lane == 0) mbar_arrive(&recfree[slot]);  // this warp is done with the slot
      }

      // ---- 2. tile r - kLag's outputs (out = local + P_t * carry), eight
      //      tokens after each eight tokens of tile r's evaluation
      const bool outs = pr_ >= 0 && pr_ * G + m < p.ntiles;
      const int pbank = outs ? pr_ % 3 : 0;
      const int t0 = outs ? (pr_ * G + m) * kT : 0;
      const int nt = outs ? min(kT, p.S - t0) : 0;  // tokens of that tile inside the sequence
      const float* Pp = P_s + (pbank * kH + h) * kT;
      __nv_bfloat16* op = outp + (size_t)t0 * p.oss;
      float2 v = Xt;
      auto out_part = [&](int part) {  // tokens 8 part .. 8 part + 7 of tile r - kLag
        float L[16];
        uint32_t Lu[16];
        tmem_ld16_nowait(tm_base + (uint32_t)(pbank * 64 + part * 16), Lu);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 16; ++k) L[k] = __uint_as_float(Lu[k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int t = part * 8 + k;
          const float Pk = Pp[t];
          v = fma2(make_float2(Pk, Pk), Xt, make_float2(L[2 * k], L[2 * k + 1]));
          if (t < nt) __stcs(reinterpret_cast<unsigned int*>(op + (size_t)t * p.oss), pack_bf16x2(v.x, v.y));
        }
      };
      float2 s_end = make_float2(0.f, 0.f);
      const float a_tile = a_next;
      __syncwarp();  // reconverged before the warp-collective TMEM accesses
      if (valid) {
        const int st = r % kStages;
        const uint8_t* xs = sm + kOffX + st * kTile + h * kBox;
        uint32_t cv[16];
        tmem_ld16_nowait(tm_const, cv);
        tmem_wait_ld();
        float2 cm[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) cm[q] = make_float2(__uint_as_float(cv[2 * q]), __uint_as_float(cv[2 * q + 1]));
        const bool first = tile == 0;  // token 0: the carried-in state enters here
        float2 s0 = make_float2(0.f, 0.f);
        if (first && p.init) s0 = __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + ch));
        const uint32_t tcol = tm_base + (uint32_t)((r % 3) * 64);
        if (outs)
          s_end = tile_scan<false>(s0, xs, xbase, lam_s + h * kT, first, cm, gamma, tcol, out_part);
        else
          s_end = tile_scan<false>(s0, xs, xbase, lam_s + h * kT, first, cm, gamma, tcol, [](int) {});
        // NaN / inf inputs: the whole warp recomputes its tile with the
        // reference's semantics (warp-uniform: the TMEM stores and waits are
        // warp-collective and must not sit in a divergent branch)
        if (__any_sync(0xffffffffu, s_end.x != s_end.x || s_end.y != s_end.y)) {
          tmem_wait_st();  // the fast states are out before their replacements go in
          s_end = tile_scan<true>(s0, xs, xbase, lam_s + h * kT, first, cm, gamma, tcol, [](int) {});
        }
        tmem_wait_st();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
      } else if (outs) {
#pragma unroll
        for (int part = 0; part < kT / 8; ++part) out_part(part);
      }
      // decays are 1 past the end, so the last tile's last state is the sequence's final state
      if (outs && p.fin && pr_ * G + m == p.ntiles - 1)
        *reinterpret_cast<float2*>(p.fin + (size_t)b * kD + ch) = make_float2(clamp1(v.x), clamp1(v.y));

      // ---- 3. tile r's aggregate into the ring (identity past the end); the
      //      exchange warp releases the flag once the 8 writers arrived
      if (has_eval) {
        float* rec = p.ring + (((size_t)b * kRing + (size_t)(r % kRing)) * kMaxG + m) * kRec;
        *reinterpret_cast<float2*>(rec + ch) = valid ? s_end : make_float2(0.f, 0.f);
        if (lane == 0) rec[kD + h] = valid ? a_tile : 1.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&pubbar[r & 3]);
      }

      // ---- 4. the next tile's decays (its x is resident: loaded two rounds ahead)
      if (r + 1 < rounds && (r + 1) * G + m < p.ntiles) {
        uint32_t cv[16], fv[16];
        tile_ready(r + 1, cv, fv);
        a_next = decays(r + 1, fv);
      }
    }
  }

  if (!ok && lane == 0) atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, kTmemCols);
  }
  if (tid == 0) {  // the last CTA to leave advances the epoch that tags the flags
    __threadfence();
    if (atomicAdd(&p.ws->exited, 1u) == gridDim.x - 1) {
      atomicExch(&p.ws->exited, 0u);
      atomicExch(&p.ws->epoch, (uint32_t)epoch + 1u);
    }
  }
}

template <bool GATE>
cudaError_t prepare() {
  auto kern = grp_fwd_kernel<GATE>;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

template <bool GATE>
cudaError_t launch(const CUtensorMap& mx, const Params& p, int grid, cudaStream_t st) {
  cudaError_t e = prepare<GATE>();
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<CUtensorMap*>(&mx), const_cast<Params*>(&p)};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(grp_fwd_kernel<GATE>), dim3(grid), dim3(kNT), args,
                                     (size_t)kSmem, st);
}

// CTAs of the grid on this device (one per SM, all resident: cooperative
// launch), or 0 if the device cannot run the kernel; queried once per device.
struct Support {
  std::once_flag once;
  int grid = 0;
};
Support g_support[64];

int grid_size() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  Support& s = g_support[dev];
  std::call_once(s.once, [&] {
    int coop = 0, nsm = 0, per0 = 0, per1 = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        prepare<false>() == cudaSuccess && prepare<true>() == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per0, grp_fwd_kernel<false>, kNT, kSmem) == cudaSuccess &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per1, grp_fwd_kernel<true>, kNT, kSmem) == cudaSuccess &&
        per0 >= 1 && per1 >= 1)
      s.grid = nsm;
    cudaGetLastError();  // a refused query leaves no sticky error behind
  });
  return s.grid;
}

}  // namespace grp
}  // namespace ossm

using namespace ossm;

bool ossm_p3_eligible(const ossm_fwd_args* a);

namespace {
// The grid for a batch of B sequences: every SM, as long as no group gets
// more members than the shared-memory staging holds.
int grp_grid(int B) {
  const int n = grp::grid_size();
  return n < B ? 0 : (n < B * grp::kMaxG ? n : B * grp::kMaxG);
}
size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }
}  // namespace

// The grouped path is taken when asked for (OSSM_F_SINGLE_EVAL) on the fast
// path with bf16 output (no precise flag) and every SM can take a group
// member: 8 to (SMs) sequences.
bool ossm_grp_eligible(const ossm_fwd_args* a) {
  if (!(a->flags & OSSM_F_SINGLE_EVAL) || !ossm_p3_eligible(a)) return false;
  if (a->out_dtype != OSSM_BF16 || (a->flags & OSSM_F_PRECISE)) return false;
  if (a->B < 8) return false;  // fewer groups of at most kMaxG members leave SMs idle: three-pass
  return grp_grid(a->B) > 0;
}

// Workspace of the grouped path: the header (epoch, exit counter, status),
// then the ring's flags and records.
size_t ossm_grp_workspace_bytes(const ossm_fwd_args* a) {
  const size_t n = (size_t)a->B * grp::kRing * grp::kMaxG;
  return al256(sizeof(WsHeader)) + al256(n * 8) + al256(n * grp::kRecBytes);
}

int ossm_grp_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st) {
  CUtensorMap mx;
  if (!fast::encode_map(&mx, a->x, a->S, a->B, a->x_stride_s, a->x_stride_b, grp::kT)) return OSSM_EINVAL;
  const int grid = grp_grid(a->B);
  if (grid <= 0) return OSSM_ELAUNCH;
  grp::Params p;
  p.B = a->B;
  p.S = a->S;
  p.K = (a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_CLENSHAW_DEG4 ? (a->degree < 4 ? a->degree : 4) : a->degree;
  p.Kd = a->degree;
  p.ntiles = (a->S + grp::kT - 1) / grp::kT;
  p.coeffs = a->coeffs;
  p.lam_h = a->lam_h;
  p.momentum = a->momentum;
  p.gate_w = a->gate_w;
  p.gate_b = a->gate_b;
  p.gate_scale = a->gate_scale;
  p.gate_lo = a->gate_lo;
  p.gate_hi = a->gate_hi;
  p.lam_in = a->lam_tok;
  p.init = a->init_state;
  p.fin = a->final_state;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.osb = a->out_stride_b;
  p.oss = a->out_stride_s;
  p.ws = reinterpret_cast<WsHeader*>(ws);
  const size_t n = (size_t)a->B * grp::kRing * grp::kMaxG;
  p.flags = reinterpret_cast<unsigned long long*>(ws + al256(sizeof(WsHeader)));
  p.ring = reinterpret_cast<float*>(ws + al256(sizeof(WsHeader)) + al256(n * 8));
  const bool gate = a->gate_w && !a->lam_tok;
  const cudaError_t e = gate ? grp::launch<true>(mx, p, grid, st) : grp::launch<false>(mx, p, grid, st);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}
