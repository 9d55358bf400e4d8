// Three-pass forward for bf16 activations, 8 heads x head_dim 64 (sm_100a).
//
// Same arithmetic contract as fwd_scan_kernel in ossm_forward.cu (which
// restates _fused_clenshaw_ema_kernel, sdpc_kernel.py:988-1209).  The EMA
// s_t = a_t s_{t-1} + (1 - a_t) u_t is a first-order linear recurrence, so the
// sequence is split into 32-token chunks and solved in three launches, none of
// which waits on another CTA:
//
//   p3_agg_kernel    one CTA per (b, chunk), warp = head: TMA-loads the
//                    [32 x 512] tile, forms the decays (the optional gate as a
//                    [32 x 512] . [512 x 8] tensor-core product with the weights
//                    held in registers), evaluates u and runs the EMA from a zero
//                    state.  Writes the chunk's end state and decay product (and
//                    the per-token decays when gated).
//   p3_carry_kernel  one CTA per (b, h) chain and block of 512 chunks: the
//                    carry into every chunk, c_k = A_{k-1} c_{k-1} + agg_{k-1},
//                    in a fixed order (32 spans of 16 chunks folded in
//                    parallel, then across spans); p3_blockfold_kernel joins
//                    the blocks of chains longer than one block.
//   p3_out_kernel    one CTA per (b, chunk), warp = head: re-reads x, evaluates
//                    u again and runs the EMA from the chunk's carry, writing
//                    each output as it is produced.  For fp32 outputs that fit
//                    in half of L2, the aggregate pass parks u in the output
//                    rows instead and p3_outu_kernel reads it back (no second
//                    evaluation).
//
// bf16 outputs of sequences holding at most 24 MB of u take the parked path
// instead: the batch runs as slabs of sequences on up to five streams, the
// aggregate pass (ring mode) also parks each u as an fp16 pair in an
// L2-resident ring slot and forms the carries itself (the last CTA of each
// 16-chunk span, then of the sequence, folds the records: atomic tickets, no
// waiting), and p3_outp_kernel reads u back from L2 and drops its lines, so
// every element is evaluated once and x is read once.
//
// Every launch streams with high occupancy and no inter-CTA waits; on the
// re-evaluating path the price is a second evaluation and a second read of
// x.  Results are bitwise reproducible (every fold has a fixed order).
//
// NaN inputs are handled off the hot path: the fast evaluation lets them
// surface as NaN, each warp checks its chunk once and recomputes it with the
// reference's semantics (u = 0 there).
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "ossm_eval.cuh"

namespace ossm {
namespace fast {

constexpr int kH = 8;    // heads
constexpr int kHD = 64;  // channels per head
constexpr int kD = kH * kHD;

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
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

// [B, S, 512] bf16 as a 3-D map (channel, token, sequence) whose box is one
// head's [rows x 64] channels, 128-byte swizzle.
bool encode_map(CUtensorMap* map, const void* base, int S, int B, long long ss, long long sb, int rows) {
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)S, (cuuint64_t)B};
  const long long sbb = B > 1 ? sb : (long long)S * ss;
  cuuint64_t strides[2] = {(cuuint64_t)ss * 2, (cuuint64_t)sbb * 2};
  cuuint32_t box[3] = {(cuuint32_t)kHD, (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace fast
}  // namespace ossm

// The bf16 fast path applies: bf16 x, 8 heads of 64, Clenshaw evaluation with
// the fused semantics, no tanh cache, 16-byte aligned rows (TMA).
bool ossm_p3_eligible(const ossm_fwd_args* a) {
  using namespace ossm::fast;
  if (a->x_dtype != OSSM_BF16 || a->H != kH || a->head_dim != kHD || a->tanh_out) return false;
  if ((a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_LUT || (a->flags & (OSSM_F_FASTPATH | OSSM_F_GENERIC))) return false;
  if (((uintptr_t)a->x % 16) || (a->x_stride_s % 8) || (a->B > 1 && (a->x_stride_b % 8))) return false;
  if (a->out_dtype == OSSM_BF16 &&
      (((uintptr_t)a->out % 16) || (a->out_stride_s % 8) || (a->B > 1 && (a->out_stride_b % 8))))
    return false;
  if (a->S > (1 << 30)) return false;
  return encode_fn() != nullptr;
}

namespace ossm {
namespace p3 {

using namespace ev;

constexpr int kNT = 256;
constexpr int kH = fast::kH;    // heads (one warp each)
constexpr int kHD = fast::kHD;  // channels per head
constexpr int kD = kH * kHD;
constexpr int kBox = kL * 128;       // one head's [32 x 128 B] box
constexpr int kTile = kH * kBox;     // 32 KB
// partial gate logits: [8 warps][8 gate outputs][32 tokens + 4] f32; the pad
// puts the mma fragment writes and the per-token reads in 32 distinct banks
constexpr int kPartRow = kL + 4;
constexpr int kOffPart = kTile;
constexpr int kOffLam = kOffPart + kH * kH * kPartRow * 4;  // [8 heads][32] float2 (l, 1 - l)
constexpr int kOffBar = kOffLam + kH * kL * 8;
constexpr int kAggSmem = kOffBar + 16 + 1024;        // + alignment slack
constexpr int kSpans = 32;                           // carry kernel: warps per block
constexpr int kPer = 16;                             // carry kernel: chunks per warp
constexpr int kBlk = kSpans * kPer;                  // chunks per carry block

struct Params {
  int B, S, K, Kd, nchunks;  // K degrees used of the coefficient tensor's Kd
  const __nv_bfloat16* x;
  long long xsb, xss;
  const float* coeffs;
  const float* lam_h;
  float momentum;
  const float* gate_w;
  const float* gate_b;
  float gate_scale, gate_lo, gate_hi;
  const float* lam_in;  // caller's per-token decay [B,S,H] or NULL
  float* lam_ws;        // per-token decays written by the gate [B,S,H] (workspace)
  float4* cmono;        // [B*8][4][32]: each lane's gamma-folded, 4^-k-scaled monomial coefficients
  uint4* wfrag;         // [8][4][32]: each lane's mma B fragments of the gate weights, bf16 hi + lo
  const float* init;
  float* fin;
  void* out;
  long long osb, oss;
  float* A;      // [N] chunk decay products
  float* agg;    // [N][64] chunk end states from zero (chunk 0: from the carried-in state)
  float* carry;  // [N][64] state entering each chunk (from a zero state at its carry block's start)
  float* P;      // [N] decay product from the carry block's start to each chunk's start
  int nblk;      // carry blocks per chain (kBlk chunks each)
  float* blk_A;  // [B*H*nblk] block decay products
  float* blk_E;  // [B*H*nblk][64] block end states from a zero state
  float* blk_X;  // [B*H*nblk][64] state entering each block (from a zero state at the shard start)
  float* blk_P;  // [B*H*nblk] decay product from the shard start to each block's start
  WsHeader* ws;  // sticky status (a tile that never arrived)
  int starts_seq;         // this call's first token is token 0 of the sequence
  float* tot_A;           // [B*H] shard decay products (or NULL)
  float* tot_E;           // [B*H][64] shard end states from a zero state (or NULL)
  const float* carry_in;  // [B][D] state entering the shard (or NULL: zero / init_state)
  float* shard_carry;     // [B][D] workspace slot where a sharded call folds carry_in
  // 1: the aggregate pass parks u (fp32) in the fp32 output buffer and the
  // output pass reads it back instead of evaluating again
  int uc;
  // bf16 outputs: the aggregate pass parks u as fp16 pairs in this L2-resident
  // ring slot, [B][nchunks][8 heads][32 tokens][32 lanes] words, and the
  // output pass reads it back (or NULL: the output pass evaluates again)
  uint32_t* park;
  // With park, the aggregate pass also forms the carries (no carry pass):
  // spans of kSpanC chunks, folded by the span's last CTA to finish (an
  // atomic ticket per span), then the spans folded by the sequence's last.
  int nsp;            // spans per sequence
  uint32_t* tk_span;  // [B][nsp] tickets (zero between launches)
  uint32_t* tk_seq;   // [B] tickets
  float* spA;         // [B*8][nsp] span decay products
  float* spE;         // [B*8][nsp][64] span end states from zero
  float* spX;         // [B*8][nsp][64] state entering each span
  uint32_t* zero_ptr;  // p3_prep_kernel clears these words first (or NULL)
  int zero_n;
};
constexpr int kSpanC = 16;  // chunks per span of the in-pass carry

// How the aggregate pass hands u to the output pass.
constexpr int kUNone = 0;  // not at all: the output pass evaluates again
constexpr int kURows = 1;  // fp32, in the fp32 output rows
constexpr int kURing = 2;  // fp16 pairs, in the ring slot p.park

// L2 policies: the parked u kept before streamed data, x (read once) first out.
OSSM_DEV uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
OSSM_DEV uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
OSSM_DEV void st_park(uint32_t* p, uint32_t v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.b32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}
// Drop a 128-byte line of parked u from L2 without writing it back to HBM
// (its last reader has it in registers).
OSSM_DEV void discard_l2(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}
OSSM_DEV uint32_t pack_f16x2(float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
OSSM_DEV float2 unpack_f16x2(uint32_t w) { return __half22float2(*reinterpret_cast<const __half2*>(&w)); }

// w = hi + lo with hi = bf16(w) and lo = bf16(w - hi), for a pair of weights,
// with packed conversions only (the scalar float -> bf16 conversion would
// take the MUFU pipe the evaluation is bound by).
OSSM_DEV void split_bf16x2(float2 w, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(w.x, w.y);
  lo = pack_bf16x2(w.x - __uint_as_float(hi << 16), w.y - __uint_as_float(hi & 0xffff0000u));
}

// The lane's 16 prepared monomial coefficients of head h of sequence b.
OSSM_DEV void load_mono(const Params& p, int b, int h, int lane, float2 (&m)[8]) {
  const float4* src = p.cmono + (size_t)(b * kH + h) * 4 * 32 + lane;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = __ldg(src + q * 32);
    m[2 * q] = make_float2(v.x, v.y);
    m[2 * q + 1] = make_float2(v.z, v.w);
  }
}

// The per-CTA setup of the streaming kernels, done once per launch: warp
// (b, h) converts head h's coefficients of sequence b for the fast path
// (MONO), and with the gate warp h splits the weight columns of head h into
// its lanes' mma fragments.  The same arithmetic the kernels did inline, so
// the results are bitwise those of an inline setup.
template <bool MONO, bool GATE>
__global__ void __launch_bounds__(32) p3_prep_kernel(const Params p) {
  const int lane = threadIdx.x;
  if (p.zero_ptr && blockIdx.x == 0)
    for (int i = lane; i < p.zero_n; i += 32) p.zero_ptr[i] = 0u;
  const int nmono = MONO ? p.B * kH : 0;
  if ((int)blockIdx.x < nmono) {
    const int b = blockIdx.x / kH, h = blockIdx.x % kH;
    const float gamma = 0.98f - 0.06f * (float)h / (float)kH;
    float2 cm[8];
    load_coeffs<false>(p.coeffs, p.Kd, p.K, b, h, lane * 2, gamma, cm);
    float4* dst = p.cmono + (size_t)blockIdx.x * 4 * 32 + lane;
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q * 32] = make_float4(cm[2 * q].x, cm[2 * q].y, cm[2 * q + 1].x, cm[2 * q + 1].y);
  } else if (GATE) {
    const int h = blockIdx.x - nmono;
    const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float* wr = p.gate_w + (size_t)gid * kD + h * kHD + ks * 16 + 2 * tig;
      uint32_t hi0, lo0, hi1, lo1;
      split_bf16x2(__ldg(reinterpret_cast<const float2*>(wr)), hi0, lo0);
      split_bf16x2(__ldg(reinterpret_cast<const float2*>(wr + 8)), hi1, lo1);
      p.wfrag[(h * 4 + ks) * 32 + lane] = make_uint4(hi0, hi1, lo0, lo1);
    }
  }
}

// Decay of token (t0 + lane), head h, from a per-token input or the constant.
OSSM_DEV float lam_token(const Params& p, const float* lam_tok, int b, int tg, int h, float lam_base) {
  if (tg >= p.S) return 1.f;  // past the end: the state is carried unchanged
  return lam_tok ? __ldg(lam_tok + ((size_t)b * p.S + tg) * kH + h) : lam_base;
}

// The carries of a parked-u launch, formed at the end of the aggregate pass
// without waiting on other CTAs: after writing its records, the CTA of chunk
// c takes a ticket of its span; the span's last CTA (its ticket is the
// span's chunk count less one) folds the span's records in chunk order into
// each chunk's carry and decay product from the span start (p.carry, p.P)
// and the span's own record (spA, spE).  It then takes a ticket of the
// sequence; the sequence's last folds the span records in span order into
// the state entering each span (spX).  A CTA's threads write, meet at a
// barrier, and one thread takes the ticket with an acquire-release atomic at
// GPU scope (its release is cumulative over the CTA's writes ordered before
// by the barrier; its acquire orders the records a last CTA's threads read
// after the next barrier).  Each last CTA resets its ticket for the next
// slab that uses this workspace.
// flag: one int of shared memory.
// Ticket with release (the CTA's writes, ordered before by the barrier) and
// acquire (the records read after) semantics at GPU scope: the old count.
OSSM_DEV uint32_t ticket_acq_rel(uint32_t* t) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(t) : "memory");
  return old;
}
OSSM_DEV void ring_carries(const Params& p, int b, int c, int h, int lane, int* flag) {
  const int tid = threadIdx.x, j0 = lane * 2;
  const int sp = c / kSpanC, c0 = sp * kSpanC, cnt = min(kSpanC, p.nchunks - c0);
  __syncthreads();
  if (tid == 0) *flag = ticket_acq_rel(p.tk_span + (size_t)b * p.nsp + sp) == (uint32_t)(cnt - 1);
  __syncthreads();
  if (!*flag) return;
  const size_t nb = (size_t)(b * kH + h) * p.nchunks + c0;
  float2 X = make_float2(0.f, 0.f);
  float P = 1.f;
#pragma unroll 1
  for (int q0 = 0; q0 < cnt; q0 += 8) {  // 8 chunk records per batch of loads
    float a[8];
    float2 g[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const bool in = q0 + q < cnt;
      a[q] = in ? __ldcg(p.A + nb + q0 + q) : 1.f;
      g[q] = in ? __ldcg(reinterpret_cast<const float2*>(p.agg + (nb + q0 + q) * kHD) + lane) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q0 + q < cnt) {
        *reinterpret_cast<float2*>(p.carry + (nb + q0 + q) * kHD + j0) = X;
        if (lane == 0) p.P[nb + q0 + q] = P;
      }
      X = make_float2(fmaf(a[q], X.x, g[q].x), fmaf(a[q], X.y, g[q].y));
      P *= a[q];
    }
  }
  const size_t ks = (size_t)(b * kH + h) * p.nsp;
  *reinterpret_cast<float2*>(p.spE + (ks + sp) * kHD + j0) = X;
  if (lane == 0) p.spA[ks + sp] = P;
  __syncthreads();
  if (tid == 0) {
    p.tk_span[(size_t)b * p.nsp + sp] = 0u;
    *flag = ticket_acq_rel(p.tk_seq + b) == (uint32_t)(p.nsp - 1);
  }
  __syncthreads();
  if (!*flag) return;
  X = make_float2(0.f, 0.f);
#pragma unroll 1
  for (int s0 = 0; s0 < p.nsp; s0 += 8) {  // 8 span records per batch of loads
    float sa[8];
    float2 se[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const bool in = s0 + q < p.nsp;
      sa[q] = in ? __ldcg(p.spA + ks + s0 + q) : 1.f;
      se[q] = in ? __ldcg(reinterpret_cast<const float2*>(p.spE + (ks + s0 + q) * kHD) + lane) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (s0 + q < p.nsp) *reinterpret_cast<float2*>(p.spX + (ks + s0 + q) * kHD + j0) = X;
      X = make_float2(fmaf(sa[q], X.x, se[q].x), fmaf(sa[q], X.y, se[q].y));
    }
  }
  if (tid == 0) p.tk_seq[b] = 0u;
}

// ---------------------------------------------------------------------------
// pass 1: chunk aggregates
// ---------------------------------------------------------------------------
template <bool GATE, bool PRECISE, int UM>
__global__ void __launch_bounds__(kNT, 4) p3_agg_kernel(const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* part_s = reinterpret_cast<float*>(sm + kOffPart);
  float2* lam_s = reinterpret_cast<float2*>(sm + kOffLam);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int j0 = lane * 2;
  const int c = (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int t0 = c * kL, tg = t0 + lane;
  const float gamma = 0.98f - 0.06f * (float)h / (float)kH;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_expect_tx(bar, kTile);
    if (UM == kURing) {  // x is read once: its lines go before the parked u
      const uint64_t pol = policy_evict_first();
#pragma unroll
      for (int hh = 0; hh < kH; ++hh) tma_load_3d_hint(sm + hh * kBox, &tmap_x, bar, hh * kHD, t0, b, pol);
    } else {
#pragma unroll
      for (int hh = 0; hh < kH; ++hh) tma_load_3d(sm + hh * kBox, &tmap_x, bar, hh * kHD, t0, b);
    }
  }
  // while the tile lands: coefficients, gate weights (both prepared by
  // p3_prep_kernel on the fast path), the caller's decay
  float2 cm[8];
  if (PRECISE)
    load_coeffs<true>(p.coeffs, p.Kd, p.K, b, h, j0, gamma, cm);
  else
    load_mono(p, b, h, lane, cm);
  const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  float lam = GATE ? lam_base : lam_token(p, p.lam_in, b, tg, h, lam_base);
  uint32_t whi[4][2], wlo[4][2];  // mma B fragments of W[gid][h*64 + ks*16 + ...], split bf16 hi + lo
  float bias_h = 0.f;
  if (GATE) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint4 f = __ldg(p.wfrag + (h * 4 + ks) * 32 + lane);
      whi[ks][0] = f.x;
      whi[ks][1] = f.y;
      wlo[ks][0] = f.z;
      wlo[ks][1] = f.w;
    }
    bias_h = __ldg(p.gate_b + h);
  }
  __syncthreads();  // the mbarrier is initialised
  const bool ok = mbar_wait(bar, 0);
  const uint8_t* xs = sm + h * kBox;

  if (GATE) {  // this head's 64-channel partial logits for all 8 heads, then the sum
    const uint32_t xa = smem_u32(xs);
    const int m = lane >> 3, rr = lane & 7, gid = lane >> 2, tig = lane & 3;
    float* pw = part_s + h * (kH * kPartRow);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t a[4];
        // A: tokens mt*16 + (m&1)*8 + rr, channels ks*16 + (m>>1)*8 of this head
        ldmatrix_x4(xa + box_off(mt * 16 + (m & 1) * 8 + rr, ks * 2 + (m >> 1)), a);
        mma_bf16_16816(d, a, whi[ks][0], whi[ks][1]);
        mma_bf16_16816(d, a, wlo[ks][0], wlo[ks][1]);
      }
      // d: tokens mt*16 + gid (+8), gate outputs 2*tig (+1)
      pw[(2 * tig) * kPartRow + mt * 16 + gid] = d[0];
      pw[(2 * tig + 1) * kPartRow + mt * 16 + gid] = d[1];
      pw[(2 * tig) * kPartRow + mt * 16 + gid + 8] = d[2];
      pw[(2 * tig + 1) * kPartRow + mt * 16 + gid + 8] = d[3];
    }
    __syncthreads();
    float logit = bias_h;
#pragma unroll
    for (int g = 0; g < kH; ++g) logit += part_s[(g * kH + h) * kPartRow + lane];
    const float sg = 1.0f / (1.0f + __expf(-logit));
    lam = fminf(fmaxf(lam_base + p.gate_scale * (sg - 0.5f), p.gate_lo), p.gate_hi);
    if (tg < p.S) p.lam_ws[((size_t)b * p.S + tg) * kH + h] = lam;  // for the output pass
    else lam = 1.f;
  }
  const bool first = c == 0 && p.starts_seq;  // token 0 of the sequence: the carried-in state enters here
  float a = (first && lane == 0) ? 0.f : lam;  // the chunk's decay product
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) a *= __shfl_xor_sync(0xffffffffu, a, o);
  lam_s[h * kL + lane] = make_float2(lam, 1.f - lam);
  __syncwarp();

  float2 s = make_float2(0.f, 0.f);
  if (first && p.init) s = __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + h * kHD + j0));
  const float2 s_in = s;
  // the lane's 4 bytes of token t sit at t*128 + ((lane/4 ^ t%8) * 16) + (lane%4)*4: 8 row patterns
  uint32_t roff[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) roff[k] = (uint32_t)((((lane >> 2) ^ k) << 4) + (lane & 3) * 4);
  auto raw = [&](int t) { return *reinterpret_cast<const uint32_t*>(xs + roff[t & 7] + t * 128); };
  auto raw_t = [&](int t) {
    return *reinterpret_cast<const uint32_t*>(xs + box_off(t, lane >> 2) + (lane & 3) * 4);
  };
  if (UM == kURing) {  // park each u as an fp16 pair in the ring: one 128-byte line per warp and token
    uint32_t* up = p.park + ((size_t)(b * p.nchunks + c) * kH + h) * (kL * 32) + lane;
    const uint64_t pol = policy_evict_last();
    auto put = [&](int t, float2 u) { st_park(up + t * 32, pack_f16x2(u), pol); };
    s = ema_chunk_u<PRECISE, false>(s, lam_s + h * kL, first, cm, gamma, raw, put);
    if (__any_sync(0xffffffffu, s.x != s.x || s.y != s.y))  // NaN / inf inputs: the reference's semantics
      s = ema_chunk_u_exact<PRECISE>(s_in, lam_s + h * kL, first, cm, gamma, raw_t, put);
  } else if (UM == kURows) {  // park each u in the fp32 output row it will become (tokens past the end have no row)
    float* uo = static_cast<float*>(p.out) + (size_t)b * p.osb + (size_t)t0 * p.oss + h * kHD + j0;
    const int nt = min(kL, p.S - t0);
    auto put = [&](int t, float2 u) {
      if (t < nt) *reinterpret_cast<float2*>(uo + (size_t)t * p.oss) = u;
    };
    s = ema_chunk_u<PRECISE, false>(s, lam_s + h * kL, first, cm, gamma, raw, put);
    if (__any_sync(0xffffffffu, s.x != s.x || s.y != s.y))  // NaN / inf inputs: the reference's semantics
      s = ema_chunk_u_exact<PRECISE>(s_in, lam_s + h * kL, first, cm, gamma, raw_t, put);
  } else {
    auto none = [](int, float2) {};
    s = ema_chunk<PRECISE, false>(s, lam_s + h * kL, first, cm, gamma, raw, none);
    if (__any_sync(0xffffffffu, s.x != s.x || s.y != s.y))  // NaN / inf inputs: the reference's semantics
      s = ema_chunk_exact<PRECISE>(s_in, lam_s + h * kL, first, cm, gamma, raw_t, none);
  }
  const size_t n = (size_t)(b * kH + h) * p.nchunks + c;
  *reinterpret_cast<float2*>(p.agg + n * kHD + j0) = s;
  if (lane == 0) p.A[n] = a;
  if (!ok && lane == 0) atomicExch(&p.ws->status, (uint32_t)OSSM_ETIMEOUT);
  if (UM == kURing) ring_carries(p, b, c, h, lane, reinterpret_cast<int*>(sm + kOffBar + 8));
}

// ---------------------------------------------------------------------------
// pass 2: carries.  A chain's chunks are cut into blocks of kBlk; one CTA per
// (chain, block), warp w folds the block's span w of kPer chunks, lane = 2
// channels.  Each warp loads its whole span at once and keeps it in registers
// for the second fold, so the kernel makes one round trip to memory.  With
// more than one block per chain a second small kernel joins the blocks.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSpans * 32) p3_carry_kernel(const Params p) {
  __shared__ float2 spanB[kSpans][32];
  __shared__ float spanA[kSpans];
  __shared__ float2 spanX[kSpans][32];
  __shared__ float spanP[kSpans];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chain = (int)(blockIdx.x / p.nblk), blk = (int)(blockIdx.x - (unsigned)chain * p.nblk);
  const size_t n0 = (size_t)chain * p.nchunks;
  const int c0 = blk * kBlk + w * kPer, cnt = max(0, min(kPer, p.nchunks - c0));
  // the span's decays and aggregates; past the end a decay of 1 and a zero
  // aggregate leave every fold unchanged
  float Ac[kPer];
  float2 g[kPer];
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const bool in = q < cnt;
    Ac[q] = in ? __ldg(p.A + n0 + c0 + q) : 1.f;
    g[q] = in ? __ldg(reinterpret_cast<const float2*>(p.agg + (n0 + c0 + q) * kHD) + lane) : make_float2(0.f, 0.f);
  }
  float2 B = make_float2(0.f, 0.f);  // span aggregate: state after the span from zero, and its decay product
  float A = 1.f;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    B = make_float2(fmaf(Ac[q], B.x, g[q].x), fmaf(Ac[q], B.y, g[q].y));
    A *= Ac[q];
  }
  spanB[w][lane] = B;
  if (lane == 0) spanA[w] = A;
  __syncthreads();
  if (w == 0) {  // carries into the spans, in span order; the block's totals
    float2 X = make_float2(0.f, 0.f);
    float P = 1.f;
    for (int q = 0; q < kSpans; ++q) {
      spanX[q][lane] = X;
      spanP[q] = P;
      X = make_float2(fmaf(spanA[q], X.x, spanB[q][lane].x), fmaf(spanA[q], X.y, spanB[q][lane].y));
      P *= spanA[q];
    }
    if (p.nblk > 1) {
      const size_t k = (size_t)chain * p.nblk + blk;
      reinterpret_cast<float2*>(p.blk_E + k * kHD)[lane] = X;
      if (lane == 0) p.blk_A[k] = P;
    } else {
      if (p.tot_E) reinterpret_cast<float2*>(p.tot_E + (size_t)chain * kHD)[lane] = X;
      if (p.tot_A && lane == 0) p.tot_A[chain] = P;
    }
  }
  __syncthreads();
  float2 X = spanX[w][lane];
  float Pc = spanP[w];
#pragma unroll
  for (int q = 0; q < kPer; ++q)
    if (q < cnt) {
      reinterpret_cast<float2*>(p.carry + (n0 + c0 + q) * kHD)[lane] = X;
      if (lane == 0) p.P[n0 + c0 + q] = Pc;
      X = make_float2(fmaf(Ac[q], X.x, g[q].x), fmaf(Ac[q], X.y, g[q].y));
      Pc *= Ac[q];
    }
}

// The state entering each block of a chain (from a zero state at the shard
// start) and the decay product up to it, folded in block order; the chain's
// totals.  One warp per chain, lane = 2 channels, loads 8 blocks at a time.
__global__ void __launch_bounds__(32) p3_blockfold_kernel(const Params p) {
  const int chain = blockIdx.x, lane = threadIdx.x;
  const size_t k0 = (size_t)chain * p.nblk;
  float2 X = make_float2(0.f, 0.f);
  float P = 1.f;
  for (int kb = 0; kb < p.nblk; kb += 8) {
    float Ab[8];
    float2 E[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const size_t k = k0 + min(kb + q, p.nblk - 1);
      Ab[q] = __ldg(p.blk_A + k);
      E[q] = __ldg(reinterpret_cast<const float2*>(p.blk_E + k * kHD) + lane);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (kb + q < p.nblk) {
        reinterpret_cast<float2*>(p.blk_X + (k0 + kb + q) * kHD)[lane] = X;
        if (lane == 0) p.blk_P[k0 + kb + q] = P;
        X = make_float2(fmaf(Ab[q], X.x, E[q].x), fmaf(Ab[q], X.y, E[q].y));
        P *= Ab[q];
      }
  }
  if (p.tot_E) reinterpret_cast<float2*>(p.tot_E + (size_t)chain * kHD)[lane] = X;
  if (p.tot_A && lane == 0) p.tot_A[chain] = P;
}

// The state after the first `nshards` shards of a sequence-sharded call,
// from the all-gathered shard totals [nshards][B*H decays | B*D end states]
// and the state before the sequence (or zero): X_0 = init,
// X_{q+1} = decay_q X_q + state_q, in shard order on every rank, so every
// rank folds bitwise the same carries.  One thread per channel.
__global__ void __launch_bounds__(256) shard_fold_kernel(int B, int H, int hd, int nshards, const float* totals,
                                                         const float* init, float* state_out) {
  const int D = H * hd;
  const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= B * D) return;
  const int b = i / D, h = (i - b * D) / hd;
  const size_t stride = (size_t)B * H + (size_t)B * D;
  float X = init ? __ldg(init + i) : 0.f;
  for (int q = 0; q < nshards; ++q) {
    const float* t = totals + (size_t)q * stride;
    X = fmaf(__ldg(t + b * H + h), X, __ldg(t + (size_t)B * H + i));
  }
  state_out[i] = X;
}

// ---------------------------------------------------------------------------
// pass 3: outputs from the carries
// ---------------------------------------------------------------------------
// One chunk of one head: x and out with token strides XS / OS (elements;
// compile-time when the tensors are contiguous, so every access is an
// immediate offset), all 32 tokens (FULL) or the ragged last chunk.
template <typename Stride>
OSSM_DEV void load_chunk(const __nv_bfloat16* xp, Stride xs, uint32_t (&r)[kL]) {
#pragma unroll
  for (int t = 0; t < kL; ++t) r[t] = __ldcs(reinterpret_cast<const unsigned int*>(xp + t * xs));
}
// The chunk from its x words r (already loaded).
template <bool PRECISE, typename OT, typename Stride>
OSSM_DEV float2 out_chunk_loaded(const uint32_t (&r)[kL], const __nv_bfloat16* xp, OT* op, Stride xs, Stride os,
                                 float2 X, const float2* lam, bool first, const float2 (&cm)[8], float gamma) {
  auto raw = [&](int t) { return r[t]; };
  auto emit = [&](int t, float2 v) { st2(op + t * os, sizeof(OT) == 4 ? make_float2(clamp1(v.x), clamp1(v.y)) : v); };
  float2 s = ema_chunk<PRECISE, false>(X, lam, first, cm, gamma, raw, emit);
  if (__any_sync(0xffffffffu, s.x != s.x || s.y != s.y)) {  // NaN / inf inputs: redo with the reference's semantics
    auto reraw = [&](int t) { return __ldcs(reinterpret_cast<const unsigned int*>(xp + t * xs)); };
    s = ema_chunk_exact<PRECISE>(X, lam, first, cm, gamma, reraw, emit);
  }
  return s;
}
template <bool PRECISE, typename OT, typename Stride>
OSSM_DEV float2 out_chunk(const __nv_bfloat16* xp, OT* op, Stride xs, Stride os, float2 X, const float2* lam, bool first,
                          const float2 (&cm)[8], float gamma) {
  uint32_t r[kL];
  load_chunk(xp, xs, r);
  return out_chunk_loaded<PRECISE, OT>(r, xp, op, xs, os, X, lam, first, cm, gamma);
}
// The ragged last chunk (nt < 32 tokens), or strided tensors: a rolled loop
// with the reference's semantics throughout.
template <bool PRECISE, typename OT>
OSSM_DEV float2 out_chunk_general(const __nv_bfloat16* xp, OT* op, long long xs, long long os, int nt, float2 X,
                                  const float2* lam, bool first, const float2 (&cm)[8], float gamma) {
  auto raw = [&](int t) { return t < nt ? __ldcs(reinterpret_cast<const unsigned int*>(xp + t * xs)) : 0u; };
  auto emit = [&](int t, float2 v) {
    if (t < nt) st2(op + t * os, sizeof(OT) == 4 ? make_float2(clamp1(v.x), clamp1(v.y)) : v);
  };
  return ema_chunk_exact<PRECISE>(X, lam, first, cm, gamma, raw, emit);
}

template <bool PRECISE, typename OT, bool CONTIG>
__global__ void __launch_bounds__(kNT, PRECISE ? 3 : 4) p3_out_kernel(const Params p, const float* lam_tok) {
  __shared__ float2 lam_s[kH * kL];
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int j0 = lane * 2, ch0 = h * kHD + j0;
  const int c = (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int t0 = c * kL, nt = min(kL, p.S - t0);
  const float gamma = 0.98f - 0.06f * (float)h / (float)kH;
  const size_t n = (size_t)(b * kH + h) * p.nchunks + c;
  const __nv_bfloat16* xp = p.x + (size_t)b * p.xsb + (size_t)t0 * p.xss + ch0;
  OT* op = reinterpret_cast<OT*>(p.out) + (size_t)b * p.osb + (size_t)t0 * p.oss + ch0;
  // A full chunk of contiguous x: its loads go out first, so their latency
  // overlaps the carry, decay and coefficient loads below.
  uint32_t r[kL];
  if (CONTIG && nt == kL) load_chunk(xp, kD, r);

  const bool first = c == 0 && p.starts_seq;
  float2 X;
  if (first) {
    X = p.init ? __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + ch0)) : make_float2(0.f, 0.f);
  } else {
    X = c == 0 ? make_float2(0.f, 0.f) : *reinterpret_cast<const float2*>(p.carry + n * kHD + j0);
    const int blk = c / kBlk;
    if (blk > 0 || p.carry_in) {  // the state entering the chunk's block, decayed to this chunk
      const size_t k = (size_t)(b * kH + h) * p.nblk + blk;
      float2 Y = make_float2(0.f, 0.f);
      float Pb = 1.f;
      if (blk > 0) {
        Y = *reinterpret_cast<const float2*>(p.blk_X + k * kHD + j0);
        Pb = p.blk_P[k];
      }
      if (p.carry_in) {  // the state entering the shard
        const float2 ci = __ldg(reinterpret_cast<const float2*>(p.carry_in + (size_t)b * kD + ch0));
        Y = make_float2(fmaf(Pb, ci.x, Y.x), fmaf(Pb, ci.y, Y.y));
      }
      const float Pn = c == 0 ? 1.f : p.P[n];
      X = make_float2(fmaf(Pn, Y.x, X.x), fmaf(Pn, Y.y, X.y));
    }
  }
  const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  const float lam = lam_token(p, lam_tok, b, t0 + lane, h, lam_base);
  lam_s[h * kL + lane] = make_float2(lam, 1.f - lam);
  float2 cm[8];
  if (PRECISE)
    load_coeffs<true>(p.coeffs, p.Kd, p.K, b, h, j0, gamma, cm);
  else
    load_mono(p, b, h, lane, cm);
  __syncwarp();

  float2 s;
  if (nt < kL)
    s = out_chunk_general<PRECISE, OT>(xp, op, p.xss, p.oss, nt, X, lam_s + h * kL, first, cm, gamma);
  else if (CONTIG)
    s = out_chunk_loaded<PRECISE, OT>(r, xp, op, kD, kD, X, lam_s + h * kL, first, cm, gamma);
  else
    s = out_chunk<PRECISE, OT>(xp, op, p.xss, p.oss, X, lam_s + h * kL, first, cm, gamma);
  // decays are 1 past the end, so the chunk's last state is the sequence's final state
  if (p.fin && t0 + kL >= p.S)
    *reinterpret_cast<float2*>(p.fin + (size_t)b * kD + ch0) = make_float2(clamp1(s.x), clamp1(s.y));
}

// pass 3 of an fp32-output forward from the u the aggregate pass parked in the
// output buffer: no second evaluation (the precise path's tanhf and IEEE
// division are most of its cost).  Each lane reads its 32 u pairs (one
// coalesced 256-byte row per warp and token), runs the EMA from the chunk's
// carry and overwrites them with the outputs: the arithmetic of the
// re-evaluating pass on the same u, so the outputs are bitwise equal.
__global__ void __launch_bounds__(kNT, 4) p3_outu_kernel(const Params p, const float* lam_tok) {
  __shared__ float2 lam_s[kH * kL];
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int j0 = lane * 2, ch0 = h * kHD + j0;
  const int c = (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int t0 = c * kL, nt = min(kL, p.S - t0);
  const size_t n = (size_t)(b * kH + h) * p.nchunks + c;
  float* op = static_cast<float*>(p.out) + (size_t)b * p.osb + (size_t)t0 * p.oss + ch0;
  // the parked u of the first 16 tokens go out first: their latency overlaps
  // the carry and decay loads (16 at a time keeps the fp32 case in registers)
  constexpr int kHalf = kL / 2;
  float2 u[kHalf];
  auto load_u = [&](int t0h) {
#pragma unroll
    for (int q = 0; q < kHalf; ++q) {
      const int t = t0h + q;
      u[q] = t < nt ? *reinterpret_cast<const float2*>(op + (size_t)t * p.oss) : make_float2(0.f, 0.f);
    }
  };
  load_u(0);
  const bool first = c == 0 && p.starts_seq;
  float2 X;
  if (first) {
    X = p.init ? __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + ch0)) : make_float2(0.f, 0.f);
  } else {
    X = c == 0 ? make_float2(0.f, 0.f) : *reinterpret_cast<const float2*>(p.carry + n * kHD + j0);
    const int blk = c / kBlk;
    if (blk > 0 || p.carry_in) {  // the state entering the chunk's block, decayed to this chunk
      const size_t k = (size_t)(b * kH + h) * p.nblk + blk;
      float2 Y = make_float2(0.f, 0.f);
      float Pb = 1.f;
      if (blk > 0) {
        Y = *reinterpret_cast<const float2*>(p.blk_X + k * kHD + j0);
        Pb = p.blk_P[k];
      }
      if (p.carry_in) {  // the state entering the shard
        const float2 ci = __ldg(reinterpret_cast<const float2*>(p.carry_in + (size_t)b * kD + ch0));
        Y = make_float2(fmaf(Pb, ci.x, Y.x), fmaf(Pb, ci.y, Y.y));
      }
      const float Pn = c == 0 ? 1.f : p.P[n];
      X = make_float2(fmaf(Pn, Y.x, X.x), fmaf(Pn, Y.y, X.y));
    }
  }
  const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  const float lam = lam_token(p, lam_tok, b, t0 + lane, h, lam_base);
  lam_s[h * kL + lane] = make_float2(lam, 1.f - lam);
  __syncwarp();
  const float2* lm = lam_s + h * kL;
  float2 s = X;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    if (hf == 1) load_u(kHalf);
#pragma unroll
    for (int q = 0; q < kHalf; ++q) {
      const int t = hf * kHalf + q;
      if (t < nt) {
        s = ema_step(s, lm[t], u[q], t == 0 && first);
        st2(op + (size_t)t * p.oss, make_float2(clamp1(s.x), clamp1(s.y)));
      }
    }
  }
  // decays are 1 past the end, so the chunk's last state is the sequence's final state
  if (p.fin && t0 + kL >= p.S)
    *reinterpret_cast<float2*>(p.fin + (size_t)b * kD + ch0) = make_float2(clamp1(s.x), clamp1(s.y));
}

// pass 3 of a bf16-output forward from the u the aggregate pass parked as fp16
// pairs in the ring (kURing): no second evaluation and no second read of x.
// Each lane loads its 32 u words first (one 128-byte line per warp and
// token, still in L2), then the chunk's entry state (its span's entry state
// carried through the span, both formed by the aggregate pass) and decays,
// runs the EMA and writes the outputs; then each lane drops one of the
// warp's lines from L2, so the parked u never goes to HBM.  The final state
// is the chunk's aggregate applied to its entry state in fp32 (A X + agg),
// so it does not carry the fp16 rounding of u.
__global__ void __launch_bounds__(kNT, 4) p3_outp_kernel(const Params p, const float* lam_tok) {
  __shared__ float2 lam_s[kH * kL];
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int j0 = lane * 2, ch0 = h * kHD + j0;
  const int c = (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int t0 = c * kL, nt = min(kL, p.S - t0);
  const size_t n = (size_t)(b * kH + h) * p.nchunks + c;
  const uint32_t* up = p.park + ((size_t)(b * p.nchunks + c) * kH + h) * (kL * 32);
  uint32_t r[kL];
#pragma unroll
  for (int t = 0; t < kL; ++t) r[t] = __ldcg(up + t * 32 + lane);
  const bool first = c == 0 && p.starts_seq;
  float2 X;  // the state entering the chunk: from its span's entry state and the in-span carry
  if (first) {
    X = p.init ? __ldg(reinterpret_cast<const float2*>(p.init + (size_t)b * kD + ch0)) : make_float2(0.f, 0.f);
  } else {
    const float2 Xs = *reinterpret_cast<const float2*>(p.spX + ((size_t)(b * kH + h) * p.nsp + c / kSpanC) * kHD + j0);
    const float2 Cl = *reinterpret_cast<const float2*>(p.carry + n * kHD + j0);
    const float Pl = p.P[n];
    X = make_float2(fmaf(Pl, Xs.x, Cl.x), fmaf(Pl, Xs.y, Cl.y));
  }
  const float lam_base = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  const float lam = lam_token(p, lam_tok, b, t0 + lane, h, lam_base);
  lam_s[h * kL + lane] = make_float2(lam, 1.f - lam);
  __syncwarp();
  const float2* lm = lam_s + h * kL;
  __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)b * p.osb + (size_t)t0 * kD + ch0;
  float2 s = X;
  if (nt == kL) {
#pragma unroll
    for (int t = 0; t < kL; ++t) {
      s = ema_step(s, lm[t], unpack_f16x2(r[t]), t == 0 && first);
      st2(op + t * kD, s);
    }
  } else {
#pragma unroll
    for (int t = 0; t < kL; ++t) {
      s = ema_step(s, lm[t], unpack_f16x2(r[t]), t == 0 && first);
      if (t < nt) st2(op + t * kD, s);
    }
  }
  __syncwarp();  // every lane holds its words of all 32 lines
  discard_l2(up + lane * 32);
  if (p.fin && t0 + kL >= p.S) {  // decays are 1 past the end, so A X + agg is the sequence's final state
    const float An = p.A[n];
    const float2 E = *reinterpret_cast<const float2*>(p.agg + n * kHD + j0);
    *reinterpret_cast<float2*>(p.fin + (size_t)b * kD + ch0) =
        make_float2(clamp1(fmaf(An, X.x, E.x)), clamp1(fmaf(An, X.y, E.y)));
  }
}

template <bool GATE, bool PRECISE, int UM>
cudaError_t launch_agg(const CUtensorMap& mx, const Params& p, cudaStream_t st) {
  auto kern = p3_agg_kernel<GATE, PRECISE, UM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAggSmem);
  if (e != cudaSuccess) return e;
  kern<<<p.B * p.nchunks, kNT, kAggSmem, st>>>(mx, p);
  return cudaGetLastError();
}

template <bool PRECISE, typename OT>
cudaError_t launch_out(const Params& p, const float* lam_tok, cudaStream_t st) {
  const bool contig = p.xss == kD && p.oss == kD;  // token strides of x and out
  if (contig)
    p3_out_kernel<PRECISE, OT, true><<<p.B * p.nchunks, kNT, 0, st>>>(p, lam_tok);
  else
    p3_out_kernel<PRECISE, OT, false><<<p.B * p.nchunks, kNT, 0, st>>>(p, lam_tok);
  return cudaGetLastError();
}

}  // namespace p3
}  // namespace ossm

using namespace ossm;

// Workspace of the three-pass path: header, chunk decay products, prefix
// products, aggregates and carries, the same four per carry block, and
// (gated) the per-token decays.
namespace {

size_t p3_al(size_t v) { return (v + 255) & ~(size_t)255; }

size_t p3_single_bytes(const ossm_fwd_args* a) {
  const size_t nch = (size_t)(a->S + p3::kL - 1) / p3::kL;
  const size_t N = (size_t)a->B * p3::kH * nch;
  const size_t NB = (size_t)a->B * p3::kH * ((nch + p3::kBlk - 1) / p3::kBlk);
  size_t bytes = p3_al(sizeof(WsHeader)) + 2 * p3_al(N * 4) + 2 * p3_al(N * p3::kHD * 4) + 2 * p3_al(NB * 4) +
                 2 * p3_al(NB * p3::kHD * 4);
  bytes += p3_al((size_t)a->B * p3::kH * 4 * 32 * 16) + p3_al((size_t)p3::kH * 4 * 32 * 16);  // cmono, wfrag
  bytes += p3_al((size_t)a->B * p3::kD * 4);  // the state entering a shard (sequence-sharded calls)
  if (a->gate_w && !a->lam_tok) bytes += p3_al((size_t)a->B * a->S * p3::kH * 4);
  return bytes;
}

// A batch runs as kGroups groups of whole sequences on kStreams streams when
// every group still fills the GPU for about two waves of the streaming
// kernels (ossm_p3_launch), else as one launch.
constexpr int kGroups = 2, kStreams = 5;
int p3_groups(const ossm_fwd_args* a) {
  if (a->flags & OSSM_F_ONE_STREAM) return 1;
  const long long nch = (a->S + p3::kL - 1) / p3::kL;
  return (a->B >= kGroups && (long long)(a->B / kGroups) * nch >= 1024) ? kGroups : 1;
}

// Sequences [b0, b1) of a batch: the same arguments, pointers moved to row b0.
ossm_fwd_args p3_rows(const ossm_fwd_args* a, int b0, int b1) {
  ossm_fwd_args h = *a;
  const size_t D = (size_t)a->H * a->head_dim;
  const size_t oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  h.B = b1 - b0;
  h.x = static_cast<const char*>(a->x) + (size_t)b0 * a->x_stride_b * 2;  // bf16 (the path's only input type)
  h.out = static_cast<char*>(a->out) + (size_t)b0 * a->out_stride_b * oel;
  h.coeffs = a->coeffs + (size_t)b0 * a->H * a->degree * a->head_dim;
  if (a->init_state) h.init_state = a->init_state + (size_t)b0 * D;
  if (a->final_state) h.final_state = a->final_state + (size_t)b0 * D;
  if (a->lam_tok) h.lam_tok = a->lam_tok + (size_t)b0 * a->S * a->H;
  return h;
}

// One long sequence (B = 1, at least 4096 chunks) runs as two consecutive
// token ranges on two streams (ossm_p3_launch).
bool p3_seq_split(const ossm_fwd_args* a) {
  if (a->flags & OSSM_F_ONE_STREAM) return false;
  const long long nch = (a->S + p3::kL - 1) / p3::kL;
  return a->B == 1 && nch >= 4096;
}
int p3_seq_cut(const ossm_fwd_args* a) { return ((a->S + p3::kL - 1) / p3::kL / 2) * p3::kL; }

// Tokens [s0, s1) of a one-sequence batch: the initial state belongs to the
// range that starts the sequence, the final state to the one that ends it.
ossm_fwd_args p3_tokens(const ossm_fwd_args* a, int s0, int s1) {
  ossm_fwd_args h = *a;
  const size_t oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  h.S = s1 - s0;
  h.x = static_cast<const char*>(a->x) + (size_t)s0 * a->x_stride_s * 2;  // bf16
  h.out = static_cast<char*>(a->out) + (size_t)s0 * a->out_stride_s * oel;
  if (a->lam_tok) h.lam_tok = a->lam_tok + (size_t)s0 * a->H;
  if (s0 > 0) h.init_state = nullptr;
  if (s1 < a->S) h.final_state = nullptr;
  return h;
}

// bf16 outputs with u parked in L2 (kURing): the batch runs as slabs of whole
// sequences, slab k on stream k % kParkStreams, two launches each (the
// aggregate pass, which also forms the carries, and the output pass).  Each
// stream has its own workspace region and ring slot, which its next slab
// reuses once its output pass is done (a stream's launches run in order), so
// at most kParkStreams slabs of parked u are live: with slabs of about 16 MB,
// 84 MB of the 126 MB L2, held there by an evict-last policy while x (loaded
// evict-first) and the outputs stream past, and dropped by the output pass
// without a write-back.  Measured at config 2 (gated step under graph
// replay): 2 streams 144 us, 3 125, 4 115, 5 109, 6 114, 8 114, against
// 120.6 us for the re-evaluating path.
constexpr size_t kParkSeqMax = 24u << 20;  // a sequence's parked u must fit this
constexpr size_t kParkSlab = 16u << 20;    // target parked u per slab
constexpr int kParkStreams = 5;            // streams, ring slots and workspace regions
static_assert(kParkStreams <= kStreams, "park streams");
size_t p3_park_seq_bytes(const ossm_fwd_args* a) {
  return (size_t)((a->S + p3::kL - 1) / p3::kL) * p3::kL * p3::kD * 2;
}
int p3_park_nsp(const ossm_fwd_args* a) {
  const int nch = (a->S + p3::kL - 1) / p3::kL;
  return (nch + p3::kSpanC - 1) / p3::kSpanC;
}
// Sequences per slab, or 0 when this mode does not apply: the bf16 fast
// path with outputs contiguous along tokens, and sequences whose parked u
// fits.  Not under OSSM_F_ONE_STREAM (the no-allocation entry point's fixed
// scratch has no room for the ring).
int p3_park_slab(const ossm_fwd_args* a) {
  if (a->flags & (OSSM_F_ONE_STREAM | OSSM_F_PRECISE)) return 0;
  if (a->out_dtype != OSSM_BF16 || a->out_stride_s != p3::kD) return 0;
  const size_t seq = p3_park_seq_bytes(a);
  if (seq > kParkSeqMax) return 0;
  return (int)std::max<size_t>(1, std::min<size_t>((size_t)a->B, kParkSlab / seq));
}
int p3_park_nstreams(const ossm_fwd_args* a, int sb) { return std::min((a->B + sb - 1) / sb, kParkStreams); }
// Front: header, every sequence's coefficients, the gate fragments, and the tickets of every stream's region (cleared by the setup
// kernel).
size_t p3_park_ticket_words(const ossm_fwd_args* a, int sb) { return (size_t)sb * (p3_park_nsp(a) + 1); }
size_t p3_park_front_bytes(const ossm_fwd_args* a, int sb) {
  return p3_al(sizeof(WsHeader)) + p3_al((size_t)a->B * p3::kH * 4 * 32 * 16) + p3_al((size_t)p3::kH * 4 * 32 * 16) +
         p3_al((size_t)p3_park_nstreams(a, sb) * p3_park_ticket_words(a, sb) * 4);
}
// One stream's region: the slab's three-pass workspace, its ring slot, and
// the span records (spA, spE, spX).
size_t p3_park_stream_bytes(const ossm_fwd_args* a, int sb) {
  const ossm_fwd_args h = p3_rows(a, 0, sb);
  const size_t nsp = (size_t)sb * p3::kH * p3_park_nsp(a);
  return p3_al(p3_single_bytes(&h)) + p3_al((size_t)sb * p3_park_seq_bytes(a)) + p3_al(nsp * 4) +
         2 * p3_al(nsp * p3::kHD * 4);
}
size_t p3_park_bytes(const ossm_fwd_args* a, int sb) {
  return p3_park_front_bytes(a, sb) + (size_t)p3_park_nstreams(a, sb) * p3_park_stream_bytes(a, sb);
}

}  // namespace

size_t ossm_p3_workspace_bytes(const ossm_fwd_args* a) {
  size_t bytes = p3_single_bytes(a);
  if (const int sb = p3_park_slab(a)) bytes = std::max(bytes, p3_park_bytes(a, sb));
  const int G = p3_groups(a);
  if (G > 1) {
    size_t sum = 0;
    for (int g = 0; g < G; ++g) {
      const ossm_fwd_args h = p3_rows(a, a->B * g / G, a->B * (g + 1) / G);
      sum += p3_al(p3_single_bytes(&h));
    }
    bytes = std::max(bytes, sum);
  }
  if (p3_seq_split(a)) {  // both ranges, then the first range's totals
    const int cut = p3_seq_cut(a);
    const ossm_fwd_args h0 = p3_tokens(a, 0, cut), h1 = p3_tokens(a, cut, a->S);
    bytes = std::max(bytes, p3_al(p3_single_bytes(&h0)) + p3_al(p3_single_bytes(&h1)) +
                                p3_al((size_t)a->B * p3::kH * 4) + p3_al((size_t)a->B * p3::kD * 4));
  }
  return bytes;
}

namespace {

int p3_params(const ossm_fwd_args* a, char* ws, p3::Params& p) {
  using namespace p3;
  p.B = a->B;
  p.S = a->S;
  p.K = (a->flags & OSSM_EVAL_MASK) == OSSM_EVAL_CLENSHAW_DEG4 ? (a->degree < 4 ? a->degree : 4) : a->degree;
  p.Kd = a->degree;
  p.nchunks = (a->S + kL - 1) / kL;
  p.x = reinterpret_cast<const __nv_bfloat16*>(a->x);
  p.xsb = a->x_stride_b;
  p.xss = a->x_stride_s;
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
  p.out = a->out;
  p.osb = a->out_stride_b;
  p.oss = a->out_stride_s;
  const bool gate = a->gate_w && !a->lam_tok;
  const size_t N = (size_t)a->B * kH * p.nchunks;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  p.ws = reinterpret_cast<WsHeader*>(ws);
  size_t off = al(sizeof(WsHeader));
  p.A = reinterpret_cast<float*>(ws + off);
  off += al(N * 4);
  p.P = reinterpret_cast<float*>(ws + off);
  off += al(N * 4);
  p.agg = reinterpret_cast<float*>(ws + off);
  off += al(N * kHD * 4);
  p.carry = reinterpret_cast<float*>(ws + off);
  off += al(N * kHD * 4);
  p.nblk = (p.nchunks + kBlk - 1) / kBlk;
  const size_t NB = (size_t)a->B * kH * p.nblk;
  p.blk_A = reinterpret_cast<float*>(ws + off);
  off += al(NB * 4);
  p.blk_P = reinterpret_cast<float*>(ws + off);
  off += al(NB * 4);
  p.blk_E = reinterpret_cast<float*>(ws + off);
  off += al(NB * kHD * 4);
  p.blk_X = reinterpret_cast<float*>(ws + off);
  off += al(NB * kHD * 4);
  p.cmono = reinterpret_cast<float4*>(ws + off);
  off += al((size_t)a->B * kH * 4 * 32 * 16);
  p.wfrag = reinterpret_cast<uint4*>(ws + off);
  off += al((size_t)kH * 4 * 32 * 16);
  p.shard_carry = reinterpret_cast<float*>(ws + off);
  off += al((size_t)a->B * kD * 4);
  p.lam_ws = gate ? reinterpret_cast<float*>(ws + off) : nullptr;
  p.starts_seq = 1;
  p.tot_A = nullptr;
  p.tot_E = nullptr;
  p.carry_in = nullptr;
  p.uc = 0;
  p.park = nullptr;
  p.nsp = 0;
  p.tk_span = p.tk_seq = nullptr;
  p.spA = p.spE = p.spX = nullptr;
  p.zero_ptr = nullptr;
  p.zero_n = 0;
  if ((long long)a->B * p.nchunks > 0x7fffffffLL || (long long)a->B * kH * p.nblk > 0x7fffffffLL) return OSSM_EINVAL;
  return OSSM_OK;
}

// Whether the aggregate pass parks u in the output buffer for the output pass:
// fp32 outputs only (u fits the output row exactly), whole-forward launches
// only (the sharded entry points may be handed another output buffer for
// their second call), not when x and out overlap in memory (the parked u
// would overwrite x another chunk still reads), and while the outputs fit in
// half of L2, so the parked u is read back from L2.  Measured: the TTT step
// of BASELINE.json configs[3] (16 forwards of 4 x 2048 tokens with fp32
// states) went from 1.50 to 1.38 ms.  (bf16 outputs park u as fp16 in a
// ring instead, slab by slab, so it stays in L2: the parked path below.
// Parked in the rows of a whole batch of bf16 outputs, it made the config-2
// step slower, 122.8 -> 135.7 us: its 134 MB left L2 before the output pass
// read them.)
int p3_uc_mode(const ossm_fwd_args* a) {
  if (a->out_dtype != OSSM_F32) return 0;
  const size_t D = (size_t)a->H * a->head_dim;
  const char* x0 = static_cast<const char*>(a->x);
  const char* x1 = x0 + ((size_t)(a->B - 1) * a->x_stride_b + (size_t)(a->S - 1) * a->x_stride_s + D) * 2;
  const char* o0 = static_cast<const char*>(a->out);
  const char* o1 = o0 + ((size_t)(a->B - 1) * a->out_stride_b + (size_t)(a->S - 1) * a->out_stride_s + D) * 4;
  if (o0 < x1 && x0 < o1) return 0;
  return (size_t)a->B * a->S * D * 4 <= (64u << 20) ? 1 : 0;
}

// pass 1: aggregates (with the per-launch setup unless the caller ran it)
int p3_aggregates(const ossm_fwd_args* a, const p3::Params& p, cudaStream_t st, bool prep = true) {
  using namespace p3;
  CUtensorMap mx;
  if (!fast::encode_map(&mx, a->x, a->S, a->B, a->x_stride_s, a->x_stride_b, kL)) return OSSM_EINVAL;
  const bool gate = a->gate_w && !a->lam_tok;
  const bool precise = (a->out_dtype == OSSM_F32) || (a->flags & OSSM_F_PRECISE);
  const int nprep = (precise ? 0 : a->B * kH) + (gate ? kH : 0);
  if (prep && nprep > 0) {
    if (precise)
      p3_prep_kernel<false, true><<<nprep, 32, 0, st>>>(p);
    else if (gate)
      p3_prep_kernel<true, true><<<nprep, 32, 0, st>>>(p);
    else
      p3_prep_kernel<true, false><<<nprep, 32, 0, st>>>(p);
  }
  cudaError_t e;
  if (p.uc)
    e = gate ? launch_agg<true, true, kURows>(mx, p, st) : launch_agg<false, true, kURows>(mx, p, st);
  else if (p.park)  // the bf16 fast path only
    e = gate ? launch_agg<true, false, kURing>(mx, p, st) : launch_agg<false, false, kURing>(mx, p, st);
  else if (precise)
    e = gate ? launch_agg<true, true, kUNone>(mx, p, st) : launch_agg<false, true, kUNone>(mx, p, st);
  else
    e = gate ? launch_agg<true, false, kUNone>(mx, p, st) : launch_agg<false, false, kUNone>(mx, p, st);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

// pass 2: carries (and the shard totals when asked)
int p3_carries(const ossm_fwd_args* a, const p3::Params& p, cudaStream_t st) {
  using namespace p3;
  p3_carry_kernel<<<a->B * kH * p.nblk, kSpans * 32, 0, st>>>(p);
  if (p.nblk > 1) p3_blockfold_kernel<<<a->B * kH, 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

// passes 1 and 2
int p3_front(const ossm_fwd_args* a, const p3::Params& p, cudaStream_t st) {
  const int r = p3_aggregates(a, p, st);
  return r != OSSM_OK ? r : p3_carries(a, p, st);
}

// pass 3: outputs
int p3_back(const ossm_fwd_args* a, const p3::Params& p, cudaStream_t st) {
  using namespace p3;
  const bool gate = a->gate_w && !a->lam_tok;
  const bool precise = (a->out_dtype == OSSM_F32) || (a->flags & OSSM_F_PRECISE);
  const float* lam_tok = gate ? p.lam_ws : a->lam_tok;
  cudaError_t e;
  if (p.uc) {
    p3_outu_kernel<<<p.B * p.nchunks, kNT, 0, st>>>(p, lam_tok);
    e = cudaGetLastError();
  } else if (p.park) {
    p3_outp_kernel<<<p.B * p.nchunks, kNT, 0, st>>>(p, lam_tok);
    e = cudaGetLastError();
  } else if (a->out_dtype == OSSM_F32)
    e = launch_out<true, float>(p, lam_tok, st);
  else
    e = precise ? launch_out<true, __nv_bfloat16>(p, lam_tok, st) : launch_out<false, __nv_bfloat16>(p, lam_tok, st);
  return e == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

// The side streams of a split launch and their events, one set per device,
// created by the first split launch on the device (make that call before any
// stream capture); a mutex keeps each launch's enqueue in one piece.
struct P3Side {
  std::mutex mu;
  bool ready = false;
  cudaStream_t s[kStreams] = {};
  cudaEvent_t fork = nullptr, join[kStreams] = {}, tot = nullptr;
};
P3Side g_p3side[64];

// The device's side streams and events, created on first use (caller holds mu).
bool p3_side_ready(P3Side& sd) {
  if (sd.ready) return true;
  for (int k = 1; k < kStreams; ++k)
    if (cudaStreamCreateWithFlags(&sd.s[k], cudaStreamNonBlocking) != cudaSuccess) return false;
  if (cudaEventCreateWithFlags(&sd.fork, cudaEventDisableTiming) != cudaSuccess) return false;
  if (cudaEventCreateWithFlags(&sd.tot, cudaEventDisableTiming) != cudaSuccess) return false;
  for (int k = 1; k < kStreams; ++k)
    if (cudaEventCreateWithFlags(&sd.join[k], cudaEventDisableTiming) != cudaSuccess) return false;
  sd.ready = true;
  return true;
}

// Groups of whole sequences, group g on stream g % kStreams (stream 0 is the
// caller's), all forked at once.  The block scheduler dispatches the first
// group's aggregate CTAs first, so its aggregates finish while the others'
// still run, and the carry pass of each group (a few dozen CTAs that would
// leave most SMs idle between the streaming passes) overlaps other groups'
// streaming work.  The groups use disjoint parts of one workspace and report
// to its header.  Every result is bitwise the one-launch result.
int p3_launch_split(const ossm_fwd_args* a, int G, char* ws, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OSSM_ELAUNCH;
  P3Side& sd = g_p3side[dev];
  std::lock_guard<std::mutex> lock(sd.mu);
  if (!p3_side_ready(sd)) return OSSM_ELAUNCH;
  cudaStream_t streams[kStreams];
  streams[0] = st;
  for (int k = 1; k < kStreams; ++k) streams[k] = sd.s[k];
  const int ns = std::min(G, kStreams);
  bool ok = cudaEventRecord(sd.fork, st) == cudaSuccess;
  for (int k = 1; k < ns; ++k) ok = ok && cudaStreamWaitEvent(sd.s[k], sd.fork, 0) == cudaSuccess;
  int r = ok ? OSSM_OK : OSSM_ELAUNCH;
  WsHeader* header = reinterpret_cast<WsHeader*>(ws);
  size_t off = 0;
  for (int g = 0; g < G && r == OSSM_OK; ++g) {
    const ossm_fwd_args h = p3_rows(a, a->B * g / G, a->B * (g + 1) / G);
    p3::Params p;
    r = p3_params(&h, ws + off, p);
    off += p3_al(p3_single_bytes(&h));
    if (r != OSSM_OK) break;
    p.ws = header;  // one header: the sticky status lives at the workspace start
    p.uc = p3_uc_mode(&h);
    r = p3_front(&h, p, streams[g % ns]);
    if (r == OSSM_OK) r = p3_back(&h, p, streams[g % ns]);
  }
  // join, also after an error, so the caller's later work never overlaps
  bool joined = true;
  for (int k = 1; k < ns; ++k)
    joined = joined && cudaEventRecord(sd.join[k], sd.s[k]) == cudaSuccess &&
             cudaStreamWaitEvent(st, sd.join[k], 0) == cudaSuccess;
  if (r != OSSM_OK) return r;
  return joined ? OSSM_OK : OSSM_ELAUNCH;
}

// One long sequence as two token ranges, range 0 on the caller's stream and
// range 1 on the side stream, forked at once.  Each range's aggregates and
// carries need nothing from the other, so the carry pass of each overlaps
// the other's streaming kernels.  Range 0 also writes its totals (the state
// at its end), and range 1's output pass waits for them and adds them as the
// state entering it, exactly as a sequence-sharded launch on two ranks does.
// The carries compose in another order than in one launch, so results match
// the one-launch results to fp32 rounding of the carries, not bitwise.
int p3_launch_seq_split(const ossm_fwd_args* a, char* ws, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OSSM_ELAUNCH;
  P3Side& sd = g_p3side[dev];
  std::lock_guard<std::mutex> lock(sd.mu);
  if (!p3_side_ready(sd)) return OSSM_ELAUNCH;
  const int cut = p3_seq_cut(a);
  const ossm_fwd_args h0 = p3_tokens(a, 0, cut), h1 = p3_tokens(a, cut, a->S);
  const size_t off1 = p3_al(p3_single_bytes(&h0)), off_tot = off1 + p3_al(p3_single_bytes(&h1));
  float* tot_A = reinterpret_cast<float*>(ws + off_tot);
  float* tot_E = reinterpret_cast<float*>(ws + off_tot + p3_al((size_t)a->B * p3::kH * 4));
  p3::Params p0, p1;
  int r = p3_params(&h0, ws, p0);
  if (r == OSSM_OK) r = p3_params(&h1, ws + off1, p1);
  if (r != OSSM_OK) return r;
  p0.tot_A = tot_A;
  p0.tot_E = tot_E;
  p1.ws = p0.ws;  // one header: the sticky status lives at the workspace start
  p1.starts_seq = 0;
  p1.carry_in = tot_E;
  p0.uc = p3_uc_mode(&h0);
  p1.uc = p3_uc_mode(&h1);
  cudaStream_t side = sd.s[1];
  bool ok = cudaEventRecord(sd.fork, st) == cudaSuccess && cudaStreamWaitEvent(side, sd.fork, 0) == cudaSuccess;
  r = ok ? p3_front(&h0, p0, st) : OSSM_ELAUNCH;
  ok = r == OSSM_OK && cudaEventRecord(sd.tot, st) == cudaSuccess;
  if (ok) r = p3_back(&h0, p0, st);
  if (ok && r == OSSM_OK) r = p3_front(&h1, p1, side);
  if (ok && r == OSSM_OK) ok = cudaStreamWaitEvent(side, sd.tot, 0) == cudaSuccess;
  if (ok && r == OSSM_OK) r = p3_back(&h1, p1, side);
  // join, also after an error, so the caller's later work never overlaps
  const bool joined = cudaEventRecord(sd.join[1], side) == cudaSuccess && cudaStreamWaitEvent(st, sd.join[1], 0) == cudaSuccess;
  if (r != OSSM_OK) return r;
  return ok && joined ? OSSM_OK : OSSM_ELAUNCH;
}

// The parked-u forward (kURing): the per-launch setup once for the whole
// batch on the caller's stream (also clearing the tickets), then the slabs,
// forked onto the streams.  One slab runs on the caller's stream alone.
int p3_launch_park(const ossm_fwd_args* a, int sb, char* ws, cudaStream_t st) {
  using namespace p3;
  const int nslab = (a->B + sb - 1) / sb;
  const int ns = p3_park_nstreams(a, sb);
  P3Side* sd = nullptr;
  std::unique_lock<std::mutex> lock;
  if (ns > 1) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OSSM_ELAUNCH;
    sd = &g_p3side[dev];
    lock = std::unique_lock<std::mutex>(sd->mu);
    if (!p3_side_ready(*sd)) return OSSM_ELAUNCH;
  }
  const int nsp = p3_park_nsp(a);
  size_t off = p3_al(sizeof(WsHeader));
  WsHeader* header = reinterpret_cast<WsHeader*>(ws);
  float4* cmono = reinterpret_cast<float4*>(ws + off);
  off += p3_al((size_t)a->B * kH * 4 * 32 * 16);
  uint4* wfrag = reinterpret_cast<uint4*>(ws + off);
  off += p3_al((size_t)kH * 4 * 32 * 16);
  uint32_t* tickets = reinterpret_cast<uint32_t*>(ws + off);
  const size_t tw = p3_park_ticket_words(a, sb);
  const ossm_fwd_args h0 = p3_rows(a, 0, sb);
  const size_t front = p3_park_front_bytes(a, sb), per = p3_park_stream_bytes(a, sb);
  const size_t ring_off = p3_al(p3_single_bytes(&h0));
  const size_t spa_off = ring_off + p3_al((size_t)sb * p3_park_seq_bytes(a));
  const size_t nspw = (size_t)sb * kH * nsp;
  const bool gate = a->gate_w && !a->lam_tok;
  {  // the setup of every slab at once
    Params pp;
    int r = p3_params(&h0, ws + front, pp);
    if (r != OSSM_OK) return r;
    pp.B = a->B;
    pp.coeffs = a->coeffs;
    pp.cmono = cmono;
    pp.wfrag = wfrag;
    pp.zero_ptr = tickets;
    pp.zero_n = (int)(ns * tw);
    const int nprep = a->B * kH + (gate ? kH : 0);
    if (gate)
      p3_prep_kernel<true, true><<<nprep, 32, 0, st>>>(pp);
    else
      p3_prep_kernel<true, false><<<nprep, 32, 0, st>>>(pp);
    if (cudaGetLastError() != cudaSuccess) return OSSM_ELAUNCH;
  }
  cudaStream_t streams[kStreams];
  streams[0] = st;
  bool ok = true;
  if (sd) {
    for (int k = 1; k < ns; ++k) streams[k] = sd->s[k];
    ok = cudaEventRecord(sd->fork, st) == cudaSuccess;
    for (int k = 1; k < ns; ++k) ok = ok && cudaStreamWaitEvent(sd->s[k], sd->fork, 0) == cudaSuccess;
  }
  int r = ok ? OSSM_OK : OSSM_ELAUNCH;
  for (int k = 0; k < nslab && r == OSSM_OK; ++k) {
    const int b0 = k * sb, b1 = std::min(a->B, b0 + sb), si = k % ns;
    const ossm_fwd_args h = p3_rows(a, b0, b1);
    char* region = ws + front + (size_t)si * per;
    Params p;
    r = p3_params(&h, region, p);
    if (r != OSSM_OK) break;
    p.ws = header;  // one header: the sticky status lives at the workspace start
    p.cmono = cmono + (size_t)b0 * kH * 4 * 32;
    p.wfrag = wfrag;
    p.park = reinterpret_cast<uint32_t*>(region + ring_off);
    p.nsp = nsp;
    p.tk_span = tickets + (size_t)si * tw;
    p.tk_seq = p.tk_span + (size_t)sb * nsp;
    p.spA = reinterpret_cast<float*>(region + spa_off);
    p.spE = reinterpret_cast<float*>(region + spa_off + p3_al(nspw * 4));
    p.spX = reinterpret_cast<float*>(region + spa_off + p3_al(nspw * 4) + p3_al(nspw * kHD * 4));
    r = p3_aggregates(&h, p, streams[si], false);
    if (r == OSSM_OK) r = p3_back(&h, p, streams[si]);
  }
  // join, also after an error, so the caller's later work never overlaps
  bool joined = true;
  if (sd)
    for (int k = 1; k < ns; ++k)
      joined = joined && cudaEventRecord(sd->join[k], sd->s[k]) == cudaSuccess &&
               cudaStreamWaitEvent(st, sd->join[k], 0) == cudaSuccess;
  if (r != OSSM_OK) return r;
  return ok && joined ? OSSM_OK : OSSM_ELAUNCH;
}

}  // namespace

// Sequences per slab of the parked path for these (fast-path) arguments, or 0.
int ossm_p3_parked(const ossm_fwd_args* a) { return p3_park_slab(a); }

int ossm_p3_launch(const ossm_fwd_args* a, char* ws, cudaStream_t st) {
  if (const int sb = p3_park_slab(a)) return p3_launch_park(a, sb, ws, st);
  const int G = p3_groups(a);
  if (G > 1) return p3_launch_split(a, G, ws, st);
  if (p3_seq_split(a)) return p3_launch_seq_split(a, ws, st);
  p3::Params p;
  int r = p3_params(a, ws, p);
  if (r != OSSM_OK) return r;
  p.uc = p3_uc_mode(a);
  if ((r = p3_front(a, p, st)) != OSSM_OK) return r;
  return p3_back(a, p, st);
}

int ossm_p3_shard_front(const ossm_fwd_args* a, int starts_sequence, char* ws, float* shard_decay, float* shard_state,
                        cudaStream_t st) {
  p3::Params p;
  int r = p3_params(a, ws, p);
  if (r != OSSM_OK) return r;
  p.starts_seq = starts_sequence ? 1 : 0;
  p.tot_A = shard_decay;
  p.tot_E = shard_state;
  return p3_front(a, p, st);
}

int ossm_p3_shard_fold(int B, int H, int hd, int nshards, const float* totals, const float* init, float* state_out,
                       cudaStream_t st) {
  const int n = B * H * hd;
  p3::shard_fold_kernel<<<(n + 255) / 256, 256, 0, st>>>(B, H, hd, nshards, totals, init, state_out);
  return cudaGetLastError() == cudaSuccess ? OSSM_OK : OSSM_ELAUNCH;
}

int ossm_p3_shard_back(const ossm_fwd_args* a, int shard, const float* totals, const float* seq_init, char* ws,
                       cudaStream_t st) {
  p3::Params p;
  int r = p3_params(a, ws, p);
  if (r != OSSM_OK) return r;
  p.starts_seq = shard == 0 ? 1 : 0;
  p.carry_in = nullptr;
  if (shard > 0) {  // the state entering this shard, folded on the device into the workspace
    r = ossm_p3_shard_fold(a->B, p3::kH, p3::kHD, shard, totals, seq_init, p.shard_carry, st);
    if (r != OSSM_OK) return r;
    p.carry_in = p.shard_carry;
  }
  return p3_back(a, p, st);
}
