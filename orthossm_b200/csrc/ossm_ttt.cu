// BASELINE-mode test-time training over a whole sequence in one call
// (no counterpart kernel in the reference, whose
// TTT is the local gated-error Lion step, sdpc_kernel.py:2126-2287).
//
// Per chunk of L tokens the loss is mean_{t<L-1,d} (W_pred s_t - x_{t+1})^2
// per sequence, whose gradient with respect to the states is
//
//   gs_t = (2/N) W_pred^T (W_pred s_t - x_{t+1}) = (2/N) (G s_t - W_pred^T x_{t+1}),
//   G = W_pred^T W_pred,  N = (L-1) D.
//
// The second form needs one GEMM per chunk instead of two chained ones, so one
// tensor-core kernel forms gs with both products in a single TMEM accumulator:
//   wpred_grad_kernel  CTA per (256 output channels, 128 tokens, sequence):
//     warp 0 issues TMA loads of [128 x 128 B] token tiles and [256 x 128 B]
//     weight tiles (128-byte swizzle) into a 4-stage ring; warp 1 issues
//     tcgen05.mma into a 128 x 256 fp32 accumulator in TMEM:
//       s . G                  kind::tf32 (s fp32, as cuBLAS's TF32 mode)
//       x_{t+1} . (-W_pred)    kind::f16, W_pred split into bf16 hi + lo
//                              (bf16 x is exact in bf16; fp32 x takes one
//                              kind::tf32 product instead);
//     warps 2-5 read the accumulator back (tcgen05.ld), scale by 2/N and
//     stage the tile in shared memory, from where TMA stores gs (t < L-1)
//     and the same warps form the reverse scan's record of each 32-token
//     block (the adjoint at its first token from a zero carry, and the decay
//     product applied to the carry);
//   ttt_grad_kernel  CTA per (sequence, 64 channels, 8 blocks), warp per
//     32-token block, a channel pair per lane: folds the later blocks'
//     records into its incoming adjoint (no carry pass), runs the reverse adjoint over its tokens and
//     sums the coefficient gradient; the CTA's blocks are summed in shared
//     memory, and the last CTA of each (sequence, channel group) sums the
//     CTAs in order and applies the spectral scale and Adam.
// G (exact fp32, SIMT) and the transposed, negated W_pred operands are formed
// once per call.  The chunk loop runs natively: gate decays, forward (fp32
// states), wpred_grad_kernel, ttt_grad_kernel, all on the caller's stream in
// one workspace: 3 launches per chunk after the forward's.
#include <cudaTypedefs.h>

#include <type_traits>

#include "orthossm_b200.h"
#include "ossm_eval.cuh"

namespace ossm {
namespace fast {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
}
namespace tttg {

using namespace sm100;

constexpr int kBM = 128;               // tokens per tile (TMEM lanes)
constexpr int kBN = 256;               // output channels per tile (TMEM columns)
constexpr int kSt = 4;                 // ring stages
constexpr int kABytes = kBM * 128;     // one 128-byte-wide K slice of the token tile
constexpr int kBBytes = kBN * 128;     // one 128-byte-wide K slice of the weight tile
constexpr int kStage = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr size_t kSmem = (size_t)kSt * kStage + 1024 + 256;

// Instruction descriptor (dense, fp32 accumulator, K-major A and B):
// bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (kind::f16: 1 =
// bf16; kind::tf32: 2 = tf32), 17-22 N/8, 24-28 M/16.
__host__ __device__ constexpr uint32_t idesc(int fmt, int M, int N) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
constexpr uint32_t kIdTF32 = idesc(2, kBM, kBN);
constexpr uint32_t kIdBF16 = idesc(1, kBM, kBN);

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle
// layout (8-row x 128-byte atoms stacked 1024 bytes apart): start address
// >> 4, stride byte offset 1024 >> 4, descriptor version 1 (bit 46), layout
// 2 = 128-byte swizzle (bits 61-63).  The leading byte offset is unused for
// swizzled K-major layouts.
OSSM_DEV uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3fff) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
template <bool TF32>
OSSM_DEV void mma(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t id, uint32_t acc) {
  if (TF32)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(ad), "l"(bd), "r"(id), "r"(acc)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(ad), "l"(bd), "r"(id), "r"(acc)
        : "memory");
}
// Arrive on `bar` once every tcgen05.mma this thread issued has completed.
OSSM_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

constexpr int kBlk = 32;  // tokens per reverse-scan block (four per token tile)
constexpr int kBoxBytes = kBM * 128;  // one [128 rows x 32 fp32] box of the staged gs tile

struct GParams {
  int L;          // chunk length (tokens)
  int t0;         // the chunk's first token in the sequence
  int D, H, HD;   // channels, heads, channels per head
  int x_bf16;     // x segment: kind::f16 hi + lo (1) or kind::tf32 (0)
  float alpha;    // 2 / ((L-1) D)
  // gs = [B, L-1, D] is written through the mGs map (one launch per chunk)
  // reverse-scan block records (the adjoint at each block's first token from
  // a zero carry, and the product of decays that multiplies the carry)
  const float* lam_h;    // [H] or NULL (momentum)
  float momentum;
  const float* lam_tok;  // [B, L, H] (chunk-relative) or NULL
  int nblk;              // ceil(L / kBlk)
  float* Rrec;           // [B, nblk, D]
  float* Arec;           // [B, nblk, H]
  uint32_t* status;
};

// Decay of token t of the chunk (1 past its end: nothing enters from there).
OSSM_DEV float decay_at(const float* lam_tok, const float* lam_h, float momentum, int L, int H, int b, int t, int h) {
  if (t >= L) return 1.f;
  if (lam_tok) return __ldg(lam_tok + ((size_t)b * L + t) * H + h);
  return lam_h ? __ldg(lam_h + h) : momentum;
}

// Segment and K slice of ring step i: s.G (D/32 slices of 32 fp32), then
// x.W (D/32 tf32 slices, or D/64 bf16 slices against hi and again against lo).
struct Step {
  int seg, k;
};
OSSM_DEV Step step_of(int i, int D, int x_bf16) {
  const int n0 = D / 32;
  if (i < n0) return {0, i};
  i -= n0;
  if (!x_bf16) return {1, i};
  const int n1 = D / 64;
  return i < n1 ? Step{1, i} : Step{2, i - n1};
}

__global__ void __launch_bounds__(kThreads, 1)
    wpred_grad_kernel(const __grid_constant__ CUtensorMap mS, const __grid_constant__ CUtensorMap mG,
                      const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mW0,
                      const __grid_constant__ CUtensorMap mW1, const __grid_constant__ CUtensorMap mGs,
                      const GParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSt * kStage);
  uint64_t* empty = full + kSt;
  uint64_t* accfull = empty + kSt;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accfull + 1);
  __shared__ int failed;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM, b = blockIdx.z;
  const int nsteps = p.D / 32 + (p.x_bf16 ? 2 * (p.D / 64) : p.D / 32);

  if (threadIdx.x == 0) {
    failed = 0;
    for (int s = 0; s < kSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, kBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0 && lane == 0) {  // TMA producer
    prefetch_tmap(&mS);
    prefetch_tmap(&mG);
    prefetch_tmap(&mX);
    prefetch_tmap(&mW0);
    if (p.x_bf16) prefetch_tmap(&mW1);
    prefetch_tmap(&mGs);
    int issued = 0;
    for (int i = 0; i < nsteps; ++i, ++issued) {
      const int s = i % kSt;
      if (i >= kSt && !mbar_wait(&empty[s], ((i / kSt) & 1) ^ 1)) {
        failed = 1;
        break;
      }
      uint8_t* a = smem + s * kStage;
      uint8_t* bb = a + kABytes;
      mbar_expect_tx(&full[s], kStage);
      const Step st = step_of(i, p.D, p.x_bf16);
      const int kw = (st.seg == 0 || !p.x_bf16) ? 32 : 64;  // elements per 128-byte slice
      if (st.seg == 0) {
        tma_load_3d(a, &mS, &full[s], st.k * kw, p.t0 + m0, b);
        tma_load_3d(bb, &mG, &full[s], st.k * kw, n0, 0);
      } else {
        tma_load_3d(a, &mX, &full[s], st.k * kw, p.t0 + m0 + 1, b);
        tma_load_3d(bb, st.seg == 1 ? &mW0 : &mW1, &full[s], st.k * kw, n0, 0);
      }
    }
    // no copy may still be landing in this CTA's shared memory when it exits
    for (int s = 0; s < kSt && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / kSt) * kSt;
      if (!mbar_wait(&full[s], (last / kSt) & 1)) failed = 1;
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    bool ok = true;
    for (int i = 0; i < nsteps; ++i) {
      const int s = i % kSt;
      if (!mbar_wait(&full[s], (i / kSt) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * kStage);
      const uint64_t ad = sdesc(a), bd = sdesc(a + kABytes);
      const Step st = step_of(i, p.D, p.x_bf16);
      const bool tf32 = st.seg == 0 || !p.x_bf16;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K per instruction: 8 tf32 or 16 bf16
        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
        if (tf32)
          mma<true>(tmem, ad + 2 * kk, bd + 2 * kk, kIdTF32, acc);
        else
          mma<false>(tmem, ad + 2 * kk, bd + 2 * kk, kIdBF16, acc);
      }
      mma_commit(&empty[s]);  // the stage is free once these products have read it
    }
    if (!ok) failed = 1;
    mma_commit(accfull);  // the accumulator is final (or the loop gave up)
  } else if (warp >= 2) {  // epilogue: TMEM -> registers -> gs
    const int q = warp & 3;  // the TMEM lane quadrant this warp may access
    // warp-uniform: tcgen05.ld is .sync.aligned
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accfull, 0));
    tc_fence_after();
    const int r = q * 32 + lane, t = m0 + r;
    const bool live = ok && t < p.L - 1;
    // the 2/N-scaled tile goes to shared memory (over the now idle ring) as 8
    // boxes of [128 rows x 32 columns] in the 128-byte swizzle: one TMA store
    // each writes gs, and the block records read it back; zero where
    // t >= L-1 (token L-1 has no loss term)
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
        uint8_t* row = smem + c * kBoxBytes + r * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 g = live ? make_float4(v[4 * j] * p.alpha, v[4 * j + 1] * p.alpha, v[4 * j + 2] * p.alpha,
                                              v[4 * j + 3] * p.alpha)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(row + ((j ^ (r & 7)) << 4)) = g;
        }
      }
    } else {
      failed = 1;
    }
    // the decays a_{t+1} of the tile's rows for its heads
    const int nh = kBN / p.HD, h0 = n0 / p.HD;
    float* dsm = reinterpret_cast<float*>(smem + (kBN / 32) * kBoxBytes);  // [128][nh]
    for (int e = threadIdx.x - 64; e < kBM * nh; e += 128)
      dsm[e] = decay_at(p.lam_tok, p.lam_h, p.momentum, p.L, p.H, b, m0 + 1 + e / nh, h0 + e % nh);
    fence_proxy_async_smem();  // the tile's writes before the TMA store reads them
    named_sync(1, 128);
    if (ok && threadIdx.x == 64) {
      for (int c = 0; c < kBN / 32; ++c) tma_store_3d(&mGs, smem + c * kBoxBytes, n0 + c * 32, m0, b);
      bulk_commit();
    }
    if (ok) {
      // thread e: columns e and e + 128 of each of the tile's 32-token blocks,
      // the 8 reverse chains (R_t = g_t + a_{t+1} R_{t+1}, the reverse adjoint
      // from a zero carry at the block's end) interleaved row by row, and a
      // record at each block's first token
      constexpr int kNB = kBM / kBlk;
      const int e = threadIdx.x - 64;
      const int c0 = e, c1 = e + 128, hh0 = c0 / p.HD, hh1 = c1 / p.HD;
      auto gat = [&](int rr, int col) {
        return *reinterpret_cast<const float*>(smem + (col >> 5) * kBoxBytes + rr * 128 +
                                               (((((col & 31) >> 2) ^ (rr & 7))) << 4) + (col & 3) * 4);
      };
      const int nrows = min(kBM, p.L - m0);  // rows of the tile inside the chunk
      float R0[kNB], R1[kNB], A0[kNB], A1[kNB];
#pragma unroll
      for (int qb = 0; qb < kNB; ++qb) {
        R0[qb] = R1[qb] = 0.f;
        A0[qb] = A1[qb] = 1.f;
      }
#pragma unroll 4
      for (int i = kBlk - 1; i >= 0; --i) {
#pragma unroll
        for (int qb = 0; qb < kNB; ++qb) {
          const int rr = qb * kBlk + i;
          if (rr < nrows) {
            const float a0 = dsm[rr * nh + hh0], a1 = dsm[rr * nh + hh1];
            R0[qb] = fmaf(a0, R0[qb], gat(rr, c0));
            R1[qb] = fmaf(a1, R1[qb], gat(rr, c1));
            A0[qb] *= a0;
            A1[qb] *= a1;
          }
        }
      }
#pragma unroll
      for (int qb = 0; qb < kNB; ++qb) {
        if (qb * kBlk >= nrows) break;
        const int blk = m0 / kBlk + qb;
        float* rec = p.Rrec + ((size_t)b * p.nblk + blk) * p.D + n0;
        rec[c0] = R0[qb];
        rec[c1] = R1[qb];
        if (c0 % p.HD == 0) p.Arec[((size_t)b * p.nblk + blk) * p.H + h0 + hh0] = A0[qb];
        if (c1 % p.HD == 0) p.Arec[((size_t)b * p.nblk + blk) * p.H + h0 + hh1] = A1[qb];
      }
    }
    if (ok && threadIdx.x == 64) bulk_wait_read0();  // the store has read the tile before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kBN);
  }
  if (threadIdx.x == 0 && failed) atomicExch(p.status, (uint32_t)OSSM_ETIMEOUT);
}

// G = W^T W in fp32 (fixed summation order, K ascending): 32 x 32 output
// tile per CTA from the two [D x 32] column panels of W staged in shared
// memory in one pass; 256 threads with 2 x 2 outputs each.
constexpr int kGramPanel = 32;
__global__ void __launch_bounds__(256) gram_kernel(const float* __restrict__ W, int D, float* __restrict__ G) {
  extern __shared__ float pan[];  // [D][32] columns i0.., then [D][32] columns j0..
  float* pa = pan;
  float* pb = pan + (size_t)D * kGramPanel;
  const int i0 = blockIdx.y * kGramPanel, j0 = blockIdx.x * kGramPanel;
  for (int e = threadIdx.x; e < D * (kGramPanel / 4); e += 256) {
    const int n = e / (kGramPanel / 4), c = (e % (kGramPanel / 4)) * 4;
    *reinterpret_cast<float4*>(pa + n * kGramPanel + c) = __ldg(reinterpret_cast<const float4*>(W + (size_t)n * D + i0 + c));
    *reinterpret_cast<float4*>(pb + n * kGramPanel + c) = __ldg(reinterpret_cast<const float4*>(W + (size_t)n * D + j0 + c));
  }
  __syncthreads();
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[2][2] = {};
  for (int n = 0; n < D; ++n) {
    const float a0 = pa[n * kGramPanel + ty * 2], a1 = pa[n * kGramPanel + ty * 2 + 1];
    const float b0 = pb[n * kGramPanel + tx * 2], b1 = pb[n * kGramPanel + tx * 2 + 1];
    acc[0][0] = fmaf(a0, b0, acc[0][0]);
    acc[0][1] = fmaf(a0, b1, acc[0][1]);
    acc[1][0] = fmaf(a1, b0, acc[1][0]);
    acc[1][1] = fmaf(a1, b1, acc[1][1]);
  }
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int w = 0; w < 2; ++w) G[(size_t)(i0 + ty * 2 + u) * D + j0 + tx * 2 + w] = acc[u][w];
}

// The x-side operand, K-major: Wt[j][n] = -W[n][j], as fp32 (tf32 product) or
// as bf16 hi = rn(-W), lo = rn(-W - hi).
__global__ void wpred_operand_kernel(const float* __restrict__ W, int D, float* __restrict__ wt32,
                                     __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)D * D) return;
  const int j = (int)(e / D), n = (int)(e % D);
  const float v = -W[(size_t)n * D + j];
  if (wt32) {
    wt32[e] = v;
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[e] = h;
    lo[e] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

OSSM_DEV float ex2_approx(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
// sech^2 z = 1 - tanh^2 z = 4e / (1 + e)^2 with e = exp(-2|z|) = 2^(-2 log2(e) |z|):
// no cancellation as |z| grows, unlike 1 - u^2 (relative error ~1e-6 on |z| < 4).
OSSM_DEV float sech2(float z) {
  const float e = ex2_approx(-2.8853900817779268f * fabsf(z));
  const float d = 1.f + e;
  return 4.f * e * rcp_fast(d * d);
}

// Reverse adjoint, coefficient gradient and Adam for one chunk, from gs and
// the block records of wpred_grad_kernel.  CTA per (sequence, 64 channels,
// span of 8 blocks), warp per 32-token block; each lane holds a channel pair
// (j, j+1), the operand layout of the packed fp32x2 arithmetic.  Arithmetic
// of rev_grad_kernel / rev_reduce_kernel in ossm_reverse.cu (the TTT
// instantiation):
//   adj_t = g_t + a_{t+1} adj_{t+1}, entering the block with the fold of the
//   later blocks' records C = R_r + A_r C (r from the last block down);
//   dy_t = (1 - a_t) adj_t (1 - u_t^2) gamma_h [|z_t| < 4] (0 for NaN x), with
//   z = gamma y by Horner on the gamma-folded monomial coefficients, 1 - u^2
//   as sech^2 z and xn by the approximate reciprocal (the gradient needs
//   ~1e-5, not the forward's rounding);
//   g_k = sum_t dy_t T_k(xn_t), summed per block, over the CTA's blocks in
//   block order (shared memory), then over the CTAs in span order by the last
//   CTA of the (sequence, channel group) to finish (an atomic ticket; no
//   waiting), which also applies the 1/(k+1)^p scale and Adam with the
//   forget gate, warp k updating coefficient k.
struct RParams {
  int B, L, H, HD, D, K, nblk;
  const void* x;
  int x_bf16;
  long long xsb, xss;
  const float* gs;       // [B, L-1, D]
  const float* lam_h;    // [H] or NULL
  float momentum;
  const float* lam_tok;  // [B, L, H] or NULL
  const float* Rrec;     // [B, nblk, D]
  const float* Arec;     // [B, nblk, H]
  float* part;           // [ceil(nblk/8), B, K, D]: one per CTA
  uint32_t* ticket;      // [B, D/64], zero between launches
  float* coeffs;
  float* m;
  float* v;
  float lr, beta1, beta2, eps, bc1, bc2, spow;
  int forget;
};

// xn = softsign(x) for a channel pair (NaN -> 0; |x| floored at 1e-7 and
// capped at 2^64 as in the forward; approximate reciprocal).
OSSM_DEV float2 softsign2(float2 x) {
  const float x0 = x.x == x.x ? x.x : 0.f, x1 = x.y == x.y ? x.y : 0.f;
  const float2 m = make_float2(fminf(fmaxf(fabsf(x0), 1e-7f), 0x1p64f), fminf(fmaxf(fabsf(x1), 1e-7f), 0x1p64f));
  const float2 d = fma2(m, make_float2(1.f, 1.f), make_float2(1.f, 1.f));
  const float2 xa = mul2(m, make_float2(rcp_fast(d.x), rcp_fast(d.y)));
  return make_float2(x0 >= 0.f ? xa.x : -xa.x, x1 >= 0.f ? xa.y : -xa.y);
}

template <bool TOK>
__global__ void __launch_bounds__(256, 2) ttt_grad_kernel(const RParams p) {
  __shared__ float2 red[8][8][33];  // [warp][k][lane]
  __shared__ float2 cR[8][32];
  __shared__ float cA[8][32];
  __shared__ uint32_t last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngrp = p.D / 64, nspan = (p.nblk + 7) / 8;
  const int span = blockIdx.x % nspan, grp = (blockIdx.x / nspan) % ngrp, b = blockIdx.x / (nspan * ngrp);
  const int blk = span * 8 + warp;  // may lie past the last block: no tokens, zero gradient
  const int ch = grp * 64 + 2 * lane, h = ch / p.HD, j = ch % p.HD;
  const int t0 = blk * kBlk, t1 = min(t0 + kBlk, p.L);
  const float gamma = 0.98f - 0.06f * (float)h / (float)p.H;

  // the adjoint entering from the right: the records of the later blocks,
  // folded C = R_r + A_r C from the last block down.  The blocks past this
  // CTA's span are split over its 8 warps (a composite R, A each, combined
  // through shared memory), then each warp folds the span's blocks after its own.
  const int se = min((span + 1) * 8, p.nblk);  // the first block past the span
  auto fold = [&](int hi, int lo, float2& R, float& A) {  // blocks hi-1 down to lo
    for (int r = hi - 1; r >= lo; r -= 8) {
      float2 Rv[8];
      float Av[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = r - i;
        Rv[i] = rr >= lo ? __ldcg(reinterpret_cast<const float2*>(p.Rrec + ((size_t)b * p.nblk + rr) * p.D + ch))
                         : make_float2(0.f, 0.f);
        Av[i] = rr >= lo ? __ldcg(p.Arec + ((size_t)b * p.nblk + rr) * p.H + h) : 1.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        R = fma2(make_float2(Av[i], Av[i]), R, Rv[i]);
        A *= Av[i];
      }
    }
  };
  {
    const int per = (p.nblk - se + 7) / 8, lo = min(se + warp * per, p.nblk), hi = min(lo + per, p.nblk);
    float2 R = make_float2(0.f, 0.f);
    float A = 1.f;
    fold(hi, lo, R, A);
    cR[warp][lane] = R;
    cA[warp][lane] = A;
  }
  __syncthreads();
  float2 adj = make_float2(0.f, 0.f);
#pragma unroll
  for (int w = 7; w >= 0; --w) adj = fma2(make_float2(cA[w][lane], cA[w][lane]), adj, cR[w][lane]);
  {
    float A = 1.f;
    fold(se, min(blk + 1, se), adj, A);
  }

  // z = gamma y(xn) by Horner on the gamma-folded monomial coefficients
  float2 ck[8], mc[8];
  const float* cb = p.coeffs + ((size_t)b * p.H + h) * p.K * p.HD + j;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    ck[k] = k < p.K ? *reinterpret_cast<const float2*>(cb + (size_t)k * p.HD) : make_float2(0.f, 0.f);
  ev::cheb_to_mono(ck, gamma, mc);
  float2 acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = make_float2(0.f, 0.f);

  const float ah = p.lam_h ? __ldg(p.lam_h + h) : p.momentum;
  auto dec = [&](int t) {  // decay of token t (1 past the chunk's end)
    if (t >= p.L) return 1.f;
    return TOK ? __ldg(p.lam_tok + ((size_t)b * p.L + t) * p.H + h) : ah;
  };
  const float* gp = p.gs + (size_t)b * (p.L - 1) * p.D + ch;
  const char* xp = static_cast<const char*>(p.x) + ((size_t)b * p.xsb + ch) * (p.x_bf16 ? 2 : 4);
  const size_t xrow = (size_t)p.xss * (p.x_bf16 ? 2 : 4);
  // tokens in batches of 8; the next batch's x is loaded once this batch's
  // xn is formed, its gs once this batch's adjoint is done, so both are in
  // flight while the other half of the work runs
  // A full block (all kBlk tokens inside the chunk, the common case) runs
  // without the per-token range checks.
  auto walk = [&](auto full_tag) {
    constexpr bool FULL = decltype(full_tag)::value;
    const int tlast = FULL ? t0 + kBlk - 1 : t1 - 1;
    float2 gv[8], xv[8];
    auto load_g = [&](int tb) {
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int t = tb - i;
        gv[i] = ((FULL || t >= t0) && t < p.L - 1) ? __ldcg(reinterpret_cast<const float2*>(gp + (size_t)t * p.D))
                                         : make_float2(0.f, 0.f);
      }
    };
    auto load_x = [&](int tb) {
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int t = tb - i;
        if (!FULL && t < t0) {
          xv[i] = make_float2(0.f, 0.f);
        } else if (p.x_bf16) {
          const uint32_t r = *reinterpret_cast<const uint32_t*>(xp + t * xrow);
          xv[i] = make_float2(__uint_as_float(r << 16), __uint_as_float(r & 0xffff0000u));
        } else {
          xv[i] = *reinterpret_cast<const float2*>(xp + t * xrow);
        }
      }
    };
    load_x(tlast);
    load_g(tlast);
    for (int tb = tlast; tb >= t0; tb -= 8) {
      const bool more = tb - 8 >= t0;
      // per token, independent of the adjoint: xn and the factor
      // w = (1 - a_t) (1 - u^2) gamma [|z| < 4] (0 for NaN x, where u = 0)
      float2 xn[8], w[8];
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        xn[i] = softsign2(xv[i]);
        float2 z = mc[7];
  #pragma unroll
        for (int q = 6; q >= 0; --q) z = fma2(z, xn[i], mc[q]);
        const float f = (FULL || tb - i >= t0) ? (1.f - dec(tb - i)) * gamma : 0.f;
        w[i] = make_float2((xv[i].x == xv[i].x && fabsf(z.x) < 4.f) ? f * sech2(z.x) : 0.f,
                           (xv[i].y == xv[i].y && fabsf(z.y) < 4.f) ? f * sech2(z.y) : 0.f);
      }
      if (more) load_x(tb - 8);
      // the serial adjoint, then dy T_k into the gradient
  #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float an = (FULL || tb - i >= t0) ? dec(tb - i + 1) : 1.f;
        adj = fma2(make_float2(an, an), adj, gv[i]);
        const float2 dy = mul2(w[i], adj);
        const float2 x2 = fma2(xn[i], make_float2(2.f, 2.f), make_float2(0.f, 0.f));
        float2 ta = make_float2(1.f, 1.f), tb2 = xn[i];
        acc[0] = fma2(dy, ta, acc[0]);
        acc[1] = fma2(dy, tb2, acc[1]);
  #pragma unroll
        for (int k = 2; k < 8; ++k) {
          const float2 tc = sub2(mul2(x2, tb2), ta);
          acc[k] = fma2(dy, tc, acc[k]);
          ta = tb2;
          tb2 = tc;
        }
      }
      if (more) load_g(tb - 8);
    }
  };
  if (t1 - t0 == kBlk)
    walk(std::true_type{});
  else
    walk(std::false_type{});

  // the CTA's 8 blocks in block order, then one partial per CTA
#pragma unroll
  for (int k = 0; k < 8; ++k) red[warp][k][lane] = acc[k];
  __syncthreads();
  const int k = warp;  // from here warp w handles coefficient k = w of the 64 channels
  if (k < p.K) {
    float2 g = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 8; ++w) g = make_float2(g.x + red[w][k][lane].x, g.y + red[w][k][lane].y);
    *reinterpret_cast<float2*>(p.part + (((size_t)span * p.B + b) * p.K + k) * p.D + ch) = g;
  }
  // the last CTA of this (sequence, channel group) to finish reduces and steps
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(p.ticket + (size_t)b * ngrp + grp, 1u) == (uint32_t)nspan - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) p.ticket[(size_t)b * ngrp + grp] = 0;  // ready for the next chunk
  if (k >= p.K) return;
  float2 g = make_float2(0.f, 0.f);
  for (int r = 0; r < nspan; ++r) {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(p.part + (((size_t)r * p.B + b) * p.K + k) * p.D + ch));
    g = make_float2(g.x + v.x, g.y + v.y);
  }
  const float sc = powf((float)(k + 1), -p.spow);
  const float fg = p.forget ? (p.lam_h ? __ldg(p.lam_h + h) : p.momentum) : 1.f;
  const size_t i0 = (((size_t)b * p.H + h) * p.K + k) * p.HD + j;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const size_t i = i0 + e;
    const float gk = (e ? g.y : g.x) * sc;
    const float m = fmaf(p.beta1, p.m[i], (1.f - p.beta1) * gk);
    const float v = fmaf(p.beta2, p.v[i], (1.f - p.beta2) * gk * gk);
    p.m[i] = m;
    p.v[i] = v;
    const float mhat = m / p.bc1, vhat = v / p.bc2;
    p.coeffs[i] = fg * p.coeffs[i] - p.lr * mhat / (sqrtf(vhat) + p.eps);
  }
}

// 3-D tiled map (inner, rows, outer) with a [box_rows x 128 B] box, 128-byte swizzle.
bool encode(CUtensorMap* map, CUtensorMapDataType dt, int esz, const void* base, long long inner, long long rows,
            long long outer, long long row_stride, long long outer_stride, int box_rows) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)outer};
  cuuint64_t strides[2] = {(cuuint64_t)(row_stride * esz), (cuuint64_t)(outer_stride * esz)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fast::encode_fn()(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace tttg
}  // namespace ossm

using namespace ossm;

namespace {

ossm_fwd_args chunk_fwd_args(const ossm_ttt_run_args* a, int t0, int Lc) {
  ossm_fwd_args f{};
  const int D = a->H * a->head_dim;
  const int xel = a->x_dtype == OSSM_BF16 ? 2 : 4;
  f.B = a->B;
  f.S = Lc;
  f.H = a->H;
  f.head_dim = a->head_dim;
  f.degree = a->degree;
  f.x = static_cast<const char*>(a->x) + (size_t)t0 * a->x_stride_s * xel;
  f.x_dtype = a->x_dtype;
  f.x_stride_b = a->x_stride_b;
  f.x_stride_s = a->x_stride_s;
  f.coeffs = a->coeffs;
  f.lam_h = a->lam_h;
  f.momentum = a->momentum;
  f.gate_w = a->gate_w;
  f.gate_b = a->gate_b;
  f.gate_scale = a->gate_scale;
  f.gate_lo = a->gate_lo;
  f.gate_hi = a->gate_hi;
  f.out = a->out + (size_t)t0 * D;
  f.out_dtype = OSSM_F32;
  f.out_stride_b = (int64_t)a->S * D;
  f.out_stride_s = D;
  f.flags = a->flags;
  return f;
}

int run_validate(const ossm_ttt_run_args* a) {
  if (!a || a->B < 1 || a->S < 1 || a->H < 1 || a->head_dim < 1 || a->degree < 1 || a->degree > 8 || a->chunk < 1)
    return OSSM_EINVAL;
  const long long D = (long long)a->H * a->head_dim;
  if (D % tttg::kBN || D > 768) return OSSM_EINVAL;  // G's two [D x 32] panels in shared memory
  if (!a->x || !a->coeffs || !a->m || !a->v || !a->w_pred || !a->out) return OSSM_EINVAL;
  if (a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) return OSSM_EINVAL;
  const int xel = a->x_dtype == OSSM_BF16 ? 2 : 4;
  // TMA: 16-byte aligned base and row / sequence strides
  if (((uintptr_t)a->x % 16) || ((a->x_stride_s * xel) % 16) || (a->B > 1 && (a->x_stride_b * xel) % 16))
    return OSSM_EINVAL;
  if (((uintptr_t)a->out % 16) || ((uintptr_t)a->w_pred % 16)) return OSSM_EINVAL;
  if (a->step0 < 0 || (a->gate_w && !a->gate_b)) return OSSM_EINVAL;
  if (!fast::encode_fn()) return OSSM_EINVAL;
  return OSSM_OK;
}

}  // namespace

namespace {

// Workspace: [forward workspace (its header first)] [G] [x-side W operand]
// [gs] [lam_tok] [state ping-pong] [block records R, A] [gradient partials]
// [tickets].
struct RunLayout {
  size_t fwd, G, wt, gs, lam, state, R, A, part, ticket, total;
  int nblk;
};

bool run_layout(const ossm_ttt_run_args* a, RunLayout* l) {
  const int Lmax = a->chunk < a->S ? a->chunk : a->S;
  const size_t D = (size_t)a->H * a->head_dim;
  ossm_fwd_args f = chunk_fwd_args(a, 0, Lmax);
  f.lam_tok = a->gate_w ? reinterpret_cast<const float*>(16) : nullptr;  // sized as the call with lam_tok
  f.gate_w = nullptr;
  f.gate_b = nullptr;
  const size_t fb = ossm_fwd_workspace_bytes(&f);
  if (!fb) return false;
  l->nblk = (Lmax + tttg::kBlk - 1) / tttg::kBlk;
  size_t off = 0;
  auto take = [&](size_t& at, size_t bytes) {
    at = off;
    off += tttg::al256(bytes);
  };
  take(l->fwd, fb);
  take(l->G, D * D * 4);
  take(l->wt, D * D * 4);  // fp32, or bf16 hi + lo
  take(l->gs, (size_t)a->B * (Lmax > 1 ? Lmax - 1 : 1) * D * 4);
  take(l->lam, a->gate_w ? (size_t)a->B * Lmax * a->H * 4 : 0);
  take(l->state, 2 * tttg::al256((size_t)a->B * D * 4));
  take(l->R, (size_t)a->B * l->nblk * D * 4);
  take(l->A, (size_t)a->B * l->nblk * a->H * 4);
  take(l->part, (size_t)((l->nblk + 7) / 8) * a->B * a->degree * D * 4);
  take(l->ticket, (size_t)a->B * (D / 64) * 4);
  l->total = off;
  return true;
}

}  // namespace

extern "C" size_t ossm_ttt_run_workspace_bytes(const ossm_ttt_run_args* a) {
  if (run_validate(a) != OSSM_OK) return 0;
  RunLayout l;
  return run_layout(a, &l) ? l.total : 0;
}

extern "C" int ossm_ttt_wpred_run(const ossm_ttt_run_args* a, void* workspace, size_t workspace_bytes,
                                  ossm_stream_t stream) {
  const int v = run_validate(a);
  if (v != OSSM_OK) return v;
  RunLayout l;
  if (!run_layout(a, &l)) return OSSM_EINVAL;
  if (!workspace || workspace_bytes < l.total || ((uintptr_t)workspace % 256)) return OSSM_EWORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int D = a->H * a->head_dim;
  const int bf16 = a->x_dtype == OSSM_BF16;
  float* G = reinterpret_cast<float*>(ws + l.G);
  float* wt32 = bf16 ? nullptr : reinterpret_cast<float*>(ws + l.wt);
  __nv_bfloat16* whi = bf16 ? reinterpret_cast<__nv_bfloat16*>(ws + l.wt) : nullptr;
  __nv_bfloat16* wlo = bf16 ? whi + (size_t)D * D : nullptr;
  float* gs = reinterpret_cast<float*>(ws + l.gs);
  float* lam = a->gate_w ? reinterpret_cast<float*>(ws + l.lam) : nullptr;
  float* state[2] = {reinterpret_cast<float*>(ws + l.state),
                     reinterpret_cast<float*>(ws + l.state + tttg::al256((size_t)a->B * D * 4))};
  uint32_t* status = &reinterpret_cast<WsHeader*>(ws + l.fwd)->status;

  // tensor maps over the whole sequence; each chunk passes its first token
  CUtensorMap mS, mG, mX, mW0, mW1;
  bool ok = tttg::encode(&mS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a->out, D, a->S, a->B, D, (long long)a->S * D,
                         tttg::kBM) &&
            tttg::encode(&mG, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, G, D, D, 1, D, (long long)D * D, tttg::kBN);
  const long long xsb = a->B > 1 ? a->x_stride_b : (long long)a->S * a->x_stride_s;
  if (bf16)
    ok = ok &&
         tttg::encode(&mX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->x, D, a->S, a->B, a->x_stride_s, xsb, tttg::kBM) &&
         tttg::encode(&mW0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, whi, D, D, 1, D, (long long)D * D, tttg::kBN) &&
         tttg::encode(&mW1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wlo, D, D, 1, D, (long long)D * D, tttg::kBN);
  else
    ok = ok &&
         tttg::encode(&mX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a->x, D, a->S, a->B, a->x_stride_s, xsb, tttg::kBM) &&
         tttg::encode(&mW0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, wt32, D, D, 1, D, (long long)D * D, tttg::kBN);
  if (!ok) return OSSM_EINVAL;
  if (!bf16) mW1 = mW0;

  if (cudaFuncSetAttribute(tttg::wpred_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)tttg::kSmem) != cudaSuccess)
    return OSSM_ELAUNCH;
  const size_t gram_smem = (size_t)2 * D * tttg::kGramPanel * 4;
  if (cudaFuncSetAttribute(tttg::gram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gram_smem) !=
      cudaSuccess)
    return OSSM_ELAUNCH;
  tttg::gram_kernel<<<dim3(D / tttg::kGramPanel, D / tttg::kGramPanel), 256, gram_smem, st>>>(a->w_pred, D, G);
  tttg::wpred_operand_kernel<<<(unsigned)(((size_t)D * D + 255) / 256), 256, 0, st>>>(a->w_pred, D, wt32, whi, wlo);
  if (cudaGetLastError() != cudaSuccess) return OSSM_ELAUNCH;

  const size_t fb = l.G - l.fwd;
  int cur = 0;
  int step = a->step0;
  for (int t0 = 0; t0 < a->S; t0 += a->chunk) {
    const int Lc = a->chunk < a->S - t0 ? a->chunk : a->S - t0;
    const bool last = t0 + a->chunk >= a->S;
    ossm_fwd_args f = chunk_fwd_args(a, t0, Lc);
    if (a->gate_w) {
      int r = ossm_gate_decay(&f, lam, stream);
      if (r != OSSM_OK) return r;
      f.lam_tok = lam;
      f.gate_w = nullptr;
      f.gate_b = nullptr;
    }
    f.init_state = t0 == 0 ? a->init_state : state[cur];
    f.final_state = (last && a->final_state) ? a->final_state : state[cur ^ 1];
    int r = ossm_cheby_ema_fwd(&f, ws + l.fwd, fb, stream);
    if (r != OSSM_OK) return r;
    cur ^= 1;
    const float* lt = a->gate_w ? lam : nullptr;
    if (Lc > 1) {
      tttg::GParams gp;
      gp.L = Lc;
      gp.t0 = t0;
      gp.D = D;
      gp.H = a->H;
      gp.HD = a->head_dim;
      gp.x_bf16 = bf16;
      gp.alpha = 2.f / ((float)(Lc - 1) * (float)D);
      gp.lam_h = a->lam_h;
      gp.momentum = a->momentum;
      gp.lam_tok = lt;
      gp.nblk = (Lc + tttg::kBlk - 1) / tttg::kBlk;
      gp.Rrec = reinterpret_cast<float*>(ws + l.R);
      gp.Arec = reinterpret_cast<float*>(ws + l.A);
      gp.status = status;
      CUtensorMap mGs;  // gs [B, Lc-1, D]: rows past Lc-1 are not stored
      if (!tttg::encode(&mGs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, gs, D, Lc - 1, a->B, D, (long long)(Lc - 1) * D,
                        tttg::kBM))
        return OSSM_EINVAL;
      const dim3 grid(D / tttg::kBN, (Lc + tttg::kBM - 1) / tttg::kBM, a->B);
      tttg::wpred_grad_kernel<<<grid, tttg::kThreads, tttg::kSmem, st>>>(mS, mG, mX, mW0, mW1, mGs, gp);
    }
    ++step;
    tttg::RParams rp;
    rp.B = a->B;
    rp.L = Lc;
    rp.H = a->H;
    rp.HD = a->head_dim;
    rp.D = D;
    rp.K = a->degree;
    rp.nblk = (Lc + tttg::kBlk - 1) / tttg::kBlk;
    rp.x = f.x;
    rp.x_bf16 = bf16;
    rp.xsb = a->x_stride_b;
    rp.xss = a->x_stride_s;
    rp.gs = gs;
    rp.lam_h = a->lam_h;
    rp.momentum = a->momentum;
    rp.lam_tok = lt;
    rp.Rrec = reinterpret_cast<float*>(ws + l.R);
    rp.Arec = reinterpret_cast<float*>(ws + l.A);
    rp.part = reinterpret_cast<float*>(ws + l.part);
    rp.ticket = reinterpret_cast<uint32_t*>(ws + l.ticket);
    rp.coeffs = a->coeffs;
    rp.m = a->m;
    rp.v = a->v;
    rp.lr = a->lr;
    rp.beta1 = a->beta1;
    rp.beta2 = a->beta2;
    rp.eps = a->eps;
    rp.bc1 = 1.f - powf(a->beta1, (float)step);
    rp.bc2 = 1.f - powf(a->beta2, (float)step);
    rp.spow = a->spectral_pow;
    rp.forget = a->forget;
    const unsigned ctas = (unsigned)(a->B * (D / 64) * ((rp.nblk + 7) / 8));
    if (lt)
      tttg::ttt_grad_kernel<true><<<ctas, 256, 0, st>>>(rp);
    else
      tttg::ttt_grad_kernel<false><<<ctas, 256, 0, st>>>(rp);
    if (cudaGetLastError() != cudaSuccess) return OSSM_ELAUNCH;
  }
  return OSSM_OK;
}
