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
//     store gs for t < L-1.
// G (exact fp32, SIMT) and the transposed, negated W_pred operands are formed
// once per call.  The chunk loop runs natively: gate decays, forward (fp32
// states), wpred_grad_kernel, then the reverse adjoint / gradient / Adam
// kernels of ossm_reverse.cu, all on the caller's stream in one workspace.
#include <cudaTypedefs.h>

#include "orthossm_b200.h"
#include "ossm_sm100.cuh"

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

struct GParams {
  int L;          // chunk length (tokens)
  int t0;         // the chunk's first token in the sequence
  int D;          // channels
  int x_bf16;     // x segment: kind::f16 hi + lo (1) or kind::tf32 (0)
  float alpha;    // 2 / ((L-1) D)
  float* gs;      // [B, L-1, D]
  uint32_t* status;
};

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
                      const __grid_constant__ CUtensorMap mW1, const GParams p) {
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
    const int t = m0 + q * 32 + lane;
    const bool live = ok && t < p.L - 1;
    float* dst = p.gs + ((size_t)b * (p.L - 1) + (live ? t : 0)) * p.D + n0;
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
        if (live) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + c * 32 + j) =
                make_float4(v[j] * p.alpha, v[j + 1] * p.alpha, v[j + 2] * p.alpha, v[j + 3] * p.alpha);
        }
      }
    } else {
      failed = 1;
    }
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

// G = W^T W in fp32 (fixed summation order): 64 x 64 output tile per CTA,
// 16 x 16 threads with 4 x 4 outputs each.
__global__ void __launch_bounds__(256) gram_kernel(const float* __restrict__ W, int D, float* __restrict__ G) {
  __shared__ float a[16][64 + 4], bsh[16][64 + 4];
  const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int n0 = 0; n0 < D; n0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      const int r = e >> 6, c = e & 63;
      a[r][c] = W[(size_t)(n0 + r) * D + i0 + c];
      bsh[r][c] = W[(size_t)(n0 + r) * D + j0 + c];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float av[4], bv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        av[u] = a[r][ty * 4 + u];
        bv[u] = bsh[r][tx * 4 + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(av[u], bv[w], acc[u][w]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int w = 0; w < 4; ++w) G[(size_t)(i0 + ty * 4 + u) * D + j0 + tx * 4 + w] = acc[u][w];
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
  if (D % tttg::kBN || D > 4096) return OSSM_EINVAL;
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

ossm_ttt_args chunk_ttt_args(const ossm_ttt_run_args* a, int t0, int Lc, const float* lam_tok, const float* gs,
                             int step) {
  ossm_ttt_args r{};
  const int xel = a->x_dtype == OSSM_BF16 ? 2 : 4;
  r.B = a->B;
  r.L = Lc;
  r.H = a->H;
  r.head_dim = a->head_dim;
  r.degree = a->degree;
  r.x = static_cast<const char*>(a->x) + (size_t)t0 * a->x_stride_s * xel;
  r.x_dtype = a->x_dtype;
  r.x_stride_b = a->x_stride_b;
  r.x_stride_s = a->x_stride_s;
  r.coeffs = a->coeffs;
  r.m = a->m;
  r.v = a->v;
  r.lam_h = a->lam_h;
  r.momentum = a->momentum;
  r.lam_tok = lam_tok;
  r.gs = gs;
  r.lr = a->lr;
  r.beta1 = a->beta1;
  r.beta2 = a->beta2;
  r.eps = a->eps;
  r.spectral_pow = a->spectral_pow;
  r.step = step;
  r.forget = a->forget;
  return r;
}

// Workspace: [forward workspace (its header first)] [G] [x-side W operand]
// [gs] [lam_tok] [state ping-pong] [reverse workspace].
struct RunLayout {
  size_t fwd, G, wt, gs, lam, state, rev, total;
};

bool run_layout(const ossm_ttt_run_args* a, RunLayout* l) {
  const int Lmax = a->chunk < a->S ? a->chunk : a->S;
  const size_t D = (size_t)a->H * a->head_dim;
  ossm_fwd_args f = chunk_fwd_args(a, 0, Lmax);
  f.lam_tok = a->gate_w ? reinterpret_cast<const float*>(16) : nullptr;  // sized as the call with lam_tok
  f.gate_w = nullptr;
  const size_t fb = ossm_fwd_workspace_bytes(&f);
  float dummy;
  ossm_ttt_args r = chunk_ttt_args(a, 0, Lmax, nullptr, &dummy, a->step0 + 1);
  const size_t rb = ossm_ttt_workspace_bytes(&r);
  if (!fb || !rb) return false;
  size_t off = 0;
  l->fwd = off;
  off += tttg::al256(fb);
  l->G = off;
  off += tttg::al256(D * D * 4);
  l->wt = off;
  off += tttg::al256(D * D * 4);  // fp32, or bf16 hi + lo
  l->gs = off;
  off += tttg::al256((size_t)a->B * (Lmax > 1 ? Lmax - 1 : 1) * D * 4);
  l->lam = off;
  if (a->gate_w) off += tttg::al256((size_t)a->B * Lmax * a->H * 4);
  l->state = off;
  off += 2 * tttg::al256((size_t)a->B * D * 4);
  l->rev = off;
  off += tttg::al256(rb);
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
  tttg::gram_kernel<<<dim3(D / 64, D / 64), 256, 0, st>>>(a->w_pred, D, G);
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
    if (Lc > 1) {
      tttg::GParams gp;
      gp.L = Lc;
      gp.t0 = t0;
      gp.D = D;
      gp.x_bf16 = bf16;
      gp.alpha = 2.f / ((float)(Lc - 1) * (float)D);
      gp.gs = gs;
      gp.status = status;
      const dim3 grid(D / tttg::kBN, (Lc + tttg::kBM - 1) / tttg::kBM, a->B);
      tttg::wpred_grad_kernel<<<grid, tttg::kThreads, tttg::kSmem, st>>>(mS, mG, mX, mW0, mW1, gp);
      if (cudaGetLastError() != cudaSuccess) return OSSM_ELAUNCH;
    }
    ++step;
    ossm_ttt_args ra = chunk_ttt_args(a, t0, Lc, a->gate_w ? lam : nullptr, Lc > 1 ? gs : nullptr, step);
    r = ossm_ttt_wpred_step(&ra, ws + l.rev, l.total - l.rev, stream);
    if (r != OSSM_OK) return r;
  }
  return OSSM_OK;
}
