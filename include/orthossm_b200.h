/*
 * orthossm_b200 — C ABI of the B200-native Cheby-RKV hot path.
 *
 * Plain pointers and sizes; no torch types.  Every entry point is
 * stream-ordered on the caller's stream, allocates no device memory, and
 * returns an ossm_status.  Some spread their work over side streams the
 * library creates once per device (the bf16 forward of a large batch, the
 * host-buffer forward); that work is forked from and joined back to the
 * caller's stream within the call.  Device pointers are caller-allocated.  Tensors are row-major
 * and contiguous along the channel axis; [B,S,D] activations take explicit
 * batch / token strides in elements.
 *
 * Reference interfaces replaced (paths relative to the Eddym06/OrthoSSM root):
 *   ossm_cheby_ema_fwd   <- _fused_clenshaw_ema_kernel launch
 *                           (sdpc_kernel.py:988-1209, launched as in
 *                           precision_tests.py:60-72) generalised to per-head
 *                           and per-token decay, carried state and bf16 I/O;
 *                           also the fast path _fast_path_forward
 *                           (sdpc_kernel.py:1708-1744) via flags.
 *   ossm_cheby_rkv_lion  <- the chunk loop of apply_cheby_rkv_v10
 *                           (sdpc_kernel.py:2574-2606) around
 *                           FusedChebyRKVv10.forward (:2352-2433) and
 *                           _launch_ortho_megakernel / _ortho_megakernel
 *                           (:2290-2344, :1889-2287): forward + local TTT
 *                           gradient + inline Lion for every chunk, in one
 *                           launch.
 */
#ifndef ORTHOSSM_B200_H
#define ORTHOSSM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* ossm_stream_t;

enum ossm_status {
  OSSM_OK = 0,
  OSSM_EINVAL = 1,    /* bad shape, pointer, alignment or flag */
  OSSM_ELAUNCH = 2,   /* CUDA launch / runtime error */
  OSSM_ETIMEOUT = 3,  /* a bounded device-side wait gave up (see ossm_workspace_status) */
  OSSM_ECOMM = 4,     /* multi-GPU exchange error */
  OSSM_EWORKSPACE = 5 /* workspace missing or too small */
};

enum ossm_dtype { OSSM_F32 = 0, OSSM_BF16 = 1 };

/* Chebyshev evaluation mode (low 2 bits of flags). */
#define OSSM_EVAL_CLENSHAW 0u      /* exact degree-K Clenshaw (sdpc_kernel.py:1147-1156) */
#define OSSM_EVAL_LUT 1u           /* 256-point half table + linear interpolation (:1098-1138) */
#define OSSM_EVAL_CLENSHAW_DEG4 2u /* megakernel USE_LUT=False: only c_0..c_3 (:2073-2077) */
#define OSSM_EVAL_MASK 3u
/* Fast-path semantics (sdpc_kernel.py:1722-1739): x.sign() softsign with
 * sign(0)=0 and NaN -> 0, and unclamped exact tanh. */
#define OSSM_F_FASTPATH (1u << 2)
/* Force correctly-rounded-grade tanh/softsign even for bf16 output. */
#define OSSM_F_PRECISE (1u << 3)
/* Use the generic forward kernel even where the TMA / tcgen05 path applies
 * (the two paths compute the same function; used to test one against the other). */
#define OSSM_F_GENERIC (1u << 4)
/* On the bf16 fast path with bf16 output and 8 to (SM count) sequences, use
 * the single-evaluation grouped kernel (x read and every element evaluated
 * once: one cooperative launch, one CTA per SM, each sequence owned by a
 * group of CTAs that exchange tile aggregates through the workspace) instead
 * of the default three-pass kernels (chunk aggregates, carry scan, outputs;
 * x read and evaluated twice).  Same function; the two differ only in the
 * fp32 rounding of the carried state.  Measured on B200 at BASELINE.json
 * configs[1] it is slower than the three-pass path, so it is opt-in. */
#define OSSM_F_SINGLE_EVAL (1u << 5)
/* Keep all of the call's work on the caller's stream: no side streams, so the
 * bf16 forward of a large batch does not split into two halves (same results,
 * bitwise) and one long sequence (at least 4096 chunks of 32 tokens) does not
 * split into two token ranges (same results up to the fp32 rounding of the
 * carried state). */
#define OSSM_F_ONE_STREAM (1u << 7)

/* ---------------------------------------------------------------------------
 * Fused softsign -> Chebyshev -> gamma_h damping -> tanh -> lambda-EMA scan.
 *
 *   xn = softsign(x); y_h = sum_k c[b,h,k,j] T_k(xn); z = gamma_h y,
 *   gamma_h = 0.98 - 0.06 h / H; u = tanh(clamp(z, -4, 4)) (0 where x is NaN);
 *   s_t = clamp(a_t s_{t-1} + (1 - a_t) u_t, -1, 1), s_{-1} = init_state.
 *   a_t = momentum (lam_h == NULL), lam_h[h], or with the gate
 *   clamp(lam_h[h] + gate_scale * (sigmoid(gate_w[h] . x_t + gate_b[h]) - 0.5),
 *         gate_lo, gate_hi).
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t B, S, H, head_dim, degree; /* head_dim power of two in [8,256]; 1 <= degree <= 8 */
  const void* x;                     /* [B,S,H*head_dim], dtype x_dtype */
  int32_t x_dtype;
  int64_t x_stride_b, x_stride_s;    /* in elements; channel stride 1 */
  const float* coeffs;               /* [B,H,degree,head_dim] contiguous */
  const float* lam_h;                /* [H] or NULL */
  float momentum;                    /* decay used when lam_h == NULL */
  const float* gate_w;               /* [H, H*head_dim] or NULL (no dynamic decay) */
  const float* gate_b;               /* [H] (required with gate_w) */
  float gate_scale, gate_lo, gate_hi;
  const float* lut;                  /* [8,256] table for OSSM_EVAL_LUT, else NULL */
  const float* init_state;           /* [B,H*head_dim] or NULL (zeros) */
  float* final_state;                /* [B,H*head_dim] or NULL */
  void* out;                         /* [B,S,H*head_dim], dtype out_dtype */
  int32_t out_dtype;
  int64_t out_stride_b, out_stride_s;
  float* tanh_out;                   /* optional f32 cache of u, same strides as out */
  const float* lam_tok;              /* optional caller-computed per-token decay [B,S,H]
                                        (e.g. from ossm_gate_decay); overrides the gate */
  uint32_t flags;
} ossm_fwd_args;

/* Bytes of device workspace ossm_cheby_ema_fwd needs for these arguments.
 * The workspace must be zero-filled once when first allocated and may then be
 * reused by any number of calls that are ordered on one stream. */
size_t ossm_fwd_workspace_bytes(const ossm_fwd_args* a);
int ossm_cheby_ema_fwd(const ossm_fwd_args* a, void* workspace, size_t workspace_bytes,
                       ossm_stream_t stream);

/* Which kernels ossm_cheby_ema_fwd runs for these arguments on the current
 * device (no launch): the generic kernel (any dtype / head size / mode), the
 * three-pass bf16 kernels (chunk aggregates, carry scan, outputs: 4 launches
 * per group of sequences), the parked three-pass kernels (bf16 outputs
 * contiguous along tokens, sequences of at most 24 MB of fp16 u: one setup
 * launch, then per slab of sequences an aggregate pass that parks u in L2
 * and forms the carries, and an output pass that reads u back), or the
 * single-evaluation grouped kernel (one cooperative launch, one CTA per SM,
 * each sequence owned by a group of CTAs that exchange tile aggregates
 * through the workspace); -1 for invalid arguments. */
#define OSSM_PATH_GENERIC 0
#define OSSM_PATH_THREE_PASS 1
#define OSSM_PATH_GROUPED 2
#define OSSM_PATH_PARKED 3
int ossm_fwd_path(const ossm_fwd_args* a);

/* ossm_cheby_ema_fwd for callers that cannot allocate device memory (a host
 * whose allocator owns all device memory, a plugin that is only handed its
 * input and output buffers).  No counterpart in the reference: its kernels
 * allocate their scratch through torch.
 *
 * The scratch comes from one fixed array of OSSM_NOALLOC_SCRATCH_BYTES inside
 * the library, held on every GPU that loads the library until the process
 * exits.  Arguments whose ossm_fwd_workspace_bytes exceeds it are rejected
 * with OSSM_EWORKSPACE before any launch (16 MiB covers, for example, bf16
 * x with 8 heads of 64 and the gate on, up to about 100,000 tokens B * S).  All
 * calls on a GPU share the array, so calls that overlap on the GPU race on it.
 * The first call on each GPU sets the array up (device address, a clear on
 * `stream`): make it before other work that could overlap it and before any
 * stream capture.  If `scratch` is not NULL it receives the array's device
 * address, for ossm_workspace_status.  All of its work stays on `stream`
 * (it runs as if OSSM_F_ONE_STREAM were set). */
#define OSSM_NOALLOC_SCRATCH_BYTES (16u << 20)
int ossm_cheby_ema_fwd_noalloc(const ossm_fwd_args* a, ossm_stream_t stream, void** scratch);

/* ossm_cheby_ema_fwd on a batch in HOST memory: a->x, a->out, a->init_state
 * and a->final_state are host pointers (x and out contiguous [B,S,D]; pinned
 * memory for the copies to overlap, pageable memory works but serialises);
 * a->coeffs, a->lam_h, a->gate_w, a->gate_b, a->lam_tok and a->lut are device
 * pointers as for ossm_cheby_ema_fwd; a->tanh_out must be NULL.  The batch
 * goes through the GPU in about `pieces` parts (groups of whole sequences, or
 * token ranges of every sequence with the EMA state carried across them):
 * the copy in of one part, the forward of the next and the copy out of the
 * one before overlap on side streams that the library keeps per device.  The
 * caller's stream waits for all of it, so host reads of out / final_state
 * are valid once that stream's work is done.  Whole-sequence parts give
 * bitwise the forward of the whole batch; token-range parts differ from it
 * only in the rounding of the carried state.  The workspace is device memory
 * of ossm_fwd_host_workspace_bytes(a, pieces), zero-filled once, reused by
 * host calls ordered on one stream; it holds staging buffers, so it must not
 * be shared with the other entry points (their workspaces keep launch state
 * between calls).  Its first 256 bytes are the forward's header, which
 * ossm_workspace_status reads.  Calls on one device are enqueued one at a
 * time (a lock); stream capture is not supported.
 * The reference has no host-buffer call: its callers move tensors to the
 * GPU themselves before the kernel launch (sdpc_kernel.py:988-1209 with
 * precision_tests.py:60-72); this entry point is that move, overlapped. */
size_t ossm_fwd_host_workspace_bytes(const ossm_fwd_args* a, int pieces);
int ossm_cheby_ema_fwd_host(const ossm_fwd_args* a, int pieces, void* workspace, size_t workspace_bytes,
                            ossm_stream_t stream);

/* The per-token decay of the gate alone: lam_tok[b,t,h] (f32, [B,S,H]) from
 * a->x, a->gate_w, a->gate_b, a->lam_h, a->gate_scale/lo/hi.  Feeding the
 * result back through a->lam_tok gives the same output as the gated call.
 * No counterpart kernel in the reference (its gate is per batch,
 * GatedComplexityPredictor, sdpc_kernel.py:1818-1830)
 * configs[1] defines the per-token form. */
int ossm_gate_decay(const ossm_fwd_args* a, float* lam_tok, ossm_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence sharding (no counterpart in the reference,
 * whose streaming loop is sequential, sdpc_kernel.py:2574-2606).  Rank r holds
 * the consecutive tokens of shard r of every sequence in a->x (a->S = shard
 * length).  Bf16 fast path only (bf16 x, 8 heads of 64); workspace as given by
 * ossm_fwd_workspace_bytes(a).
 *
 *  1. ossm_fwd_shard_aggregate: chunk aggregates and carries of the shard from
 *     a zero state (from a->init_state on the shard that starts the sequence),
 *     and the shard's totals: shard_decay[b*H + h] = the product of the decays
 *     over the shard, shard_state[b*D + d] = the state at its end.  With
 *     shard_state = shard_decay + B*H the totals form one packed record of
 *     B*H + B*D floats, so one all-gather moves them.
 *  2. The caller all-gathers the packed records into totals
 *     [nshards][B*H + B*D] (rank order).
 *  3. ossm_fwd_shard_output: folds, on the device and in shard order, the
 *     state entering shard `shard` from totals[0 .. shard) and seq_init (the
 *     state before token 0 of the sequence, or NULL for zeros):
 *     X_0 = seq_init, X_{q+1} = shard_decay_q * X_q + shard_state_q; then
 *     writes the shard's outputs (and final_state, the state after its last
 *     token) on the workspace step 1 filled.  Shard 0 starts from
 *     a->init_state and reads no totals.
 *  ossm_fwd_shard_fold writes the state after the first `nshards` shards
 *  ([B*D], the same fold; nshards = all shards gives the sequence's final
 *  state on every rank). */
int ossm_fwd_shard_aggregate(const ossm_fwd_args* a, int starts_sequence, void* workspace, size_t workspace_bytes,
                             float* shard_decay, float* shard_state, ossm_stream_t stream);
int ossm_fwd_shard_output(const ossm_fwd_args* a, int shard, const float* totals, const float* seq_init,
                          void* workspace, size_t workspace_bytes, ossm_stream_t stream);
int ossm_fwd_shard_fold(int32_t B, int32_t H, int32_t head_dim, int32_t nshards, const float* totals,
                        const float* seq_init, float* state_out, ossm_stream_t stream);

/* Read (and optionally clear) the sticky device status word of a workspace:
 * OSSM_OK, or OSSM_ETIMEOUT if a look-back wait gave up.  Synchronises the
 * stream. */
int ossm_workspace_status(void* workspace, int clear, ossm_stream_t stream, int32_t* status);

/* ---------------------------------------------------------------------------
 * Reference-mode TTT: apply_cheby_rkv_v10's full path over the whole sequence.
 * For each chunk of `chunk` tokens: EMA from zero with scalar momentum, output
 * (rounded to bf16 as the reference does), local gated-error gradient
 * g_k = sum_t e_t sigmoid(3|e_t|) T_k(xn_t) / (L-1), e_t = xn_{t+1} - s_t,
 * then Lion: c <- (lam_eff - lr wd) c + lr (k+1)^-1.5 sign(b1 m + (1-b1) g),
 * m <- b2 m + (1-b2) g, with lam_h / lr_scale_h of _get_lion_constants
 * (sdpc_kernel.py:1423-1437).  coeffs and momentum are updated in place.
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t B, S, H, head_dim, degree, chunk;
  const void* x;                  /* [B,S,D]; rounded to bf16 on load when f32 */
  int32_t x_dtype;
  int64_t x_stride_b, x_stride_s;
  float* coeffs;                  /* [B,H,degree,head_dim], in/out */
  float* momentum;                /* [B,H,degree,head_dim], in/out */
  const float* gate_global;       /* [B] lr multiplier or NULL */
  const float* dynamic_lambda;    /* [B] forget-factor modulation or NULL */
  float ema_momentum, base_lr, beta1, beta2, weight_decay;
  const float* lut;               /* [8,256] for OSSM_EVAL_LUT */
  void* out;                      /* [B,S,D] */
  int32_t out_dtype;
  int64_t out_stride_b, out_stride_s;
  float* tanh_out;                /* optional f32 [B,S,D] (contiguous strides of out) */
  float* final_state;             /* optional [B,D]: EMA state at the end of the last chunk */
  uint32_t flags;                 /* OSSM_EVAL_* */
  float* coeff_trace;             /* optional [ceil(S/chunk)][B,H,degree,head_dim]: the
                                     coefficients each chunk starts from (for the backward) */
} ossm_lion_args;

int ossm_cheby_rkv_lion(const ossm_lion_args* a, ossm_stream_t stream);

/* ---------------------------------------------------------------------------
 * Backward of ossm_cheby_ema_fwd (Clenshaw evaluation, fused semantics):
 * given grad_out = dL/dout [B,S,D], writes grad_x [B,S,D], grad_coeffs
 * [B,H,degree,head_dim] and (if not NULL) grad_init [B,D].  The decays (lam_h /
 * momentum, or the per-token lam_tok a gated forward used) are constants, as
 * in the reference's backward (FusedChebyRKVv10.backward,
 * sdpc_kernel.py:2435-2515, gradients for x and the coefficients only):
 *   adj_t = g_t + a_{t+1} adj_{t+1};  dy_t = (1-a_t) adj_t (1-u_t^2) gamma_h [|z_t| < 4];
 *   dc_k = sum_t dy_t T_k(xn_t);  dx_t = dy_t y'(xn_t) / (1+|x_t|)^2;
 *   d init = a_0 adj_0 (zero where the token-0 clamp bites).
 * head_dim <= 256.
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t B, S, H, head_dim, degree;
  const void* x;                     /* the forward's input */
  int32_t x_dtype;
  int64_t x_stride_b, x_stride_s;
  const float* coeffs;               /* [B,H,degree,head_dim] */
  const float* lam_h;                /* [H] or NULL (momentum) */
  float momentum;
  const float* lam_tok;              /* [B,S,H] or NULL */
  const float* init_state;           /* [B,D] or NULL: the forward's carried-in state */
  const void* grad_out;              /* dL/dout */
  int32_t grad_out_dtype;
  int64_t grad_out_stride_b, grad_out_stride_s;
  void* grad_x;                      /* dL/dx (written) */
  int32_t grad_x_dtype;
  int64_t grad_x_stride_b, grad_x_stride_s;
  float* grad_coeffs;                /* dL/dcoeffs (written) */
  float* grad_init;                  /* dL/dinit_state [B,D] (written) or NULL */
  int32_t segment;                   /* 0, or the forward restarted its EMA from zero every
                                        `segment` tokens (the reference's chunk loop) */
  const float* segment_coeffs;       /* with segment: [ceil(S/segment)][B,H,degree,head_dim], the
                                        coefficients of each segment (coeffs is then segment 0's) */
  uint32_t flags;                    /* OSSM_F_FASTPATH: the fast-path forward (unclamped tanh,
                                        sign(0) = 0, NaN -> xn = 0) */
} ossm_bwd_args;

size_t ossm_bwd_workspace_bytes(const ossm_bwd_args* a);
int ossm_cheby_ema_bwd(const ossm_bwd_args* a, void* workspace, size_t workspace_bytes, ossm_stream_t stream);

/* ---------------------------------------------------------------------------
 * BASELINE-mode TTT step for one chunk (no
 * counterpart kernel in the reference, whose TTT is the local gated-error Lion
 * step of sdpc_kernel.py:2126-2287).  Inputs: the chunk's x, its coefficients
 * (those the forward used), the per-token decays, and
 * gs = dL/ds = (2/N) W_pred^T (W_pred s_t - x_{t+1}) for t < L-1 ([B,L-1,D]
 * fp32, contiguous; the caller forms it with two GEMMs).  Runs the reverse EMA
 * adjoint, dy = (1-a_t) adj_t (1-u_t^2) gamma_h [|z_t| < 4], the gradient
 * g_k = sum_t dy_t T_k(xn_t) / (k+1)^spectral_pow, and Adam on coeffs / m / v
 * in place: c <- lam_h c - lr mhat / (sqrt(vhat) + eps) (lam_h = 1 when
 * forget == 0), with bias corrections for Adam step `step` (>= 1).
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t B, L, H, head_dim, degree; /* head_dim <= 256, degree <= 8 */
  const void* x;                     /* [B,L,H*head_dim] */
  int32_t x_dtype;
  int64_t x_stride_b, x_stride_s;
  float* coeffs;                     /* [B,H,degree,head_dim], in/out */
  float* m;                          /* Adam first moment, same shape, in/out */
  float* v;                          /* Adam second moment, same shape, in/out */
  const float* lam_h;                /* [H] or NULL (momentum) */
  float momentum;
  const float* lam_tok;              /* [B,L,H] per-token decays or NULL (lam_h) */
  const float* gs;                   /* [B,L-1,H*head_dim] fp32 */
  float lr, beta1, beta2, eps, spectral_pow;
  int32_t step;                      /* Adam step number of this update, >= 1 */
  int32_t forget;                    /* 1: forget gate lam_h on c */
} ossm_ttt_args;

size_t ossm_ttt_workspace_bytes(const ossm_ttt_args* a);
int ossm_ttt_wpred_step(const ossm_ttt_args* a, void* workspace, size_t workspace_bytes, ossm_stream_t stream);

/* ---------------------------------------------------------------------------
 * BASELINE-mode TTT over a whole sequence in one call (BASELINE.json
 * configs[3]; no counterpart in the reference).  For each chunk of `chunk`
 * tokens, in order: the gate's per-token decays (gate_w != NULL), the forward
 * with fp32 states into out[:, chunk] (carried state across chunks, starting
 * from init_state), gs_t = (2/N) W_pred^T (W_pred s_t - x_{t+1}) for t < L-1
 * (N = (L-1) D), and ossm_ttt_wpred_step's reverse adjoint, gradient and Adam
 * with step number step0 + chunk index + 1.  gs is formed on the tensor cores
 * by one kernel per chunk as (2/N) (G s_t - W_pred^T x_{t+1}) with
 * G = W_pred^T W_pred (exact fp32, formed once per call): s . G as a TF32
 * product, x . W_pred as bf16 x times W_pred split into two bf16 terms (fp32
 * x: one TF32 product).  H * head_dim must be a multiple of 256; x needs
 * 16-byte aligned rows.  out is [B,S,H*head_dim] fp32, contiguous.
 * The workspace (ossm_ttt_run_workspace_bytes) must be zero-filled once when
 * first allocated; its first 256 bytes are a header that
 * ossm_workspace_status reads.
 * ------------------------------------------------------------------------ */
typedef struct {
  int32_t B, S, H, head_dim, degree, chunk;
  const void* x;                     /* [B,S,H*head_dim] */
  int32_t x_dtype;
  int64_t x_stride_b, x_stride_s;
  float* coeffs;                     /* [B,H,degree,head_dim], in/out */
  float* m;                          /* Adam first moment, in/out */
  float* v;                          /* Adam second moment, in/out */
  const float* lam_h;                /* [H] or NULL (momentum) */
  float momentum;
  const float* gate_w;               /* [H, H*head_dim] or NULL (no gate) */
  const float* gate_b;               /* [H] (with gate_w) */
  float gate_scale, gate_lo, gate_hi;
  const float* w_pred;               /* [D,D] fp32, row-major */
  const float* init_state;           /* [B,D] or NULL (zeros) */
  float* final_state;                /* [B,D] or NULL: the state after the last token */
  float* out;                        /* [B,S,D] fp32 contiguous: the states */
  float lr, beta1, beta2, eps, spectral_pow;
  int32_t step0;                     /* Adam steps already taken */
  int32_t forget;                    /* 1: forget gate lam_h on c */
  uint32_t flags;                    /* forward flags (OSSM_EVAL_*) */
} ossm_ttt_run_args;

size_t ossm_ttt_run_workspace_bytes(const ossm_ttt_run_args* a);
int ossm_ttt_wpred_run(const ossm_ttt_run_args* a, void* workspace, size_t workspace_bytes, ossm_stream_t stream);

/* Library metadata. */
const char* ossm_version(void);
const char* ossm_status_string(int status);
/* sizeof() of the argument structs, so bindings can check their layout. */
size_t ossm_sizeof_fwd_args(void);
size_t ossm_sizeof_lion_args(void);
size_t ossm_sizeof_ttt_args(void);
size_t ossm_sizeof_bwd_args(void);
size_t ossm_sizeof_ttt_run_args(void);

#ifdef __cplusplus
}
#endif
#endif /* ORTHOSSM_B200_H */
