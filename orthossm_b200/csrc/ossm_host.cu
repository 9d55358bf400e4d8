// ossm_cheby_ema_fwd_host: the forward of a batch that lives in host memory.
//
// The batch goes through the GPU in parts: groups of whole sequences when
// there are at least as many sequences as parts, else every sequence cut into
// consecutive token ranges with its EMA state carried from range to range.
// Every part is one contiguous host range, so it moves with one
// cudaMemcpyAsync per direction.  Three side streams overlap the host-to-device
// copy of part k+1, the forward of part k (ossm_cheby_ema_fwd on device staging
// buffers) and the device-to-host copy of part k-1, on two staging buffers per
// direction; a PCIe link moves both directions at once.  Only the first part's
// copy in and the last part's copy out are not overlapped.  The initial states
// go in with one copy before the first part and the final states come out
// with one copy after the last, so no part pays for a small copy of its own.
//
// The side streams and their events are created once per device and shared by
// every call on that device; a mutex makes each call's enqueue atomic, so calls
// from several host threads are ordered, never interleaved.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "orthossm_b200.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kHeader = 256;  // the device forward's workspace header

struct Part {
  int b0, b1;  // sequences [b0, b1)
  int s0, s1;  // tokens [s0, s1) of each
};

// The parts for these arguments; identical in the size query and the call.
std::vector<Part> plan_parts(int B, int S, int pieces) {
  std::vector<Part> plan;
  const int want = std::max(1, pieces);
  if (B >= want) {
    for (int k = 0; k < want; ++k)
      plan.push_back({(int)((long long)B * k / want), (int)((long long)B * (k + 1) / want), 0, S});
  } else {
    const int q = std::max(1, std::min(S, (want + B - 1) / B));
    for (int b = 0; b < B; ++b)
      for (int j = 0; j < q; ++j)
        plan.push_back({b, b + 1, (int)((long long)S * j / q), (int)((long long)S * (j + 1) / q)});
  }
  return plan;
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// The arguments of one part's device forward: staging buffers for x, out,
// the initial and final state, the part's rows of the per-sequence device inputs.
ossm_fwd_args part_args(const ossm_fwd_args& a, const Part& p, void* x, void* out, const float* init, float* fin) {
  const long long D = (long long)a.H * a.head_dim;
  const int mb = p.b1 - p.b0, ms = p.s1 - p.s0;
  ossm_fwd_args r = a;
  // Every part runs on the three-pass kernels, whatever its number of
  // sequences, so the result does not depend on how the batch was cut (and
  // whole-sequence parts give bitwise the forward of the batch).  The call
  // is bound by the host link, not by the kernel.
  r.flags &= ~OSSM_F_SINGLE_EVAL;
  r.B = mb;
  r.S = ms;
  r.x = x;
  r.x_stride_s = D;
  r.x_stride_b = (long long)ms * D;
  r.out = out;
  r.out_stride_s = D;
  r.out_stride_b = (long long)ms * D;
  r.coeffs = a.coeffs + (size_t)p.b0 * a.H * a.degree * a.head_dim;
  r.lam_tok = a.lam_tok ? a.lam_tok + ((size_t)p.b0 * a.S + p.s0) * a.H : nullptr;
  r.init_state = init;
  r.final_state = fin;
  r.tanh_out = nullptr;
  return r;
}

struct HostLayout {
  std::vector<Part> plan;
  int big_b = 0, big_s = 0;
  size_t xbuf = 0, obuf = 0, sbuf = 0;  // bytes of one x / out / carried-state staging buffer
  size_t off_ws = 0, fws = 0;           // the device forward's workspace (first, header at offset 0)
  size_t off_x[2], off_o[2], off_c[2];  // per slot: x, out, state carried to the sequence's next part
  size_t off_init = 0, off_fin = 0;     // [B, D] f32: every initial state in, every final state out
  size_t total = 0;
};

int host_layout(const ossm_fwd_args* a, int pieces, HostLayout& l) {
  if (!a || pieces < 1) return OSSM_EINVAL;
  if (a->B < 1 || a->S < 1 || a->H < 1 || a->head_dim < 1) return OSSM_EINVAL;
  if (!a->x || !a->out || !a->coeffs || a->tanh_out) return OSSM_EINVAL;
  if ((a->x_dtype != OSSM_F32 && a->x_dtype != OSSM_BF16) || (a->out_dtype != OSSM_F32 && a->out_dtype != OSSM_BF16))
    return OSSM_EINVAL;
  const long long D = (long long)a->H * a->head_dim;
  // host activations contiguous [B, S, D]: every part is one contiguous range
  if (a->x_stride_s != D || a->out_stride_s != D) return OSSM_EINVAL;
  if (a->B > 1 && (a->x_stride_b != (long long)a->S * D || a->out_stride_b != (long long)a->S * D)) return OSSM_EINVAL;
  l.plan = plan_parts(a->B, a->S, pieces);
  for (const Part& p : l.plan) {
    l.big_b = std::max(l.big_b, p.b1 - p.b0);
    l.big_s = std::max(l.big_s, p.s1 - p.s0);
  }
  // The device forward's workspace comes first, sized for the largest need
  // of any part, so its header (launch counters, sticky status) sits at the
  // start of the caller's workspace, where ossm_workspace_status reads it.
  const uintptr_t fake = 1u << 20;  // dummy, suitably aligned device addresses: only the sizes matter here
  for (const Part& p : l.plan) {
    const ossm_fwd_args pa = part_args(*a, p, reinterpret_cast<void*>(fake), reinterpret_cast<void*>(fake),
                                       a->init_state ? reinterpret_cast<const float*>(fake) : nullptr,
                                       reinterpret_cast<float*>(fake));
    const size_t need = ossm_fwd_workspace_bytes(&pa);
    if (need == 0) return OSSM_EINVAL;
    l.fws = std::max(l.fws, al256(need));
  }
  const int xel = a->x_dtype == OSSM_F32 ? 4 : 2, oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  l.xbuf = al256((size_t)l.big_b * l.big_s * D * xel);
  l.obuf = al256((size_t)l.big_b * l.big_s * D * oel);
  l.sbuf = al256((size_t)l.big_b * D * 4);
  l.off_ws = 0;
  size_t off = l.fws;
  for (int i = 0; i < 2; ++i) {
    l.off_x[i] = off;
    off += l.xbuf;
    l.off_o[i] = off;
    off += l.obuf;
    l.off_c[i] = off;
    off += l.sbuf;
  }
  l.off_init = off;
  off += al256((size_t)a->B * D * 4);
  l.off_fin = off;
  off += al256((size_t)a->B * D * 4);
  l.total = off;
  return OSSM_OK;
}

struct SideStreams {
  std::mutex mu;
  bool ready = false;
  cudaStream_t s_in = nullptr, s_cmp = nullptr, s_out = nullptr;
  cudaEvent_t start = nullptr, ev_in[2] = {}, ev_cmp[2] = {}, ev_out[2] = {}, tail[3] = {};
};
SideStreams g_side[kMaxDevices];

cudaError_t side_setup(SideStreams& s) {
  if (s.ready) return cudaSuccess;
  cudaError_t e;
  for (cudaStream_t* p : {&s.s_in, &s.s_cmp, &s.s_out})
    if ((e = cudaStreamCreateWithFlags(p, cudaStreamNonBlocking)) != cudaSuccess) return e;
  std::vector<cudaEvent_t*> evs = {&s.start, &s.tail[0], &s.tail[1], &s.tail[2]};
  for (int i = 0; i < 2; ++i) {
    evs.push_back(&s.ev_in[i]);
    evs.push_back(&s.ev_cmp[i]);
    evs.push_back(&s.ev_out[i]);
  }
  for (cudaEvent_t* p : evs)
    if ((e = cudaEventCreateWithFlags(p, cudaEventDisableTiming)) != cudaSuccess) return e;
  s.ready = true;
  return cudaSuccess;
}

}  // namespace

extern "C" size_t ossm_fwd_host_workspace_bytes(const ossm_fwd_args* a, int pieces) {
  HostLayout l;
  return host_layout(a, pieces, l) == OSSM_OK ? l.total : 0;
}

extern "C" int ossm_cheby_ema_fwd_host(const ossm_fwd_args* a, int pieces, void* workspace, size_t workspace_bytes,
                                       ossm_stream_t stream) {
  HostLayout l;
  const int v = host_layout(a, pieces, l);
  if (v != OSSM_OK) return v;
  if (!workspace || workspace_bytes < l.total || ((uintptr_t)workspace % 256)) return OSSM_EWORKSPACE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return OSSM_ELAUNCH;
  if (dev >= kMaxDevices) return OSSM_EINVAL;
  SideStreams& ss = g_side[dev];
  std::lock_guard<std::mutex> lock(ss.mu);
  if (side_setup(ss) != cudaSuccess) return OSSM_ELAUNCH;

  cudaStream_t cur = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const long long D = (long long)a->H * a->head_dim;
  const size_t xel = a->x_dtype == OSSM_F32 ? 4 : 2, oel = a->out_dtype == OSSM_F32 ? 4 : 2;
  const char* xh = static_cast<const char*>(a->x);
  char* oh = static_cast<char*>(a->out);
  float* init_d = reinterpret_cast<float*>(ws + l.off_init);
  float* fin_d = reinterpret_cast<float*>(ws + l.off_fin);
  int rc = OSSM_OK;
  bool ok = cudaEventRecord(ss.start, cur) == cudaSuccess;
  for (cudaStream_t s : {ss.s_in, ss.s_cmp, ss.s_out}) ok = ok && cudaStreamWaitEvent(s, ss.start, 0) == cudaSuccess;
  // The forward's region past its header starts every call cleared: an
  // earlier call with another part plan may have left staging bytes there,
  // and the look-back flags of the generic kernel must start at zero.
  if (l.fws > kHeader) ok = ok && cudaMemsetAsync(ws + l.off_ws + kHeader, 0, l.fws - kHeader, ss.s_cmp) == cudaSuccess;
  // every initial state in one copy, ahead of the first part's activations
  if (a->init_state)
    ok = ok && cudaMemcpyAsync(init_d, a->init_state, (size_t)a->B * D * 4, cudaMemcpyHostToDevice, ss.s_in) ==
                   cudaSuccess;

  const int n = (int)l.plan.size();
  for (int k = 0; k < n && ok && rc == OSSM_OK; ++k) {
    const Part& p = l.plan[k];
    const int i = k & 1;
    const size_t rows = (size_t)p.b0 * a->S + p.s0;  // first host token row of the part
    const size_t ntok = (size_t)(p.b1 - p.b0) * (p.s1 - p.s0);
    char* xd = ws + l.off_x[i];
    char* od = ws + l.off_o[i];
    const bool cont = p.s0 > 0;      // the rest of the sequence the previous part began
    const bool last = p.s1 == a->S;  // the sequence's last part: its state goes to the final array
    // A part that does not end its sequence leaves its state in slot i's carry
    // buffer, where the sequence's next part (slot i ^ 1) starts from it.
    const float* init = cont ? reinterpret_cast<const float*>(ws + l.off_c[i ^ 1])
                             : (a->init_state ? init_d + (size_t)p.b0 * D : nullptr);
    float* fin = last ? fin_d + (size_t)p.b0 * D : reinterpret_cast<float*>(ws + l.off_c[i]);
    // copy in (staging buffers i were read by the forward of part k-2)
    if (k >= 2) ok = ok && cudaStreamWaitEvent(ss.s_in, ss.ev_cmp[i], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(xd, xh + rows * D * xel, ntok * D * xel, cudaMemcpyHostToDevice, ss.s_in) == cudaSuccess;
    ok = ok && cudaEventRecord(ss.ev_in[i], ss.s_in) == cudaSuccess;
    // forward (output buffer i was copied out after part k-2)
    ok = ok && cudaStreamWaitEvent(ss.s_cmp, ss.ev_in[i], 0) == cudaSuccess;
    if (k >= 2) ok = ok && cudaStreamWaitEvent(ss.s_cmp, ss.ev_out[i], 0) == cudaSuccess;
    if (!ok) break;
    const ossm_fwd_args pa = part_args(*a, p, xd, od, init, fin);
    rc = ossm_cheby_ema_fwd(&pa, ws + l.off_ws, l.fws, ss.s_cmp);
    if (rc != OSSM_OK) break;
    ok = ok && cudaEventRecord(ss.ev_cmp[i], ss.s_cmp) == cudaSuccess;
    // copy out
    ok = ok && cudaStreamWaitEvent(ss.s_out, ss.ev_cmp[i], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(oh + rows * D * oel, od, ntok * D * oel, cudaMemcpyDeviceToHost, ss.s_out) == cudaSuccess;
    ok = ok && cudaEventRecord(ss.ev_out[i], ss.s_out) == cudaSuccess;
  }
  // every final state in one copy: the forwards run in order on one stream,
  // and the copy-out stream has waited for the last of them
  if (ok && rc == OSSM_OK && a->final_state)
    ok = cudaMemcpyAsync(a->final_state, fin_d, (size_t)a->B * D * 4, cudaMemcpyDeviceToHost, ss.s_out) == cudaSuccess;
  // the caller's stream waits for everything enqueued on the side streams,
  // also after an error, so later work on it never overlaps this call's
  cudaStream_t sides[3] = {ss.s_in, ss.s_cmp, ss.s_out};
  for (int j = 0; j < 3; ++j) {
    const bool t = cudaEventRecord(ss.tail[j], sides[j]) == cudaSuccess &&
                   cudaStreamWaitEvent(cur, ss.tail[j], 0) == cudaSuccess;
    ok = ok && t;
  }
  if (rc != OSSM_OK) return rc;
  return ok ? OSSM_OK : OSSM_ELAUNCH;
}
