// Library metadata entry points of the orthossm_b200 C ABI.
#include "orthossm_b200.h"

extern "C" const char* ossm_version(void) { return "orthossm_b200 0.1.0 (sm_100a)"; }

extern "C" const char* ossm_status_string(int status) {
  switch (status) {
    case OSSM_OK: return "ok";
    case OSSM_EINVAL: return "invalid argument (shape, pointer, alignment or flag)";
    case OSSM_ELAUNCH: return "CUDA launch or runtime error";
    case OSSM_ETIMEOUT: return "a bounded device-side wait timed out";
    case OSSM_ECOMM: return "multi-GPU exchange error";
    case OSSM_EWORKSPACE: return "workspace missing, misaligned or too small";
    default: return "unknown status";
  }
}

extern "C" size_t ossm_sizeof_fwd_args(void) { return sizeof(ossm_fwd_args); }
extern "C" size_t ossm_sizeof_lion_args(void) { return sizeof(ossm_lion_args); }
extern "C" size_t ossm_sizeof_ttt_args(void) { return sizeof(ossm_ttt_args); }
extern "C" size_t ossm_sizeof_bwd_args(void) { return sizeof(ossm_bwd_args); }
extern "C" size_t ossm_sizeof_ttt_run_args(void) { return sizeof(ossm_ttt_run_args); }
