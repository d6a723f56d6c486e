// Device-side error reporting for bounded waits.
//
// A kernel that spins on an mbarrier (or any flag) counts its polls; when the
// count passes the limit it records a code in g_device_error and returns
// instead of spinning on, so the context stays usable and the host can turn
// the code into an error (tileops_device_error_flag).  Codes:
#pragma once

namespace tileops {

constexpr int kErrMbarTimeout = 1;  // an mbarrier wait exceeded its poll limit
constexpr int kErrBadSeqlens = 2;   // cu_seqlens not 0 = cu[0] <= ... <= cu[N] = total

// Device address of the per-device error word (defined in capi.cu).  Kernels
// receive it as an argument: each translation unit is a separate module, so
// the symbol is resolved on the host once per device.
int* device_error_ptr();

__device__ __forceinline__ void report_device_error(int* flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

}  // namespace tileops
