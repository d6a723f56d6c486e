// Self-test of the give-up path the tensor-core kernels of this library take
// when a wait runs out: a one-warp kernel that holds the same resources a real
// kernel holds when a wait gives up -- TMEM columns and a bulk copy in flight
// -- waits on an mbarrier that nothing ever arrives on, and must then do what
// the kernels do: record kErrMbarTimeout in the device error word, let its
// own copy land (a drain wait), free TMEM and return.  Its waits are
// sm100::mbar_wait_polled (test_wait polls against the global timer), which
// always end; nothing here can hang.
#include "common.cuh"
#include "device_error.cuh"
#include "sm100.cuh"

namespace tileops {
namespace {

constexpr int kSelftestMaxBytes = 4096;

struct SelftestSmem {
  alignas(128) uint8_t buf[kSelftestMaxBytes];
  alignas(8) uint64_t copy_bar;
  alignas(8) uint64_t never_bar;
  uint32_t tmem_base;
  int abort_flag;
};

// out[0] = 1 if the unarmed wait gave up, out[1] = 1 if the drain saw the copy
// land, out[2] = the sum of the copied bytes (proves the data arrived before
// the CTA read it), out[3] = 1 once TMEM was released, out[4] / out[5] = low /
// high 32 bits of the nanoseconds the unarmed wait took before giving up.
__global__ void __launch_bounds__(32, 1)
    selftest_wait_timeout_kernel(const uint8_t* __restrict__ src, int bytes, uint64_t limit_ns,
                                 int* __restrict__ out, int* err) {
  __shared__ SelftestSmem sm;
  const int lane = threadIdx.x;
  if (lane == 0) {
    sm.abort_flag = 0;
    sm100::mbar_init(&sm.copy_bar, 1);
    sm100::mbar_init(&sm.never_bar, 1);
    sm100::fence_mbar_init();
  }
  __syncwarp();
  sm100::tmem_alloc(&sm.tmem_base, 32);
  sm100::tmem_relinquish();
  sm100::tc_fence_before();
  __syncwarp();
  sm100::tc_fence_after();

  int landed = 0;
  if (lane == 0) {
    sm100::mbar_arrive_expect_tx(&sm.copy_bar, static_cast<uint32_t>(bytes));
    sm100::bulk_load(sm.buf, src, static_cast<uint32_t>(bytes), &sm.copy_bar);
    // Nothing arrives on never_bar: this wait must give up after limit_ns.
    const uint64_t t0 = sm100::globaltimer_ns();
    const bool got =
        sm100::mbar_wait_polled(&sm.never_bar, 0, err, &sm.abort_flag, false, limit_ns);
    const uint64_t waited = sm100::globaltimer_ns() - t0;
    out[0] = got ? 0 : 1;
    out[4] = static_cast<int>(waited & 0xffffffffu);
    out[5] = static_cast<int>(waited >> 32);
    // The give-up path: the copy issued above still targets shared memory, so
    // wait for it (ignoring the abort flag) before the CTA may exit.
    landed = sm100::mbar_wait_polled(&sm.copy_bar, 0, err, &sm.abort_flag, true) ? 1 : 0;
    out[1] = landed;
  }
  landed = __shfl_sync(0xffffffffu, landed, 0);
  int sum = 0;
  if (landed) {
    for (int i = lane; i < bytes; i += 32) sum += sm.buf[i];
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  sm100::tc_fence_before();
  __syncwarp();
  sm100::tc_fence_after();
  sm100::tmem_dealloc(sm.tmem_base, 32);
  if (lane == 0) {
    out[2] = sum;
    out[3] = 1;
  }
}

}  // namespace
}  // namespace tileops

extern "C" int tileops_selftest_wait_timeout(const void* src, int64_t bytes, int64_t limit_ns,
                                             int* out, void* stream) {
  using namespace tileops;
  if (!src || !out) return TILEOPS_EINVAL;
  if (bytes <= 0 || bytes > kSelftestMaxBytes || bytes % 16 != 0) return TILEOPS_EBADSHAPE;
  if (reinterpret_cast<uintptr_t>(src) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 4 != 0)
    return TILEOPS_EALIGN;
  if (limit_ns < 1000 || limit_ns > 1000000000) return TILEOPS_EBADSHAPE;
  int* err = device_error_ptr();
  if (!err) return TILEOPS_ELAUNCH;
  selftest_wait_timeout_kernel<<<1, 32, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(src), static_cast<int>(bytes),
      static_cast<uint64_t>(limit_ns), out, err);
  return cudaGetLastError() == cudaSuccess ? TILEOPS_OK : TILEOPS_ELAUNCH;
}
