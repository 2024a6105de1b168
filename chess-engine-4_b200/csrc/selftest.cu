// Self-test of the bounded device waits: a kernel that waits for something that never
// happens must give up after its limit, record the code in the device error word and
// return, leaving the context usable. The forward's kernels rely on this to turn a lost
// dependency or a stuck pipeline stage into an error status instead of a hang.
#include "forward_types.h"
#include "ptx.cuh"
#include "internal.h"

namespace ce4b {

namespace {

// A counter nothing publishes to (the never-arriving dependency), and the measured wait.
__device__ int g_selftest_counter;
__device__ unsigned long long g_selftest_waited;

// One thread. kind 0: wait_counter on g_selftest_counter for a value it never reaches (the
// persistent forward's cross-CTA dependency wait); kind 1: mbar_wait on a shared-memory
// mbarrier that expects one arrival which never comes (a pipeline-stage wait). On timeout
// the kernel records `code` and the measured wait in ns.
__global__ void bounded_wait_kernel(int kind, unsigned long long limit_ns, int code, int* err,
                                    unsigned long long* waited_ns) {
  __shared__ alignas(8) unsigned long long bar_storage;
  const unsigned long long start = global_timer_ns();
  bool ok;
  if (kind == 0) {
    ok = wait_counter(&g_selftest_counter, 1, limit_ns);
  } else {
    const uint32_t bar = smem_u32(&bar_storage);
    mbar_init(bar, 1);
    fence_mbar_init();
    ok = mbar_wait(bar, 0, limit_ns);
  }
  *waited_ns = global_timer_ns() - start;
  if (!ok) record_error(err, code);
}

}  // namespace

}  // namespace ce4b

using namespace ce4b;

extern "C" int ce4b_selftest_bounded_wait(int kind, long long limit_ns, long long* waited_ns,
                                          void* stream) {
  try {
    require(kind == 0 || kind == 1, "kind must be 0 (counter) or 1 (mbarrier)");
    require(limit_ns > 0 && limit_ns <= 100ll * 1000 * 1000, "limit must be in (0, 100 ms]");
    require(waited_ns != nullptr, "null waited_ns");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* counter = nullptr;
    check_cuda(cudaGetSymbolAddress(reinterpret_cast<void**>(&counter), g_selftest_counter),
               "cudaGetSymbolAddress(selftest counter)");
    check_cuda(cudaMemsetAsync(counter, 0, sizeof(int), s), "clear selftest counter");
    unsigned long long* slot = nullptr;
    check_cuda(cudaGetSymbolAddress(reinterpret_cast<void**>(&slot), g_selftest_waited),
               "cudaGetSymbolAddress(selftest wait)");
    bounded_wait_kernel<<<1, 1, 0, s>>>(kind, static_cast<unsigned long long>(limit_ns),
                                        kind == 0 ? kErrTimeoutDependency : kErrTimeoutProducer,
                                        device_error_word(), slot);
    check_cuda(cudaGetLastError(), "bounded wait launch");
    unsigned long long host_waited = 0;
    check_cuda(cudaMemcpyAsync(&host_waited, slot, sizeof(host_waited), cudaMemcpyDeviceToHost, s),
               "read measured wait");
    check_cuda(cudaStreamSynchronize(s), "bounded wait");
    *waited_ns = static_cast<long long>(host_waited);
    return CE4B_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.status;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return CE4B_ERR_INVALID_ARGUMENT;
  } catch (...) {
    set_last_error("unknown error");
    return CE4B_ERR_INVALID_ARGUMENT;
  }
}
