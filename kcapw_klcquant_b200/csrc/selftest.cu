// Self-test of the bounded mbarrier wait every tensor-core kernel uses.
//
// One CTA initialises an mbarrier that nothing ever arrives on and waits for
// its first phase with the given cycle limit; the wait gives up, records
// KLC_ERR_DEVICE_TIMEOUT (site 999) in a status word and the kernel returns,
// leaving the context usable.  Lets a deployment check, without faulting or
// hanging a GPU, that an expired wait is reported instead of hanging.
#include "tc_common.cuh"

namespace klc {
namespace {

__device__ DeviceStatus g_selftest_status;

__global__ void wait_selftest_kernel(long long limit) {
  using namespace tc;
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const Ctl ctl{reinterpret_cast<volatile int*>(&abort_flag), &g_selftest_status};
  if (threadIdx.x == 0) wait_bar_limit(smem_u32(&bar), 0, ctl, 999, limit);  // nothing ever arrives
  __syncthreads();
}

}  // namespace
}  // namespace klc

extern "C" int klc_selftest_wait_timeout(int64_t limit_cycles, int* code, int* where, void* stream) {
  using namespace klc;
  KLC_CHECK_ARG(limit_cycles > 0 && limit_cycles <= (int64_t(1) << 32), "klc_selftest_wait_timeout: limit out of range");
  const DeviceStatus zero{};
  KLC_CUDA(cudaMemcpyToSymbolAsync(g_selftest_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, as_stream(stream)));
  wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(static_cast<long long>(limit_cycles));
  KLC_LAUNCH_CHECK("klc_selftest_wait_timeout launch");
  DeviceStatus st{};
  KLC_CUDA(cudaMemcpyFromSymbolAsync(&st, g_selftest_status, sizeof(st), 0, cudaMemcpyDeviceToHost, as_stream(stream)));
  KLC_CUDA(cudaStreamSynchronize(as_stream(stream)));
  if (code) *code = st.code;
  if (where) *where = st.where;
  return KLC_OK;
}
