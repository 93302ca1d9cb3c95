// tcgen05 grouped expert GEMM (placeholder until the tensor-core path lands).
#include "permute.cuh"

namespace klc {

bool tc_path_supported(int64_t, int64_t) { return false; }

int launch_experts_tc(const ExpertArgs&, cudaStream_t) {
  return fail(KLC_ERR_UNSUPPORTED, "tensor-core expert path not built");
}

}  // namespace klc
