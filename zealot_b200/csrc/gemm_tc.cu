// gemm_tc.cu -- tcgen05 tensor-core GEMMs (tf32 / bf16, fp32 accumulate).
#include <cuda_runtime.h>

#include "zrl_gemm.h"

namespace zrl {

zrl_status gemm_tc_init(int, std::string *err) {
  *err = "tensor-core GEMM not built yet";
  return ZRL_NOT_SUPPORTED;
}

zrl_status gemm_tc(const GemmArgs &, int, cudaStream_t, int *launched,
                   std::string *err) {
  *launched = 0;
  *err = "tensor-core GEMM not built yet";
  return ZRL_NOT_SUPPORTED;
}

}  // namespace zrl
