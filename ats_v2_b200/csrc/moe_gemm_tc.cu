// tcgen05 / TMEM grouped GEMMs for the bf16 SwiGLU experts (sm_100a).
#include "moe_gemm.cuh"

namespace ats {

int tc_experts_fwd(const void*, const void*, const void*, void*, void*, void*, int, int64_t, int64_t,
                   const MoePlan&, cudaStream_t) {
  return ATS_EUNSUPPORTED;
}

int tc_experts_bwd(const void*, const void*, const void*, const void*, const void*, const void*, void*, void*,
                   void*, void*, int, int64_t, int64_t, const MoePlan&, cudaStream_t) {
  return ATS_EUNSUPPORTED;
}

}  // namespace ats
