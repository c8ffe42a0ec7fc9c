// tcgen05 GEMM instantiations for tile width 128 (see gemm_sm100.cu).
#include "gemm_kernel.cuh"

namespace sb {
namespace gemm {

void dispatch_bn128(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                    const CUtensorMap& td2, const Params& p, int hint, cudaStream_t stream) {
  if (!a_mn && !b_mn) launch<128, false, false>(ta, tb, td, td2, p, hint, stream);
  else if (!a_mn && b_mn) launch<128, false, true>(ta, tb, td, td2, p, hint, stream);
  else if (a_mn && b_mn) launch<128, true, true>(ta, tb, td, td2, p, hint, stream);
  else TORCH_CHECK(false, "gemm: unsupported major combination (A MN-major, B K-major)");
}

}  // namespace gemm
}  // namespace sb
