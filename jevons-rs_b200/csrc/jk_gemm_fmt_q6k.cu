// jk_gemm_fmt_q6k.cu -- the tensor-core product's kernels for Q6_K weights (every activation type,
// row tile, CTA pairing and schedule), instantiated from jk_gemm_sm100.cuh.
#include "jk_gemm_sm100.cuh"

namespace jk {
namespace tc {

jk_status launch_q6k(const LaunchArgs& a, int bt, bool bf16) {
    return bf16 ? launch_tc_bt<FMT_Q6K, true>(a, bt) : launch_tc_bt<FMT_Q6K, false>(a, bt);
}

}  // namespace tc
}  // namespace jk
