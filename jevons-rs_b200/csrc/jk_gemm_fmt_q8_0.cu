// jk_gemm_fmt_q8_0.cu -- the tensor-core product's kernels for Q8_0 weights (every activation type,
// row tile, CTA pairing and schedule), instantiated from jk_gemm_sm100.cuh.
#include "jk_gemm_sm100.cuh"

namespace jk {
namespace tc {

jk_status launch_q8_0(const LaunchArgs& a, int bt, bool bf16) {
    return bf16 ? launch_tc_bt<FMT_Q8_0, true>(a, bt) : launch_tc_bt<FMT_Q8_0, false>(a, bt);
}

}  // namespace tc
}  // namespace jk
