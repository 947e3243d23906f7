// jk_gemm_fmt_f16.cu -- the tensor-core product's kernels for FP16 weights (every activation type,
// row tile, CTA pairing and schedule), instantiated from jk_gemm_sm100.cuh.
#include "jk_gemm_sm100.cuh"

namespace jk {
namespace tc {

jk_status launch_f16(const LaunchArgs& a, int bt, bool bf16) {
    return bf16 ? launch_tc_bt<FMT_F16, true>(a, bt) : launch_tc_bt<FMT_F16, false>(a, bt);
}

}  // namespace tc
}  // namespace jk
