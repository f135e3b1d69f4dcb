// Failure-injection instances of the tensor-core attention kernel: the same
// code as the default instances, except that every pipeline wait gives up
// after TcParams::wait_limit mbarrier probes instead of the compile-time
// bound (a runtime bound in the default instances' hot loops measured ~3 us
// slower per launch). Launched only while tlb_attention_set_wait_limit holds a
// limit other than the default, by the tests of the bounded waits.
#include "paged_attention_tc.cuh"

namespace tlb {
namespace attn {

cudaError_t launch_tc_inject(int dtype, int head_dim, int group, const TcParams& p,
                             const CUtensorMap& tm_k, const CUtensorMap& tm_v, int grid,
                             bool overlap, cudaStream_t stream) {
    if (dtype == TLB_BFLOAT16)
        return dispatch_tc<__nv_bfloat16, true>(head_dim, group, p, tm_k, tm_v, grid, overlap,
                                                 stream);
    return dispatch_tc<__half, true>(head_dim, group, p, tm_k, tm_v, grid, overlap, stream);
}

}  // namespace attn
}  // namespace tlb
