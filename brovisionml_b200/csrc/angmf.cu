// AngMF launch entry point: inputs already activated (prob in [0, 1], angle in
// radians), as brovisionml's angmf_propagate takes them
// (include/brovisionml/dsine_ops.h:28-54). Raw head outputs go to
// angmf_logits.cu. The kernels live in angmf_kernels.cuh.
#include "angmf_kernels.cuh"

namespace bvml {

cudaError_t launch_angmf(const AngmfLaunch& L, cudaStream_t s) {
    if (L.act) return launch_angmf_logits(L, s);
    return launch_angmf_act<false>(L, s);
}

cudaError_t launch_angmf_iters(const AngmfItersLaunch& L, cudaStream_t s) {
    if (L.act) return launch_angmf_iters_logits(L, s);
    return launch_angmf_iters_act<false>(L, s);
}

BVML_CHECK_READER(check_word_angmf)

}  // namespace bvml
