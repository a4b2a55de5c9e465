// AngMF on the prediction heads' raw outputs: prob = sigmoid(prob_logit) and
// angle = pi * sigmoid(angle_logit) are applied while the kernel loads them
// (src/dsine_refine.cpp:262-267 does them as separate passes). Same kernels
// as angmf.cu (angmf_kernels.cuh), instantiated here so the two halves
// compile in parallel.
#include "angmf_kernels.cuh"

namespace bvml {

cudaError_t launch_angmf_logits(const AngmfLaunch& L, cudaStream_t s) {
    return launch_angmf_act<true>(L, s);
}

cudaError_t launch_angmf_iters_logits(const AngmfItersLaunch& L, cudaStream_t s) {
    return launch_angmf_iters_act<true>(L, s);
}

BVML_CHECK_READER(check_word_angmf_logits)

}  // namespace bvml
