// Tensor-core (tcgen05) TurboQuant compress for head_dim 128.
#include "common.cuh"
#include "tq_common.cuh"

namespace fb {

int tq_compress_umma(const TqArgs& a, cudaStream_t s, bool* handled) {
    (void)a;
    (void)s;
    *handled = false;
    return 0;
}

}  // namespace fb
