// Tensor-core (tcgen05) path of the wide matmul: not yet enabled; every
// problem goes to the exact CUDA-core kernel.
#include "sfb_wide_simt.cuh"

namespace sfb {

int64_t wide_tc_workspace(int, int, int64_t, int64_t, int64_t, int64_t) { return 0; }

int wide_tc_try(int, int, const int16_t *, const int16_t *, const int8_t *, int, int16_t *, uint8_t *, int64_t,
                int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                void *, int64_t, sfb_counts *, cudaStream_t, bool *handled) {
    *handled = false;
    return SFB_OK;
}

}  // namespace sfb
