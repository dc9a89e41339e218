// conv_tc.cu -- placeholder until the tcgen05 kernel lands: every conv takes the CUDA-core path.
#include "conv_tc.cuh"

namespace uq {

struct ConvTc {};

int conv_tc_prepare(const int8_t *, const int32_t *, const uint8_t *, const ConvGeom &,
                    const std::function<void *(size_t)> &, ConvTc **out) {
    *out = nullptr;
    return 0;
}
void conv_tc_launch(const ConvTc &, const int8_t *, int8_t *, const ConvGeom &, cudaStream_t) {}
void conv_tc_free(ConvTc *c) { delete c; }

}  // namespace uq
