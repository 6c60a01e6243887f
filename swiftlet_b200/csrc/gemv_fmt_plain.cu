// Instantiates the weight-streaming kernels for one family of weight formats.
#include "slice_impl.cuh"

namespace swl {
SWL_INSTANTIATE_FORMAT(0, DT_F32)
SWL_INSTANTIATE_SLICE(0, DT_F32)
SWL_INSTANTIATE_FORMAT(0, DT_BF16)
SWL_INSTANTIATE_SLICE(0, DT_BF16)
SWL_INSTANTIATE_FORMAT(0, DT_F16)
SWL_INSTANTIATE_SLICE(0, DT_F16)
}  // namespace swl
