// cf_conv_tp4.cu — instantiates the fused conv kernels for time blocks of
// 4 steps (all residual modes, both LIF forms, both kernel variants).
#define CF_CONV_INSTANTIATE 1
#include "cf_conv_kernels.cuh"

namespace cf {
namespace convk {
template int dispatch_res<4>(int, bool, const CUtensorMap&, const CUtensorMap&,
                               const ConvArgs&, int, cudaStream_t);
}  // namespace convk
}  // namespace cf
