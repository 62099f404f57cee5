// cf_conv_tp2.cu — instantiates the fused conv kernels for time blocks of
// 2 steps (all residual modes, both LIF forms, both kernel variants).
#define CF_CONV_INSTANTIATE 1
#include "cf_conv_kernels.cuh"

namespace cf {
namespace convk {
template int dispatch_res<2>(int, bool, const CUtensorMap&, const CUtensorMap&,
                               const ConvArgs&, int, cudaStream_t);
}  // namespace convk
}  // namespace cf
