// cf_conv_tp1.cu — instantiates the fused conv kernels for time blocks of
// 1 step (all residual modes, both LIF forms, both kernel variants).
#define CF_CONV_INSTANTIATE 1
#include "cf_conv_kernels.cuh"

namespace cf {
namespace convk {
template int dispatch_res<1>(int, bool, const CUtensorMap&, const CUtensorMap&,
                               const ConvArgs&, int, cudaStream_t);
}  // namespace convk
}  // namespace cf
