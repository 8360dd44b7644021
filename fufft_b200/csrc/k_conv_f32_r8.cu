// kernel family: conv_f32_r8 (fp32 fused convolution, radix-8 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_conv_f32_r8(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_conv<8, false>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
