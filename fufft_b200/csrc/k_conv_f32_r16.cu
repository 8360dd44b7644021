// kernel family: conv_f32_r16 (fp32 fused convolution, radix-16 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_conv_f32_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_conv<16, false>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
