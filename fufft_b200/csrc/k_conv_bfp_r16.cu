// kernel family: conv_bfp_r16 (int16 BFP fused convolution, radix-16 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_conv_bfp_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_conv<16, true>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
