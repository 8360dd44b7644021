// kernel family: fp32 fused convolution with an int16-BFP filter (the middle
// of the BFP four-step), radix-16 chain.  Instantiations of fufft_conv.cuh.
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_mid_bfpfilter_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_mid<16, In::C32, Out::C32, true>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
