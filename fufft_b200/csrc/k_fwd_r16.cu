// kernel family: fwd_r16 (split forward, radix-16 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_fwd_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   (void)mid;
   return dispatch_fwd<16, In::C32>(n, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
