// kernel family: apply_r8 (split apply, radix-8 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_apply_r8(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_apply<8, Out::C32>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
