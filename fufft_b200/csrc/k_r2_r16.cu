// kernel family: r2_r16 (two-for-one real convolution, radix-16 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_r2_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_mid<16, In::REAL2, Out::REAL2, false>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
