// kernel family: apply_r2_r16 (split apply with real-pair output, radix-16 chain).  Instantiations of the
// fused engine (fufft_conv.cuh): the spectrum of a packed pair xr + i*yr times a real filter's spectrum,
// inverse transform, re -> ur and im -> vr.
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_apply_r2_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   return dispatch_apply<16, Out::REAL2>(n, mid, bperm, a, st, dev);
}
fufft_status family_fwd_r2_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   (void)mid;
   return dispatch_fwd<16, In::REAL2>(n, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
