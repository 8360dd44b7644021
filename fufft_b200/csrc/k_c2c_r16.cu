// kernel family: c2c_r16 (natural-order transform, radix-16 chain).  Instantiations of the fused engine
// (fufft_conv.cuh) with the spectrum scattered to natural order at the register boundary.
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
fufft_status family_c2c_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   (void)mid; (void)bperm;
   return launch_n<16, In::C32, Out::NAT, Mid::NONE, Flt::NONE, false>(n, a, st, dev);
}
}  // namespace host
}  // namespace fufft
