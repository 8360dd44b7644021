// kernel family: r2_r16 (two-for-one real convolution, radix-16 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
// chain-order filters (mixedrev16) of n >= 512: staged per warp through the
// exchange buffer (Flt::LIN_STAGED), as the complex convolution does.
// Measured on B200 (2^28 real points, per-transform filters, % of HBM, staged
// / 128 contiguous bytes per thread from global memory): 1024: 85 / 71,
// 2048: 81 / 57, 4096: 80 / 54
#ifndef FUFFT_R2_LIN_STAGED
#define FUFFT_R2_LIN_STAGED 1
#endif
fufft_status family_r2_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(FUFFT_R2_LIN_STAGED && !bperm && mid != FUFFT_MID_NONE && n >= 512 && n <= MAX_N_R16 && aligned(a.b, 16) &&
      (a.filter_stride * 8) % 16 == 0)
      return mid == FUFFT_MID_MULTIPLY ? launch_lin_staged<16, In::REAL2, Out::REAL2, Mid::MUL>(n, a, st, dev)
                                       : launch_lin_staged<16, In::REAL2, Out::REAL2, Mid::CONJ>(n, a, st, dev);
   return dispatch_mid<16, In::REAL2, Out::REAL2, false>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
