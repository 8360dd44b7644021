// kernel family: r2_r8 (two-for-one real convolution, radix-8 chain).  Instantiations of the fused engine (fufft_conv.cuh).
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
// the reference's two-for-one filter layout is the radix-8 chain order
// (verify_kernel.cpp:580): at n >= 1024 the radix-16 engine reads it through
// the per-warp bit-permutation staging (Flt::R8_STAGED / R8BP_STAGED).
// Measured on B200 (2^28 real points, per-transform filters, median of three
// interleaved runs, % of HBM at 24 B per complex slot, radix-16 / radix-8
// engine): R8 1024: 81 / 70, 2048: 77 / 61, 4096: 75 / 41; R8_BPERM 2048:
// 69 / 59, 4096: 71 / 48
#ifndef FUFFT_R2_R8_ON_R16_LIN
#define FUFFT_R2_R8_ON_R16_LIN ((1 << 10) | (1 << 11) | (1 << 12))
#endif
#ifndef FUFFT_R2_R8_ON_R16_BP
#define FUFFT_R2_R8_ON_R16_BP ((1 << 11) | (1 << 12))
#endif
fufft_status family_r2_r8(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   const fufft_status s = dispatch_r8_on_r16<In::REAL2, Out::REAL2, FUFFT_R2_R8_ON_R16_LIN, FUFFT_R2_R8_ON_R16_BP>(
      n, mid, bperm, a, st, dev);
   if(s != FUFFT_ERR_UNSUPPORTED) return s;
   return dispatch_mid<8, In::REAL2, Out::REAL2, false>(n, mid, bperm, a, st, dev);
}
}  // namespace host
}  // namespace fufft
