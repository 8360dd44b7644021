// kernel family: fused 2-D convolution (rows x cols in one CTA), radix-8 chains.
// Instantiations of the fused engine (fufft_conv.cuh) over Chain2<H, W, 8>.
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
template<Mid MID, Flt FLT>
static fufft_status conv2d_shape(int h, int w, const ConvArgs& a, cudaStream_t st, int dev)
{
#define FUFFT_2D(HH, WW) \
   if(h == HH && w == WW) return launch_chain<Chain2<HH, WW, 8>, In::C32, Out::C32, MID, FLT, false>(a, st, dev);
   FUFFT_2D(8, 8)
   FUFFT_2D(8, 16)
   FUFFT_2D(8, 32)
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 256)
   FUFFT_2D(8, 512)
   FUFFT_2D(16, 8)
   FUFFT_2D(16, 16)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 128)
   FUFFT_2D(16, 256)
   FUFFT_2D(32, 8)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 64)
   FUFFT_2D(32, 128)
   FUFFT_2D(64, 8)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 32)
   FUFFT_2D(64, 64)
   FUFFT_2D(128, 8)
   FUFFT_2D(128, 16)
   FUFFT_2D(128, 32)
   FUFFT_2D(256, 8)
   FUFFT_2D(256, 16)
   FUFFT_2D(512, 8)
#undef FUFFT_2D
   return FUFFT_ERR_INVALID_SIZE;
}

// The reference's 2-D filter order (slot (r, c) = spectrum(rev8_H(r),
// rev8_W(c)), verify_kernel.cpp:738-748) on the radix-16 engine, the filter
// staged per warp through the bit permutation (R8Perm), for images of
// n = 2^k points with bit k of the mask and rows of 16 or more.  Measured on
// B200 (1 GiB, per-image / shared filter, radix-16 / radix-8 engine, the two
// builds interleaved kernel by kernel): 64x64 72 / 52%, 50 / 36%; 8x512 77 /
// 48%; 16x256 91 / 43%; 32x128 68 / 45%; 16x64 76 / 63%; 16x32 91 / 56%;
// 8x64 even.  2048-point images spill at the three-CTA target (76-136 bytes)
// and measured 12-21% slower: they stay on the radix-8 engine.
#ifndef FUFFT_2D_R8_ON_R16
#define FUFFT_2D_R8_ON_R16 ((1 << 9) | (1 << 10) | (1 << 12))
#endif
template<Mid MID, Flt FLT>
static fufft_status conv2d_on_r16(int h, int w, const ConvArgs& a, cudaStream_t st, int dev)
{
#define FUFFT_2D(HH, WW) \
   if(h == HH && w == WW) return launch_chain<Chain2<HH, WW, 16>, In::C32, Out::C32, MID, FLT, false>(a, st, dev);
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 512)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 256)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 128)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 64)
   FUFFT_2D(128, 32)
   FUFFT_2D(256, 16)
#undef FUFFT_2D
   return FUFFT_ERR_UNSUPPORTED;
}

fufft_status family_conv2d_r8(int h, int w, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(mid != FUFFT_MID_NONE && w >= 16 && in_mask(FUFFT_2D_R8_ON_R16, h * w) && aligned(a.b, 16) &&
      (a.filter_stride * 8) % 16 == 0) {
      const bool mul = mid == FUFFT_MID_MULTIPLY;
      const fufft_status s = bperm ? (mul ? conv2d_on_r16<Mid::MUL, R8BP_FLT>(h, w, a, st, dev)
                                          : conv2d_on_r16<Mid::CONJ, R8BP_FLT>(h, w, a, st, dev))
                                   : (mul ? conv2d_on_r16<Mid::MUL, Flt::R8_STAGED>(h, w, a, st, dev)
                                          : conv2d_on_r16<Mid::CONJ, Flt::R8_STAGED>(h, w, a, st, dev));
      if(s != FUFFT_ERR_UNSUPPORTED) return s;
   }
   switch(mid) {
   case FUFFT_MID_NONE: return conv2d_shape<Mid::NONE, Flt::NONE>(h, w, a, st, dev);
   case FUFFT_MID_MULTIPLY:
      return bperm ? conv2d_shape<Mid::MUL, Flt::SMEM>(h, w, a, st, dev) : conv2d_shape<Mid::MUL, Flt::GLOBAL>(h, w, a, st, dev);
   case FUFFT_MID_CONJ_MULTIPLY:
      return bperm ? conv2d_shape<Mid::CONJ, Flt::SMEM>(h, w, a, st, dev) : conv2d_shape<Mid::CONJ, Flt::GLOBAL>(h, w, a, st, dev);
   }
   return FUFFT_ERR_INVALID_ARG;
}
// the shapes this build instantiates
bool conv2d_supported_r8(int h, int w)
{
#define FUFFT_2D(HH, WW) if(h == HH && w == WW) return true;
   FUFFT_2D(8, 8)
   FUFFT_2D(8, 16)
   FUFFT_2D(8, 32)
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 256)
   FUFFT_2D(8, 512)
   FUFFT_2D(16, 8)
   FUFFT_2D(16, 16)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 128)
   FUFFT_2D(16, 256)
   FUFFT_2D(32, 8)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 64)
   FUFFT_2D(32, 128)
   FUFFT_2D(64, 8)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 32)
   FUFFT_2D(64, 64)
   FUFFT_2D(128, 8)
   FUFFT_2D(128, 16)
   FUFFT_2D(128, 32)
   FUFFT_2D(256, 8)
   FUFFT_2D(256, 16)
   FUFFT_2D(512, 8)
#undef FUFFT_2D
   return false;
}
}  // namespace host
}  // namespace fufft
