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

fufft_status family_conv2d_r8(int h, int w, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
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
