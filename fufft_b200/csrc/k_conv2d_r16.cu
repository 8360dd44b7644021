// kernel family: fused 2-D convolution (rows x cols in one CTA), radix-16 chains.
// Instantiations of the fused engine (fufft_conv.cuh) over Chain2<H, W, 16>.
#include "fufft_internal.cuh"
namespace fufft {
namespace host {
template<Mid MID, Flt FLT>
static fufft_status conv2d_shape(int h, int w, const ConvArgs& a, cudaStream_t st, int dev)
{
#define FUFFT_2D(HH, WW) \
   if(h == HH && w == WW) return launch_chain<Chain2<HH, WW, 16>, In::C32, Out::C32, MID, FLT, false>(a, st, dev);
   FUFFT_2D(8, 16)
   FUFFT_2D(8, 32)
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 256)
   FUFFT_2D(8, 512)
   FUFFT_2D(8, 1024)
   FUFFT_2D(16, 16)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 128)
   FUFFT_2D(16, 256)
   FUFFT_2D(16, 512)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 64)
   FUFFT_2D(32, 128)
   FUFFT_2D(32, 256)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 32)
   FUFFT_2D(64, 64)
   FUFFT_2D(64, 128)
   FUFFT_2D(128, 16)
   FUFFT_2D(128, 32)
   FUFFT_2D(128, 64)
   FUFFT_2D(256, 16)
   FUFFT_2D(256, 32)
   FUFFT_2D(512, 16)
#undef FUFFT_2D
   return FUFFT_ERR_INVALID_SIZE;
}

// 4096-point images with rows of 64 or more: the register-boundary filter read
// straight from global memory at the boundary (coalesced; no shared-memory
// filter tile, so three CTAs per SM fit), as the 1-D radix-16 kernels do.
// Measured on B200 (1 GiB batches, A/B against the TMA-staged tile): 64x64
// +6%, 32x128 +7%, 16x256 +7% (per-image filters) / +22% (one shared
// filter); 128x32, 2048-point (spills) and 8192-point shapes were 2-24% slower
// and keep the tile.
#ifndef FUFFT_2D_FILTER_DIRECT
#define FUFFT_2D_FILTER_DIRECT 1
#endif
template<Mid MID>
static fufft_status conv2d_direct(int h, int w, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(h == 64 && w == 64) return launch_chain<Chain2<64, 64, 16>, In::C32, Out::C32, MID, Flt::BP_DIRECT, false>(a, st, dev);
   if(h == 32 && w == 128) return launch_chain<Chain2<32, 128, 16>, In::C32, Out::C32, MID, Flt::BP_DIRECT, false>(a, st, dev);
   if(h == 16 && w == 256) return launch_chain<Chain2<16, 256, 16>, In::C32, Out::C32, MID, Flt::BP_DIRECT, false>(a, st, dev);
   return FUFFT_ERR_UNSUPPORTED;
}

// chain-order (linear) 2-D filters of images with whole warps (n >= 512),
// n = 2^k with bit k of the mask: staged per warp through the exchange
// slots, as in 1-D.  Measured on B200 (1 GiB, per-image / shared filter,
// staged against 128 contiguous bytes per thread from global memory, the two
// builds interleaved kernel by kernel): +24-42% at 1024-4096 points (e.g.
// 8x256 90 / 64%, 16x128 89 / 63%, 32x128 72 / 55%), +14-20% at 8192
#ifndef FUFFT_2D_LIN_STAGED
#define FUFFT_2D_LIN_STAGED ((1 << 9) | (1 << 10) | (1 << 11) | (1 << 12) | (1 << 13))
#endif
template<Mid MID>
static fufft_status conv2d_lin_staged(int h, int w, const ConvArgs& a, cudaStream_t st, int dev)
{
#define FUFFT_2D(HH, WW)                                                                                     \
   if constexpr(in_mask(FUFFT_2D_LIN_STAGED, HH * WW))                                                        \
      if(h == HH && w == WW)                                                                                  \
         return launch_chain<Chain2<HH, WW, 16>, In::C32, Out::C32, MID, Flt::LIN_STAGED, false>(a, st, dev);
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 256)
   FUFFT_2D(8, 512)
   FUFFT_2D(8, 1024)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 128)
   FUFFT_2D(16, 256)
   FUFFT_2D(16, 512)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 64)
   FUFFT_2D(32, 128)
   FUFFT_2D(32, 256)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 32)
   FUFFT_2D(64, 64)
   FUFFT_2D(64, 128)
   FUFFT_2D(128, 16)
   FUFFT_2D(128, 32)
   FUFFT_2D(128, 64)
   FUFFT_2D(256, 16)
   FUFFT_2D(256, 32)
   FUFFT_2D(512, 16)
#undef FUFFT_2D
   return FUFFT_ERR_UNSUPPORTED;
}

fufft_status family_conv2d_r16(int h, int w, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(!bperm && mid != FUFFT_MID_NONE && aligned(a.b, 16) && (a.filter_stride * 8) % 16 == 0) {
      const fufft_status s = mid == FUFFT_MID_MULTIPLY ? conv2d_lin_staged<Mid::MUL>(h, w, a, st, dev)
                                                       : conv2d_lin_staged<Mid::CONJ>(h, w, a, st, dev);
      if(s != FUFFT_ERR_UNSUPPORTED) return s;
   }
   if(FUFFT_2D_FILTER_DIRECT && bperm && mid != FUFFT_MID_NONE) {
      const fufft_status s = mid == FUFFT_MID_MULTIPLY ? conv2d_direct<Mid::MUL>(h, w, a, st, dev)
                                                       : conv2d_direct<Mid::CONJ>(h, w, a, st, dev);
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
bool conv2d_supported_r16(int h, int w)
{
#define FUFFT_2D(HH, WW) if(h == HH && w == WW) return true;
   FUFFT_2D(8, 16)
   FUFFT_2D(8, 32)
   FUFFT_2D(8, 64)
   FUFFT_2D(8, 128)
   FUFFT_2D(8, 256)
   FUFFT_2D(8, 512)
   FUFFT_2D(8, 1024)
   FUFFT_2D(16, 16)
   FUFFT_2D(16, 32)
   FUFFT_2D(16, 64)
   FUFFT_2D(16, 128)
   FUFFT_2D(16, 256)
   FUFFT_2D(16, 512)
   FUFFT_2D(32, 16)
   FUFFT_2D(32, 32)
   FUFFT_2D(32, 64)
   FUFFT_2D(32, 128)
   FUFFT_2D(32, 256)
   FUFFT_2D(64, 16)
   FUFFT_2D(64, 32)
   FUFFT_2D(64, 64)
   FUFFT_2D(64, 128)
   FUFFT_2D(128, 16)
   FUFFT_2D(128, 32)
   FUFFT_2D(128, 64)
   FUFFT_2D(256, 16)
   FUFFT_2D(256, 32)
   FUFFT_2D(512, 16)
#undef FUFFT_2D
   return false;
}
}  // namespace host
}  // namespace fufft
