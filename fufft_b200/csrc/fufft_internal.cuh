// fufft_internal.cuh -- host-side plumbing shared by the library's
// translation units: per-device context (twiddle tables, status word),
// CUDA error capture, argument validation and the templated launcher that
// maps a runtime n onto the compiled kernel instantiations.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/fufft_b200.h"
#include "fufft_conv.cuh"

namespace fufft {
namespace host {

struct DeviceCtx {
   const float2* tw;        // twiddle tables of this device
   unsigned int* status;    // device status word
   int device;
};

// current device's context; builds its twiddle tables on first use
fufft_status device_ctx(DeviceCtx* out);
// remember a CUDA error for fufft_last_cuda_error(); returns FUFFT_ERR_CUDA
fufft_status cuda_fail(cudaError_t e);
inline fufft_status check(cudaError_t e) { return e == cudaSuccess ? FUFFT_OK : cuda_fail(e); }
void count_launch();

inline bool pow2(long long n) { return n > 0 && (n & (n - 1)) == 0; }
inline bool aligned(const void* p, unsigned a) { return ((uintptr_t)p % a) == 0; }

inline int layout_radix(fufft_layout l)
{
   switch(l) {
   case FUFFT_LAYOUT_R8: case FUFFT_LAYOUT_R8_BPERM: return 8;
   case FUFFT_LAYOUT_R16: case FUFFT_LAYOUT_R16_BPERM: return 16;
   default: return 0;
   }
}
inline bool layout_bperm(fufft_layout l) { return l == FUFFT_LAYOUT_R8_BPERM || l == FUFFT_LAYOUT_R16_BPERM; }
constexpr int MAX_N_R8 = 4096;
constexpr int MAX_N_R16 = 8192;
inline int max_n(int radix) { return radix == 8 ? MAX_N_R8 : radix == 16 ? MAX_N_R16 : 0; }

// transforms per CTA: about 256 threads per CTA, at least one full warp
constexpr int cpb_for(int T) { return T >= 256 ? 1 : 256 / T; }

template<int N, int R, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
fufft_status launch(const ConvArgs& args, cudaStream_t st, int device)
{
   constexpr int T = N / R;
   constexpr int CPB = cpb_for(T);
   using K = ConvKernel<N, R, CPB, IN, OUT, MID, FLT, FBFP>;
   auto kern = conv_kernel<N, R, CPB, IN, OUT, MID, FLT, FBFP>;
   static std::atomic<uint64_t> configured{0};
   const uint64_t bit = 1ull << (device & 63);
   if(!(configured.load(std::memory_order_acquire) & bit)) {
      fufft_status s = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM));
      if(s != FUFFT_OK) return s;
      configured.fetch_or(bit, std::memory_order_acq_rel);
   }
   const long long grid = (args.batch + CPB - 1) / CPB;
   kern<<<(unsigned)grid, K::THREADS, K::SMEM, st>>>(args);
   count_launch();
   return check(cudaGetLastError());
}

// runtime n -> instantiation
template<int R, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
fufft_status launch_n(int n, const ConvArgs& args, cudaStream_t st, int device)
{
#define FUFFT_CASE(NN)                                                                 \
   case NN:                                                                            \
      if constexpr(NN >= R && NN <= (R == 8 ? MAX_N_R8 : MAX_N_R16))                   \
         return launch<NN, R, IN, OUT, MID, FLT, FBFP>(args, st, device);              \
      else return FUFFT_ERR_INVALID_SIZE;
   switch(n) {
      FUFFT_CASE(8) FUFFT_CASE(16) FUFFT_CASE(32) FUFFT_CASE(64) FUFFT_CASE(128) FUFFT_CASE(256)
      FUFFT_CASE(512) FUFFT_CASE(1024) FUFFT_CASE(2048) FUFFT_CASE(4096) FUFFT_CASE(8192)
   default: return FUFFT_ERR_INVALID_SIZE;
   }
#undef FUFFT_CASE
}

}  // namespace host
}  // namespace fufft

namespace fufft {
namespace host {

// mid-op / filter-read selection -> instantiation
template<int R, In IN, Out OUT, bool FBFP>
fufft_status dispatch_mid(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   switch(mid) {
   case FUFFT_MID_NONE: return launch_n<R, IN, OUT, Mid::NONE, Flt::NONE, FBFP>(n, a, st, dev);
   case FUFFT_MID_MULTIPLY:
      return bperm ? launch_n<R, IN, OUT, Mid::MUL, Flt::SMEM, FBFP>(n, a, st, dev)
                   : launch_n<R, IN, OUT, Mid::MUL, Flt::GLOBAL, FBFP>(n, a, st, dev);
   case FUFFT_MID_CONJ_MULTIPLY:
      return bperm ? launch_n<R, IN, OUT, Mid::CONJ, Flt::SMEM, FBFP>(n, a, st, dev)
                   : launch_n<R, IN, OUT, Mid::CONJ, Flt::GLOBAL, FBFP>(n, a, st, dev);
   }
   return FUFFT_ERR_INVALID_ARG;
}

// one entry per kernel family and radix (each lives in its own translation
// unit so the instantiations compile in parallel)
using FamilyFn = fufft_status (*)(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev);
fufft_status family_conv_f32_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_conv_f32_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_conv_bfp_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_conv_bfp_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_fwd_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_fwd_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_apply_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_apply_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_r2_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_r2_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);

}  // namespace host
}  // namespace fufft
