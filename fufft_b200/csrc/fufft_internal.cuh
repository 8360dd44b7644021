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
#include "fufft_stream.cuh"

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

int sm_count(int device);

template<class C, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
fufft_status launch_chain(const ConvArgs& args, cudaStream_t st, int device)
{
   constexpr int CPB = cpb_for(C::T);
   using K = ConvKernel<C, CPB, IN, OUT, MID, FLT, FBFP>;
   auto kern = conv_kernel<C, CPB, IN, OUT, MID, FLT, FBFP>;
   static std::atomic<uint64_t> configured{0};
   static std::atomic<int> resident[64];
   const uint64_t bit = 1ull << (device & 63);
   if(!(configured.load(std::memory_order_acquire) & bit)) {
      fufft_status s = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM));
      if(s != FUFFT_OK) return s;
#ifndef FUFFT_CARVEOUT_CAP
#define FUFFT_CARVEOUT_CAP 1
#endif
      if(FUFFT_CARVEOUT_CAP) {
         // hold the kernel at its occupancy target (resident_threads) even when
         // it needs fewer registers than the target allows: a shared-memory
         // carve-out that fits exactly that many CTAs (1 KB reserved per CTA),
         // the rest of the SM's 256 KB stays L1
         constexpr int target = resident_for<C, IN, OUT, FLT>();
         constexpr int ctas = target >= K::THREADS ? target / K::THREADS : 1;
         constexpr long long need = (long long)ctas * ((long long)K::SMEM + 1024);
         const int pct = need >= 228 * 1024 ? 100 : (int)((need * 100 + 228 * 1024 - 1) / (228 * 1024));
         if(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct) != cudaSuccess)
            cudaGetLastError();
      }
      int nb = 0;
      if(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, K::THREADS, K::SMEM) != cudaSuccess) {
         cudaGetLastError();
         nb = 0;
      }
      resident[device & 63].store(nb * sm_count(device));
      configured.fetch_or(bit, std::memory_order_acq_rel);
   }
   const long long grid = (args.batch + CPB - 1) / CPB;
#ifndef FUFFT_L2_PREFETCH
#define FUFFT_L2_PREFETCH 1
#endif
   // L2 prefetch one wave ahead: +2-3% for fp32 signals at N = 1024..4096
   // over 1 GiB (B200, A/B), neutral for int16-BFP, and -7% for a launch of
   // 3-4 waves (N=1024 x 4096), so fp32 launches of 8 waves or more only
   const long long res = resident[device & 63].load();
   ConvArgs a2 = args;
   if(FUFFT_L2_PREFETCH && IN == In::C32 && aligned(args.a, 16) && (MID == Mid::NONE || aligned(args.b, 16)) &&
      res > 0 && grid >= 8 * res)
      a2.prefetch_ahead = res;
#if FUFFT_PDL
   // programmatic dependent launch: this grid may be scheduled while the
   // stream's previous kernel finishes (its CTAs wait on griddepcontrol.wait
   // before touching global memory, so every dependency still holds)
   cudaLaunchConfig_t cfg = {};
   cfg.gridDim = dim3((unsigned)grid);
   cfg.blockDim = dim3(K::THREADS);
   cfg.dynamicSmemBytes = K::SMEM;
   cfg.stream = st;
   cudaLaunchAttribute at[1];
   at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
   at[0].val.programmaticStreamSerializationAllowed = 1;
   cfg.attrs = at;
   cfg.numAttrs = 1;
   fufft_status ls = check(cudaLaunchKernelEx(&cfg, kern, a2));
   if(ls != FUFFT_OK) return ls;
#else
   kern<<<(unsigned)grid, K::THREADS, K::SMEM, st>>>(a2);
#endif
   count_launch();
   return check(cudaGetLastError());
}

// ---- persistent TMA-pipelined kernel (fufft_stream.cuh) -------------------
// 2-D tensor map over `bytes` of data seen as 128-byte rows (32 fp32 or 32
// 32-bit words each), box = box_rows rows, SWIZZLE_128B
fufft_status encode_rows_tmap(CUtensorMap* tm, const void* base, unsigned long long bytes, int box_rows, bool words);
int sm_count(int device);

template<int N, int R, bool BFP, Mid MID, bool FLIN>
fufft_status launch_stream(const ConvArgs& args, cudaStream_t st, int device)
{
   constexpr int T = N / R;
   constexpr int CPB = cpb_for(T);
   using K = StreamKernel<N, R, CPB, BFP, MID, FLIN>;
   auto kern = conv_stream_kernel<N, R, CPB, BFP, MID, FLIN>;
   static std::atomic<uint64_t> configured{0};
   static std::atomic<int> blocks_per_sm[64];
   const uint64_t bit = 1ull << (device & 63);
   if(!(configured.load(std::memory_order_acquire) & bit)) {
      fufft_status s = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM));
      if(s != FUFFT_OK) return s;
      // ask for the smallest shared-memory carveout that still holds the
      // resident CTAs, so the rest of the 256 KB stays L1 for the twiddle tables
      const int per_sm_kb = (int)(((K::THREADS <= 256 ? 2 : 1) * (K::SMEM + 1024) + 1023) / 1024);
      const int pct = per_sm_kb >= 228 ? 100 : (per_sm_kb * 100 + 227) / 228;
      s = check(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct));
      if(s != FUFFT_OK) return s;
      int nb = 0;
      s = check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, K::THREADS, K::SMEM));
      if(s != FUFFT_OK) return s;
      blocks_per_sm[device & 63].store(nb > 0 ? nb : 1);
      configured.fetch_or(bit, std::memory_order_acq_rel);
   }
   const long long ngroups = (args.batch + CPB - 1) / CPB;
   CUtensorMap ta, tb;
   fufft_status s = encode_rows_tmap(&ta, args.a, (unsigned long long)args.batch * N * K::EB, K::SIG_BOX, BFP);
   if(s != FUFFT_OK) return s;
   if constexpr(MID != Mid::NONE) {
      const unsigned long long fbytes = ((unsigned long long)(args.batch - 1) * args.filter_stride + N) * K::EB;
      s = encode_rows_tmap(&tb, args.b, fbytes, K::FLT_BOX, BFP);
      if(s != FUFFT_OK) return s;
   } else {
      tb = ta;
   }
   const long long cap = (long long)sm_count(device) * blocks_per_sm[device & 63].load();
   const long long grid = ngroups < cap ? ngroups : cap;
   kern<<<(unsigned)grid, K::THREADS, K::SMEM, st>>>(ta, tb, args, ngroups);
   count_launch();
   return check(cudaGetLastError());
}

template<int R, bool BFP, Mid MID, bool FLIN>
fufft_status launch_stream_n(int n, const ConvArgs& args, cudaStream_t st, int device)
{
#define FUFFT_SCASE(NN)                                                                \
   case NN:                                                                            \
      if constexpr(NN >= R && NN * (BFP ? 4 : 8) >= 128 && NN <= (R == 8 ? MAX_N_R8 : MAX_N_R16)) \
         return launch_stream<NN, R, BFP, MID, FLIN>(args, st, device);                \
      else return FUFFT_ERR_UNSUPPORTED;
   switch(n) {
      FUFFT_SCASE(16) FUFFT_SCASE(32) FUFFT_SCASE(64) FUFFT_SCASE(128) FUFFT_SCASE(256)
      FUFFT_SCASE(512) FUFFT_SCASE(1024) FUFFT_SCASE(2048) FUFFT_SCASE(4096) FUFFT_SCASE(8192)
   default: return FUFFT_ERR_UNSUPPORTED;
   }
#undef FUFFT_SCASE
}

template<int N, int R, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
fufft_status launch(const ConvArgs& args, cudaStream_t st, int device)
{
   return launch_chain<Chain<N, R>, IN, OUT, MID, FLT, FBFP>(args, st, device);
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
// fp32 radix-16 (complex, and two-for-one real) with the register-boundary
// filter, n >= CONV_DIRECT_MIN_N: the filter
// read straight from global memory at three CTAs per SM (resident_for)
#ifndef FUFFT_CONV_FILTER_DIRECT
#define FUFFT_CONV_FILTER_DIRECT 1
#endif
#ifndef FUFFT_R2_FILTER_DIRECT
#define FUFFT_R2_FILTER_DIRECT 1   // two-for-one real: +6-8% at n = 4096, +1% at 2048
#endif
// fp32 radix-8 register-boundary layout (R8_BPERM): the filter read straight
// from global memory for n = 2^k with bit k of the mask set, else the
// TMA-staged tile.  Measured on B200 (complex convolution, 1 GiB signals,
// median of three interleaved runs on each of two boxes, % of measured HBM,
// direct / tile): 512: 104.5 / 88.1 and 97.4 / 86.6; 1024: 74.5 / 64.1 and
// 69.2 / 64.6; 2048: 76.3 / 74.5 and 73.6 / 76.3 (even, kept on the tile);
// 4096: 65.4 / 71.0.  (Two radix-8 butterfly groups per thread on 16
// registers -- half the threads per transform -- measured 66-100% at the
// same sizes: no gain, not built.)
#ifndef FUFFT_R8_BP_DIRECT
#define FUFFT_R8_BP_DIRECT ((1 << 9) | (1 << 10))
#endif
constexpr bool in_mask(long long mask, int n)
{
   return n > 0 && (1 << ilog2c(n)) == n && ((mask >> ilog2c(n)) & 1);
}
// launch_n restricted to the sizes of a mask (instantiates only those)
template<long long MASK, int R, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
fufft_status launch_masked(int n, const ConvArgs& args, cudaStream_t st, int device)
{
#define FUFFT_MCASE(NN)                                                                \
   case NN:                                                                            \
      if constexpr(in_mask(MASK, NN) && NN >= R && NN <= (R == 8 ? MAX_N_R8 : MAX_N_R16)) \
         return launch<NN, R, IN, OUT, MID, FLT, FBFP>(args, st, device);              \
      else return FUFFT_ERR_UNSUPPORTED;
   switch(n) {
      FUFFT_MCASE(8) FUFFT_MCASE(16) FUFFT_MCASE(32) FUFFT_MCASE(64) FUFFT_MCASE(128) FUFFT_MCASE(256)
      FUFFT_MCASE(512) FUFFT_MCASE(1024) FUFFT_MCASE(2048) FUFFT_MCASE(4096) FUFFT_MCASE(8192)
   default: return FUFFT_ERR_UNSUPPORTED;
   }
#undef FUFFT_MCASE
}

template<int R, In IN, Out OUT, bool FBFP>
fufft_status dispatch_mid(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if constexpr(FUFFT_CONV_FILTER_DIRECT && R == 16 && !FBFP &&
                ((IN == In::C32 && OUT == Out::C32) || (FUFFT_R2_FILTER_DIRECT && IN == In::REAL2 && OUT == Out::REAL2))) {
      const bool small = IN == In::C32 && n == CONV_DIRECT_SMALL_N && a.batch * n <= CONV_DIRECT_SMALL_POINTS;
      if(bperm && (n >= CONV_DIRECT_MIN_N || small) && mid != FUFFT_MID_NONE)
         return mid == FUFFT_MID_MULTIPLY ? launch_n<R, IN, OUT, Mid::MUL, Flt::BP_DIRECT, FBFP>(n, a, st, dev)
                                          : launch_n<R, IN, OUT, Mid::CONJ, Flt::BP_DIRECT, FBFP>(n, a, st, dev);
   }
   if constexpr(R == 8 && !FBFP && IN == In::C32 && OUT == Out::C32) {
      constexpr long long M = FUFFT_R8_BP_DIRECT;
      if(bperm && mid != FUFFT_MID_NONE && in_mask(M, n) && n <= MAX_N_R8)
         return mid == FUFFT_MID_MULTIPLY ? launch_masked<M, R, IN, OUT, Mid::MUL, Flt::BP_DIRECT, FBFP>(n, a, st, dev)
                                          : launch_masked<M, R, IN, OUT, Mid::CONJ, Flt::BP_DIRECT, FBFP>(n, a, st, dev);
   }
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

// fp32 / BFP convolution.  Measured on B200 (N = 512..8192, 1 GiB signal):
// the direct kernel (fufft_conv.cuh) is fastest whenever the filter arrives in
// the register-boundary layout (TMA bulk prefetch) and for BFP; the
// persistent TMA-pipelined kernel (fufft_stream.cuh) wins for an fp32 filter
// in the linear chain order (it stages that filter through a swizzled TMA
// tensor load instead of 128-byte-per-thread global reads).  The pipelined
// kernel needs 16-byte aligned signal and filter and whole 128-byte rows per
// transform and per filter stride; otherwise the direct kernel runs.
// fp32 convolution with a chain-order filter staged warp by warp
// (Flt::LIN_STAGED): radix 16 for 512 <= n <= 8192, radix 8 for 256 <= n <= 4096
template<int R, In IN, Out OUT, Mid MID>
fufft_status launch_lin_staged(int n, const ConvArgs& a, cudaStream_t st, int dev)
{
   switch(n) {
   case 256:
      if constexpr(R == 8) return launch<256, 8, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
      else return FUFFT_ERR_UNSUPPORTED;
   case 512: return launch<512, R, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
   case 1024: return launch<1024, R, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
   case 2048: return launch<2048, R, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
   case 4096: return launch<4096, R, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
   case 8192:
      if constexpr(R == 16) return launch<8192, 16, IN, OUT, MID, Flt::LIN_STAGED, false>(a, st, dev);
      else return FUFFT_ERR_UNSUPPORTED;
   default: return FUFFT_ERR_UNSUPPORTED;
   }
}

// fp32 convolution with a filter in a radix-8 layout (the reference's mixedrev
// order of fufft_pipeline_ip, or its register-boundary order) on the radix-16
// engine: at n = 4096 three passes each way instead of four, two exchanges
// instead of three; the filter staged per warp through a compile-time bit
// permutation (R8Perm).  Bit k of a mask selects n = 2^k.  Measured on B200
// (complex convolution, 1 GiB signals, median of three interleaved runs, % of
// measured HBM, radix-16 engine / radix-8 engine): R8 1024: 76.3 / 67.3,
// 2048: 75.2 / 65.0, 4096: 73.4 / 58.7 (512: 83.5 / 81.0, kept on radix 8);
// R8_BPERM 2048: 73.7 / 71.9, 4096: 67.4-70.6 / 62.8-63.6 (512: 87.0 / 96.6,
// 1024: 69.3 / 70.5, kept on radix 8).
#ifndef FUFFT_R8_ON_R16_LIN
#define FUFFT_R8_ON_R16_LIN ((1 << 10) | (1 << 11) | (1 << 12))
#endif
#ifndef FUFFT_R8_ON_R16_BP
#define FUFFT_R8_ON_R16_BP ((1 << 10) | (1 << 11) | (1 << 12))
#endif
template<Mid MID, long long MASK, Flt FLT, In IN = In::C32, Out OUT = Out::C32>
fufft_status launch_r8_on_r16(int n, const ConvArgs& a, cudaStream_t st, int dev)
{
#define FUFFT_PCASE(NN)                                                                          \
   case NN:                                                                                      \
      if constexpr(in_mask(MASK, NN)) return launch<NN, 16, IN, OUT, MID, FLT, false>(a, st, dev); \
      else return FUFFT_ERR_UNSUPPORTED;
   switch(n) {
      FUFFT_PCASE(512) FUFFT_PCASE(1024) FUFFT_PCASE(2048) FUFFT_PCASE(4096)
   default: return FUFFT_ERR_UNSUPPORTED;
   }
#undef FUFFT_PCASE
}

// the radix-8 register-boundary filter: read straight from global memory
// (whole 32-byte sectors per four lanes) or staged per warp like the chain
// order.  Interleaved A/B on B200 (1 GiB, % of HBM, direct / staged): 2048:
// 83.3 / 77.3, 4096: 77.0 / 74.7; against the radix-8 engine at 1024: 81.8 /
// 75.1 (512: 95.5 / 103.7, kept on radix 8)
#ifndef FUFFT_R8BP_DIRECT
#define FUFFT_R8BP_DIRECT 1
#endif
constexpr Flt R8BP_FLT = FUFFT_R8BP_DIRECT ? Flt::R8BP_DIRECT : Flt::R8BP_STAGED;

// the two radix-8 layouts on the radix-16 engine, for one kernel family
template<In IN, Out OUT, long long ML, long long MB>
fufft_status dispatch_r8_on_r16(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(mid == FUFFT_MID_NONE || !in_mask(bperm ? MB : ML, n) || !aligned(a.b, 16) || (a.filter_stride * 8) % 16)
      return FUFFT_ERR_UNSUPPORTED;
   if(bperm)
      return mid == FUFFT_MID_MULTIPLY ? launch_r8_on_r16<Mid::MUL, MB, R8BP_FLT, IN, OUT>(n, a, st, dev)
                                       : launch_r8_on_r16<Mid::CONJ, MB, R8BP_FLT, IN, OUT>(n, a, st, dev);
   return mid == FUFFT_MID_MULTIPLY ? launch_r8_on_r16<Mid::MUL, ML, Flt::R8_STAGED, IN, OUT>(n, a, st, dev)
                                    : launch_r8_on_r16<Mid::CONJ, ML, Flt::R8_STAGED, IN, OUT>(n, a, st, dev);
}

// split apply: the spectrum comes in the layout family of the filter --
// register-boundary order with the register-boundary filter, chain order with
// the chain-order filter
#ifndef FUFFT_APPLY_FILTER_DIRECT
#define FUFFT_APPLY_FILTER_DIRECT 1
#endif
constexpr Flt APPLY_FLT = FUFFT_APPLY_FILTER_DIRECT ? Flt::BP_DIRECT : Flt::SMEM;
// radix-8 spectra and filters (the reference's fufft_pipeline_fwd / _apply
// layouts, fufft.cuh:1343-1407) on the radix-16 engine, for n = 2^k with bit
// k of the mask: spectra and filters staged per warp through the bit
// permutation (R8Perm).  Measured on B200 (1 GiB, % of HBM at 16 B/pt
// forward and 24 B/pt apply, radix-16 engine / radix-8 engine, the two
// builds interleaved kernel by kernel in one process): forward R8 512: 99 /
// 82, 1024: 88 / 58, 2048: 88 / 53, 4096: 93 / 42; forward R8_BPERM 4096:
// 86 / 55 (1024, 2048: 85 / 89, 75 / 79, kept on radix 8); apply R8 4096:
// 82 / 59 (1024, 2048: 87 / 90, 72 / 80); apply R8_BPERM (spectrum and
// filter read directly by the radix-8 engine) 74 / 107, 64 / 108, 63 / 93.
#ifndef FUFFT_FWD_R8_ON_R16
#define FUFFT_FWD_R8_ON_R16 ((1 << 9) | (1 << 10) | (1 << 11) | (1 << 12))
#endif
#ifndef FUFFT_FWD_R8BP_ON_R16
#define FUFFT_FWD_R8BP_ON_R16 (1 << 12)
#endif
#ifndef FUFFT_APPLY_R8_ON_R16
#define FUFFT_APPLY_R8_ON_R16 (1 << 12)
#endif
#ifndef FUFFT_APPLY_R8BP_ON_R16
#define FUFFT_APPLY_R8BP_ON_R16 0
#endif
#ifndef FUFFT_APPLY_LIN_STAGED
#define FUFFT_APPLY_LIN_STAGED 1
#endif

template<int R, Out OUT>
fufft_status dispatch_apply(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   const bool filt_ok = aligned(a.b, 16) && (a.filter_stride * 8) % 16 == 0;
   if constexpr(R == 8) {
      constexpr long long M = FUFFT_APPLY_R8_ON_R16, MB = FUFFT_APPLY_R8BP_ON_R16;
      if(bperm && in_mask(MB, n) && (mid == FUFFT_MID_NONE || filt_ok)) {
         switch(mid) {
         case FUFFT_MID_NONE: return launch_r8_on_r16<Mid::NONE, MB, Flt::NONE, In::SPEC_R8BP, OUT>(n, a, st, dev);
         case FUFFT_MID_MULTIPLY:
            return launch_r8_on_r16<Mid::MUL, MB, Flt::R8BP_STAGED, In::SPEC_R8BP, OUT>(n, a, st, dev);
         case FUFFT_MID_CONJ_MULTIPLY:
            return launch_r8_on_r16<Mid::CONJ, MB, Flt::R8BP_STAGED, In::SPEC_R8BP, OUT>(n, a, st, dev);
         }
         return FUFFT_ERR_INVALID_ARG;
      }
      if(!bperm && in_mask(M, n) && (mid == FUFFT_MID_NONE || filt_ok)) {
         switch(mid) {
         case FUFFT_MID_NONE: return launch_r8_on_r16<Mid::NONE, M, Flt::NONE, In::SPEC_R8, OUT>(n, a, st, dev);
         case FUFFT_MID_MULTIPLY:
            return launch_r8_on_r16<Mid::MUL, M, Flt::R8_STAGED, In::SPEC_R8, OUT>(n, a, st, dev);
         case FUFFT_MID_CONJ_MULTIPLY:
            return launch_r8_on_r16<Mid::CONJ, M, Flt::R8_STAGED, In::SPEC_R8, OUT>(n, a, st, dev);
         }
         return FUFFT_ERR_INVALID_ARG;
      }
   }
   // radix-16 chain-order filter with whole warps per transform: staged per
   // warp (the spectrum too: SPEC_ROWS)
   if constexpr(FUFFT_APPLY_LIN_STAGED && R == 16) {
      if(!bperm && mid != FUFFT_MID_NONE && n >= 32 * R && n <= max_n(R) && filt_ok)
         return mid == FUFFT_MID_MULTIPLY ? launch_lin_staged<R, In::SPEC, OUT, Mid::MUL>(n, a, st, dev)
                                          : launch_lin_staged<R, In::SPEC, OUT, Mid::CONJ>(n, a, st, dev);
   }
   switch(mid) {
   case FUFFT_MID_NONE:
      return bperm ? launch_n<R, In::SPEC_BP, OUT, Mid::NONE, Flt::NONE, false>(n, a, st, dev)
                   : launch_n<R, In::SPEC, OUT, Mid::NONE, Flt::NONE, false>(n, a, st, dev);
   case FUFFT_MID_MULTIPLY:
      return bperm ? launch_n<R, In::SPEC_BP, OUT, Mid::MUL, APPLY_FLT, false>(n, a, st, dev)
                   : launch_n<R, In::SPEC, OUT, Mid::MUL, Flt::GLOBAL, false>(n, a, st, dev);
   case FUFFT_MID_CONJ_MULTIPLY:
      return bperm ? launch_n<R, In::SPEC_BP, OUT, Mid::CONJ, APPLY_FLT, false>(n, a, st, dev)
                   : launch_n<R, In::SPEC, OUT, Mid::CONJ, Flt::GLOBAL, false>(n, a, st, dev);
   }
   return FUFFT_ERR_INVALID_ARG;
}

// forward transform to a spectrum in the layout's order (fwd, fwd_r2, filter
// preparation); radix-8 layouts on the radix-16 engine as for the apply
template<int R, In IN>
fufft_status dispatch_fwd(int n, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if constexpr(R == 8) {
      constexpr long long M = FUFFT_FWD_R8_ON_R16, MB = FUFFT_FWD_R8BP_ON_R16;
      if(bperm && in_mask(MB, n)) return launch_r8_on_r16<Mid::NONE, MB, Flt::NONE, IN, Out::SPEC_R8BP>(n, a, st, dev);
      if(!bperm && in_mask(M, n)) return launch_r8_on_r16<Mid::NONE, M, Flt::NONE, IN, Out::SPEC_R8>(n, a, st, dev);
   }
   return bperm ? launch_n<R, IN, Out::SPEC_BP, Mid::NONE, Flt::NONE, false>(n, a, st, dev)
                : launch_n<R, IN, Out::SPEC, Mid::NONE, Flt::NONE, false>(n, a, st, dev);
}

#ifndef FUFFT_LIN_STAGED
#define FUFFT_LIN_STAGED 1
#endif
template<int R, bool BFP>
fufft_status dispatch_conv(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if constexpr(!BFP && R == 8) {
      const fufft_status s =
         dispatch_r8_on_r16<In::C32, Out::C32, FUFFT_R8_ON_R16_LIN, FUFFT_R8_ON_R16_BP>(n, mid, bperm, a, st, dev);
      if(s != FUFFT_ERR_UNSUPPORTED) return s;
   }
   // fp32, chain-order filter (the reference's v16 / ip layouts), at least one
   // warp per transform: the direct kernel staging the filter through the
   // exchange buffer
   if constexpr(!BFP && FUFFT_LIN_STAGED) {
      if(!bperm && mid != FUFFT_MID_NONE && n >= 32 * R && n <= max_n(R) && aligned(a.b, 16) &&
         (a.filter_stride * 8) % 16 == 0)
         return mid == FUFFT_MID_MULTIPLY ? launch_lin_staged<R, In::C32, Out::C32, Mid::MUL>(n, a, st, dev)
                                          : launch_lin_staged<R, In::C32, Out::C32, Mid::CONJ>(n, a, st, dev);
   }
#ifndef FUFFT_NO_STREAM
   // fp32 signal with a multiply / conjugate-multiply filter in the linear chain order
   if constexpr(!BFP) {
      if(!bperm && mid != FUFFT_MID_NONE && n * 8 >= 128 && aligned(a.a, 16) && aligned(a.b, 16) &&
         (a.filter_stride * 8) % 128 == 0) {
         const fufft_status s = mid == FUFFT_MID_MULTIPLY ? launch_stream_n<R, false, Mid::MUL, true>(n, a, st, dev)
                                                          : launch_stream_n<R, false, Mid::CONJ, true>(n, a, st, dev);
         if(s != FUFFT_ERR_UNSUPPORTED) return s;
      }
   }
#endif
   // if constexpr: each kernel family's translation unit instantiates only its
   // own kernels (one definition of every kernel in the library)
   if constexpr(BFP) return dispatch_mid<R, In::BFP, Out::BFP, true>(n, mid, bperm, a, st, dev);
   else return dispatch_mid<R, In::C32, Out::C32, false>(n, mid, bperm, a, st, dev);
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
fufft_status family_apply_r2_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_apply_r2_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_fwd_r2_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_fwd_r2_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_c2c_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_c2c_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_r2_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_r2_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_conv2d_r8(int h, int w, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_conv2d_r16(int h, int w, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
bool conv2d_supported_r8(int h, int w);
fufft_status family_mid_bfpfilter_r8(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
fufft_status family_mid_bfpfilter_r16(int, fufft_midop, bool, const ConvArgs&, cudaStream_t, int);
// fp32 -> int16 pairs with the per-transform abs-max already in `scale`
// (fp32 bits); leaves scale = max(mx, 1e-30) / 32767
fufft_status bfp_requantize(const float2* x, float* scale, uint32_t* q, long long n, long long batch, cudaStream_t st);
bool conv2d_supported_r16(int h, int w);
// cluster-fused convolutions (fufft_cluster.cu); FUFFT_ERR_UNSUPPORTED when the
// device cannot host the cluster
fufft_status cluster_conv1d(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev);
fufft_status cluster_large(int r_out, int mid_n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st,
                           int dev);
fufft_status cluster_large_bfp(int r_out, int mid_n, fufft_midop mid, bool bperm, const ConvArgs& a,
                               cudaStream_t st, int dev);
fufft_status cluster_conv2d(int h, int w, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev);
bool cluster_conv2d_shape(int h, int w);
constexpr int MAX_N_CLUSTER = 65536;   // radix-16 layouts, one cluster-fused kernel
// argument checks of the int16-BFP four-step (fufft_large.cu), shared by its
// workspace and allocation-free entry points
fufft_status validate_large_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq, const float* b_scale,
                                const int16_t* oq, const float* o_scale, int64_t n, int64_t batch, int r_out,
                                int mid, fufft_layout layout, fufft_midop midop, bool check_workspace,
                                const void* workspace, size_t workspace_bytes, int* lout, bool* nothing_to_do);

}  // namespace host
}  // namespace fufft
