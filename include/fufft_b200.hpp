// fufft_b200.hpp -- the reference's C++ entry points and mid-op policy structs
// (weiwang217/FuFFT, fufft.cuh) as a header-only layer over the C ABI in
// fufft_b200.h.
//
// The reference's callers launch kernel templates themselves:
//     fufft_pipeline_v16<N, L16, NR16, CPB><<<batch / CPB, CPB * N / 16, CPB * N * 8>>>(
//         d_a, d_out, MidMultiply{d_b16}, nullptr);                 // bench_fufft.cu:218
// Here the same template names and arguments become one host call that also
// takes the batch size and a stream:
//     fufft_b200::fufft_pipeline_v16<N, L16, NR16, CPB>(d_a, d_out, MidMultiply{d_b16}, nullptr, batch);
// The template parameters keep their meaning (N = LEAD * 8^NR8 or
// LEAD * 16^NRV; the factorisation is checked at compile time) and CPB is
// accepted for source compatibility (the library picks its own transforms per
// CTA, and the batch no longer has to be a multiple of it).  Filter layouts
// are exactly the reference's: mixedrev for the radix-8 kernels, mixedrev16
// for the radix-16 ones, the register-boundary bperm for _fused / _v16f.
// `timing` (the reference's in-kernel phase timer buffer) is accepted and
// ignored.  Calls return fufft_status instead of exiting on error.
#pragma once
#include <cuda_runtime.h>

#include "fufft_b200.h"

namespace fufft_b200 {

// ---- mid-op policies (fufft.cuh:625-650) ----------------------------------
struct MidNothing {};
struct MidMultiply { const float2* b; };
struct MidConjMultiply { const float2* b; };

namespace detail {
constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n / 2); }
constexpr int ipow(int b, int e) { return e == 0 ? 1 : b * ipow(b, e - 1); }
inline fufft_stream_t st(cudaStream_t s) { return reinterpret_cast<fufft_stream_t>(s); }
inline fufft_midop op(const MidNothing&) { return FUFFT_MID_NONE; }
inline fufft_midop op(const MidMultiply&) { return FUFFT_MID_MULTIPLY; }
inline fufft_midop op(const MidConjMultiply&) { return FUFFT_MID_CONJ_MULTIPLY; }
inline const float* filt(const MidNothing&) { return nullptr; }
inline const float* filt(const MidMultiply& m) { return reinterpret_cast<const float*>(m.b); }
inline const float* filt(const MidConjMultiply& m) { return reinterpret_cast<const float*>(m.b); }
template<int N, int LEAD, int NR, int R> constexpr bool factors() { return N == LEAD * ipow(R, NR); }
}  // namespace detail

// radix-8 in-place conv, any mid-op, filter in mixedrev order (fufft.cuh:1757)
template<int N, int LEAD, int NR8, int CPB, class Mid>
fufft_status fufft_pipeline_ip(const float2* a, float2* out, Mid mid, unsigned int* timing, long long batch,
                               cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR8, 8>(), "N must equal LEAD * 8^NR8");
   (void)timing;
   return fufft_conv_c2c_f32(reinterpret_cast<const float*>(a), detail::filt(mid), reinterpret_cast<float*>(out), N,
                             batch, FUFFT_LAYOUT_R8, detail::op(mid), N, detail::st(stream));
}

// radix-8 with the register-resident boundary, filter in bperm order (fufft.cuh:1774)
template<int N, int LEAD, int NR8, int CPB>
fufft_status fufft_pipeline_fused(const float2* a, const float2* bperm, float2* out, unsigned int* timing,
                                  long long batch, cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR8, 8>(), "N must equal LEAD * 8^NR8");
   (void)timing;
   return fufft_conv_c2c_f32(reinterpret_cast<const float*>(a), reinterpret_cast<const float*>(bperm),
                             reinterpret_cast<float*>(out), N, batch, FUFFT_LAYOUT_R8_BPERM, FUFFT_MID_MULTIPLY, N,
                             detail::st(stream));
}

// radix-16, sixteen values per lane, filter in mixedrev16 order (fufft.cuh:1518)
template<int N, int LEAD, int NRV, int CPB>
fufft_status fufft_pipeline_v16(const float2* a, float2* out, MidMultiply mid, unsigned int* timing, long long batch,
                                cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NRV, 16>(), "N must equal LEAD * 16^NRV");
   (void)timing;
   return fufft_conv_c2c_f32(reinterpret_cast<const float*>(a), detail::filt(mid), reinterpret_cast<float*>(out), N,
                             batch, FUFFT_LAYOUT_R16, FUFFT_MID_MULTIPLY, N, detail::st(stream));
}

// the same for middles above 4096 (fufft.cuh:1717): one entry point covers both
template<int N, int LEAD, int NRV, int CPB>
fufft_status fufft_pipeline_v16_wide(const float2* a, float2* out, MidMultiply mid, unsigned int* timing,
                                     long long batch, cudaStream_t stream = 0)
{
   return fufft_pipeline_v16<N, LEAD, NRV, CPB>(a, out, mid, timing, batch, stream);
}

// radix-16 register boundary, filter in bperm16 order (fufft.cuh:1499)
template<int N, int LEAD, int NRV, int CPB>
fufft_status fufft_pipeline_v16f(const float2* a, const float2* bperm, float2* out, unsigned int* timing,
                                 long long batch, cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NRV, 16>(), "N must equal LEAD * 16^NRV");
   (void)timing;
   return fufft_conv_c2c_f32(reinterpret_cast<const float*>(a), reinterpret_cast<const float*>(bperm),
                             reinterpret_cast<float*>(out), N, batch, FUFFT_LAYOUT_R16_BPERM, FUFFT_MID_MULTIPLY, N,
                             detail::st(stream));
}

// radix-16 lane-pair kernel (fufft.cuh:1736): same transform and filter order as v16
template<int N, int LEAD, int NR16, int CPB, class Mid>
fufft_status fufft_pipeline_r16(const float2* a, float2* out, Mid mid, unsigned int* timing, long long batch,
                                cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR16, 16>(), "N must equal LEAD * 16^NR16");
   (void)timing;
   return fufft_conv_c2c_f32(reinterpret_cast<const float*>(a), detail::filt(mid), reinterpret_cast<float*>(out), N,
                             batch, FUFFT_LAYOUT_R16, detail::op(mid), N, detail::st(stream));
}

// int16 block floating point, radix-16 (fufft.cuh:1614)
template<int N, int LEAD, int NRV, int CPB>
fufft_status fufft_pipeline_v16_bfp(const short2* aq, const float* a_scale, const short2* bq, const float* b_scale,
                                    short2* outq, float* out_scale, unsigned int* timing, long long batch,
                                    cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NRV, 16>(), "N must equal LEAD * 16^NRV");
   (void)timing;
   return fufft_conv_c2c_bfp(reinterpret_cast<const int16_t*>(aq), a_scale, reinterpret_cast<const int16_t*>(bq),
                             b_scale, reinterpret_cast<int16_t*>(outq), out_scale, N, batch, FUFFT_LAYOUT_R16,
                             FUFFT_MID_MULTIPLY, N, detail::st(stream));
}

// split forward / apply, radix-8 chain (fufft.cuh:1343, :1375)
// natural-order forward c2c, N = 8^LOG8N (Mode A, fufft.cuh:878-904)
template<int N, int LOG8N, int CPB>
fufft_status fufft_c2c(const float2* in, float2* out, unsigned int* timing, long long batch, cudaStream_t stream = 0)
{
   static_assert(N == detail::ipow(8, LOG8N), "N must equal 8^LOG8N");
   (void)timing;
   return fufft_c2c_f32(reinterpret_cast<const float*>(in), reinterpret_cast<float*>(out), N, batch, -1,
                        detail::st(stream));
}

template<int N, int LEAD, int NR8, int CPB>
fufft_status fufft_pipeline_fwd(const float2* a, float2* spec, unsigned int* timing, long long batch,
                                cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR8, 8>(), "N must equal LEAD * 8^NR8");
   (void)timing;
   return fufft_fwd_f32(reinterpret_cast<const float*>(a), reinterpret_cast<float*>(spec), N, batch, FUFFT_LAYOUT_R8,
                        detail::st(stream));
}
template<int N, int LEAD, int NR8, int CPB>
fufft_status fufft_pipeline_apply(const float2* spec, const float2* bspec_dr, float2* out, unsigned int* timing,
                                  long long batch, cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR8, 8>(), "N must equal LEAD * 8^NR8");
   (void)timing;
   return fufft_apply_f32(reinterpret_cast<const float*>(spec), reinterpret_cast<const float*>(bspec_dr),
                          reinterpret_cast<float*>(out), N, batch, FUFFT_LAYOUT_R8, FUFFT_MID_MULTIPLY, N, N,
                          detail::st(stream));
}

// two-for-one real convolution, radix-8 chain (fufft.cuh:1273)
template<int N, int LEAD, int NR8, int CPB>
fufft_status fufft_conv_r2(const float* xr, const float* yr, const float2* bspec_dr, float* ur, float* vr,
                           unsigned int* timing, long long batch, cudaStream_t stream = 0)
{
   static_assert(detail::factors<N, LEAD, NR8, 8>(), "N must equal LEAD * 8^NR8");
   (void)timing;
   return fufft_conv_r2_f32(xr, yr, reinterpret_cast<const float*>(bspec_dr), ur, vr, N, batch, FUFFT_LAYOUT_R8,
                            FUFFT_MID_MULTIPLY, N, detail::st(stream));
}

// fused 2-D conv, H x W powers of 8, radix-8 chains (fufft.cuh:1209)
template<int H, int W, int CPB>
fufft_status fufft_conv2d(const float2* a, float2* out, MidMultiply mid, unsigned int* timing, long long batch,
                          cudaStream_t stream = 0)
{
   (void)timing;
   return fufft_conv2d_f32(reinterpret_cast<const float*>(a), detail::filt(mid), reinterpret_cast<float*>(out), H, W,
                           batch, FUFFT_LAYOUT_R8, FUFFT_MID_MULTIPLY, (long long)H * W, detail::st(stream));
}

// four-step: run_large<N, LOUT, ROUT, MID, MLEAD, MNRV> (bench_fufft.cu:391), in place
template<int N, int LOUT, int ROUT, int MID, int MLEAD, int MNRV>
fufft_status run_large(float2* buf, const float2* bdr, long long batch, cudaStream_t stream = 0)
{
   static_assert(detail::factors<MID, MLEAD, MNRV, 16>(), "MID must equal MLEAD * 16^MNRV");
   static_assert((long long)N == (long long)MID * detail::ipow(ROUT, LOUT), "N must equal ROUT^LOUT * MID");
   return fufft_conv_large_f32(reinterpret_cast<float*>(buf), reinterpret_cast<const float*>(bdr), N, batch, ROUT,
                               MID, FUFFT_LAYOUT_R16, FUFFT_MID_MULTIPLY, detail::st(stream));
}

}  // namespace fufft_b200
