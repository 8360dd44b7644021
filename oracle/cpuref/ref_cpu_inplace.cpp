// ref_cpu_inplace.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Gives a C ABI to the reference's in-place radix-8 CPU program
// (cpu_inplace.cpp of weiwang217/FuFFT, included from the read-only reference
// tree at build time, never copied): forward DIF (natural in, digit-reversed
// out), inverse DIT, and the convolution of its main (cpu_inplace.cpp:173-193):
// filter spectrum = DIF(b) / N, left in digit-reversed order, times DIF(a),
// then DIT.  fp64 or fp32 (the passes are templates on the complex type).
#define main fufft_reference_cpu_inplace_main
#include "cpu_inplace.cpp"
#undef main

namespace {
template<typename C> std::vector<C> load(const double* p, int n)
{
   typedef typename C::value_type R;
   std::vector<C> v(n);
   for(int i = 0; i < n; i++) v[i] = C((R)p[2 * i], (R)p[2 * i + 1]);
   return v;
}
template<typename C> void store(const std::vector<C>& v, double* p)
{
   for(size_t i = 0; i < v.size(); i++) { p[2 * i] = (double)v[i].real(); p[2 * i + 1] = (double)v[i].imag(); }
}
template<typename C> void conv(int N, const double* a, const double* b, double* bs_out, double* out)
{
   typedef typename C::value_type R;
   std::vector<C> B = load<C>(b, N), Bs(N);
   fft_dif<C>(B.data(), N, -1);
   for(int i = 0; i < N; i++) Bs[i] = B[i] * ((R)1 / (R)N);
   std::vector<C> A = load<C>(a, N);
   fft_dif<C>(A.data(), N, -1);
   for(int i = 0; i < N; i++) A[i] *= Bs[i];
   fft_dit<C>(A.data(), N, +1);
   store(Bs, bs_out);
   store(A, out);
}
}  // namespace

extern "C" {

int ref_inplace_main(void) { return fufft_reference_cpu_inplace_main(); }

int ref_inplace_digitrev8(int i, int S) { return digitrev8(i, S); }

// bs_out: the digit-reversed filter spectrum / N; out: the convolution
void ref_inplace_conv(int N, int fp32, const double* a, const double* b, double* bs_out, double* out)
{
   if(fp32) conv<cf>(N, a, b, bs_out, out);
   else conv<cd>(N, a, b, bs_out, out);
}

}  // extern "C"
