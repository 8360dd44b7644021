// ref_cpu_fufft.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Gives a C ABI to the reference's Stockham radix-8 CPU program
// (cpu_fufft.cpp of weiwang217/FuFFT, included from the read-only reference
// tree at build time, never copied): its forward / inverse transforms
// (fufft_stockham8, natural order in and out, 1/N in the inverse) in fp64 and
// fp32, and the cyclic convolution of its check_convolution (cpu_fufft.cpp:
// 212-236), with that function's seeded input generator.  The wrappers only
// move data between interleaved double arrays and std::vector<std::complex>.
#define main fufft_reference_cpu_fufft_main
#include "cpu_fufft.cpp"
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
template<typename C> void conv(int N, const double* a, const double* b, double* out)
{
   // fwd(a), fwd(b), pointwise product, inverse with 1/N (cpu_fufft.cpp:225-229)
   std::vector<C> A = load<C>(a, N), B = load<C>(b, N), T(N);
   fufft_forward<C>(A, T, N);
   fufft_forward<C>(B, T, N);
   for(int i = 0; i < N; i++) A[i] *= B[i];
   fufft_inverse<C>(A, T, N);
   store(A, out);
}
}  // namespace

extern "C" {

int ref_cpufufft_main(void) { return fufft_reference_cpu_fufft_main(0, nullptr); }

// the inputs of check_convolution(N) (cpu_fufft.cpp:214-218), same seed and
// same draw order
void ref_cpufufft_gen_conv(int N, double* a, double* b)
{
   std::mt19937 rng(N * 7 + 1);
   std::uniform_real_distribution<double> d(-1.0, 1.0);
   for(int i = 0; i < N; i++) {
      cd va = cd(d(rng), d(rng));
      cd vb = cd(d(rng), d(rng));
      a[2 * i] = va.real(); a[2 * i + 1] = va.imag();
      b[2 * i] = vb.real(); b[2 * i + 1] = vb.imag();
   }
}

// fp32 != 0: the same algorithm on std::complex<float> (cpu_fufft.cpp:251-255)
void ref_cpufufft_conv(int N, int fp32, const double* a, const double* b, double* out)
{
   if(fp32) conv<cf>(N, a, b, out);
   else conv<cd>(N, a, b, out);
}

void ref_cpufufft_forward(int N, int fp32, const double* x, double* out)
{
   if(fp32) {
      std::vector<cf> A = load<cf>(x, N), T(N);
      fufft_forward<cf>(A, T, N);
      store(A, out);
   } else {
      std::vector<cd> A = load<cd>(x, N), T(N);
      fufft_forward<cd>(A, T, N);
      store(A, out);
   }
}

}  // extern "C"
