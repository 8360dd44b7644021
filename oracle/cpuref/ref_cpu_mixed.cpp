// ref_cpu_mixed.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Gives a C ABI to the reference's mixed-radix in-place CPU program
// (cpu_mixed.cpp of weiwang217/FuFFT, included from the read-only reference
// tree at build time, never copied): the greedy factorisation over V = 8 or
// 16 values per lane (cpu_mixed.cpp:37-51), the mixed-radix digit reversal
// (mixedrev, :181-193) and the convolution of its run_for_V (:238-252):
// filter spectrum = DIF(b) / N in chain order, times DIF(a), then DIT.  fp64
// (the program is written for std::complex<double> only).
#define main fufft_reference_cpu_mixed_main
#include "cpu_mixed.cpp"
#undef main

extern "C" {

int ref_mixed_main(void) { return fufft_reference_cpu_mixed_main(); }

// radices of N for V values per lane; returns their count (0: unsupported)
int ref_mixed_factorise(int N, int V, int* R) { return factorise(N, V, R); }

int ref_mixed_rev(int idx, const int* R, int p) { return mixedrev(idx, R, p); }

// bs_out: DIF(b) / N in chain order; out: the convolution
int ref_mixed_conv(int N, int V, const double* a, const double* b, double* bs_out, double* out)
{
   int R[16];
   const int p = factorise(N, V, R);
   if(!p) return -1;
   std::vector<cd> B(N), A(N);
   for(int i = 0; i < N; i++) {
      B[i] = cd(b[2 * i], b[2 * i + 1]);
      A[i] = cd(a[2 * i], a[2 * i + 1]);
   }
   fft_dif(B.data(), N, -1, R, p, V);
   for(int i = 0; i < N; i++) B[i] /= (double)N;
   fft_dif(A.data(), N, -1, R, p, V);
   for(int i = 0; i < N; i++) A[i] *= B[i];
   fft_dit(A.data(), N, +1, R, p, V);
   for(int i = 0; i < N; i++) {
      bs_out[2 * i] = B[i].real(); bs_out[2 * i + 1] = B[i].imag();
      out[2 * i] = A[i].real(); out[2 * i + 1] = A[i].imag();
   }
   return p;
}

}  // extern "C"
