// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own CPU transcription (verify_kernel.cpp of
// weiwang217/FuFFT, included from the read-only reference tree at build time,
// never copied) into oracle/_ref/libfufft_ref.so and gives its static
// functions a C ABI, so that:
//   * tests/golden/make_golden.py can record golden input/output vectors
//     produced by the reference itself;
//   * the C restatement in fufft_oracle.c can be pinned against it;
//   * bench.py --impl reference can time the reference's own CPU path.
// The wrappers below only convert between interleaved float arrays and the
// std::vector<std::complex<float>> the reference functions take; they do not
// touch the arithmetic.  The input generators replay the seeded mt19937
// recipes of the reference's tests so the goldens are the reference's cases.
#define main fufft_reference_verify_main
#include "verify_kernel.cpp"
#undef main

#include <cstdint>
#include <cstring>

namespace {
std::vector<cf> to_cf(const float* p, size_t n)
{
   std::vector<cf> v(n);
   for(size_t i = 0; i < n; i++) v[i] = cf(p[2 * i], p[2 * i + 1]);
   return v;
}
void from_cf(const std::vector<cf>& v, float* p)
{
   for(size_t i = 0; i < v.size(); i++) { p[2 * i] = v[i].real(); p[2 * i + 1] = v[i].imag(); }
}
}  // namespace

extern "C" {

// the reference's whole suite (verify_kernel.cpp:1412-1469); 0 means ALL PASS
int ref_run_suite(void) { return fufft_reference_verify_main(); }

int ref_mixedrev(int idx, int lead, int nr8) { return mixedrev(idx, lead, nr8); }
int ref_mixedrev16(int idx, int lead, int nr16) { return mixedrev16(idx, lead, nr16); }
int ref_chain_rev(int idx, const int* radices, int nrad)
{
   return chain_rev(idx, std::vector<int>(radices, radices + nrad));
}

void ref_pipeline_ip(int N, int CPB, const float* a, const float* b_dr, float* out, int batch)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_ip(N, LEAD, NR8, CPB, CPP_OPT, to_cf(a, n), to_cf(b_dr, n), o, batch);
   from_cf(o, out);
}

void ref_pipeline_fused(int N, int CPB, const float* a, const float* bperm, float* out, int batch)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_fused(N, LEAD, NR8, CPB, to_cf(a, n), to_cf(bperm, n), o, batch);
   from_cf(o, out);
}

void ref_pipeline_v16(int N, int CPB, const float* a, const float* b16, float* out, int batch)
{
   int L16, NR16; factorise16(N, L16, NR16);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_v16(N, L16, NR16, CPB, CPP_OPT, to_cf(a, n), to_cf(b16, n), o, batch);
   from_cf(o, out);
}

void ref_pipeline_v16f(int N, int CPB, const float* a, const float* bp16, float* out, int batch)
{
   int L16, NR16; factorise16(N, L16, NR16);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_v16f(N, L16, NR16, CPB, CPP_OPT, to_cf(a, n), to_cf(bp16, n), o, batch);
   from_cf(o, out);
}

void ref_pipeline_r16(int N, int CPB, const float* a, const float* b16, float* out, int batch)
{
   int L16, NR16; factorise16(N, L16, NR16);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_r16(N, L16, NR16, CPB, CPP_OPT, to_cf(a, n), to_cf(b16, n), o, batch);
   from_cf(o, out);
}

// natural-order forward c2c (Mode A, radix-8 Stockham; N a power of 8)
void ref_c2c(int N, int CPB, const float* a, float* out, int batch)
{
   const int LOG8N = [](int n) { int s = 0; while(n > 1) { n /= 8; s++; } return s; }(N);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_c2c(N, LOG8N, CPB, CPP_OPT, to_cf(a, n), o, batch);
   from_cf(o, out);
}

void ref_pipeline_fwd(int N, int CPB, const float* a, float* spec, int batch)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_fwd(N, LEAD, NR8, CPB, CPP_OPT, to_cf(a, n), o, batch);
   from_cf(o, spec);
}

void ref_pipeline_apply(int N, int CPB, const float* spec, const float* b_dr, float* out, int batch)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   const size_t n = (size_t)N * batch;
   std::vector<cf> o;
   kernel_pipeline_apply(N, LEAD, NR8, CPB, CPP_OPT, to_cf(spec, n), to_cf(b_dr, n), o, batch);
   from_cf(o, out);
}

void ref_conv_r2(int N, int CPB, const float* xr, const float* yr, const float* b_dr,
                 float* ur, float* vr, int batch)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   const size_t n = (size_t)N * batch;
   std::vector<float> x(xr, xr + n), y(yr, yr + n), u, v;
   kernel_conv_r2(N, LEAD, NR8, CPB, CPP_OPT, x, y, to_cf(b_dr, n), u, v, batch);
   std::memcpy(ur, u.data(), n * sizeof(float));
   std::memcpy(vr, v.data(), n * sizeof(float));
}

void ref_conv2d(int H, int W, const float* a, const float* b_dr, float* out, int batch)
{
   const size_t n = (size_t)H * W * batch;
   std::vector<cf> o;
   kernel_conv2d(H, W, CPP_OPT, to_cf(a, n), to_cf(b_dr, n), o, batch);
   from_cf(o, out);
}

void ref_bfp_quantize(const float* x, int N, int16_t* q, float* scale)
{
   const std::vector<cf> v = to_cf(x, N);
   BfpQuant r = bfp_quantize(v.data(), N);
   for(int i = 0; i < N; i++) { q[2 * i] = r.qre[i]; q[2 * i + 1] = r.qim[i]; }
   *scale = r.scale;
}

// one transform (the reference's BFP transcription is per transform)
void ref_v16_bfp(int N, const int16_t* aq, float as, const int16_t* bq, float bs,
                 int16_t* oq, float* os)
{
   int L16, NR16; factorise16(N, L16, NR16);
   BfpQuant qa, qb, qo;
   qa.qre.resize(N); qa.qim.resize(N); qb.qre.resize(N); qb.qim.resize(N);
   for(int i = 0; i < N; i++) {
      qa.qre[i] = aq[2 * i]; qa.qim[i] = aq[2 * i + 1];
      qb.qre[i] = bq[2 * i]; qb.qim[i] = bq[2 * i + 1];
   }
   qa.scale = as; qb.scale = bs;
   kernel_v16_bfp(N, L16, NR16, CPP_OPT, qa, qb, qo);
   for(int i = 0; i < N; i++) { oq[2 * i] = qo.qre[i]; oq[2 * i + 1] = qo.qim[i]; }
   *os = qo.scale;
}

void ref_foursteps_cfg(int N, int batch, int R_OUT, int MID, int v16_mid, float* A, const float* b_dr)
{
   const size_t n = (size_t)N * batch;
   std::vector<cf> v = to_cf(A, n);
   conv_foursteps_cfg(v, to_cf(b_dr, n), N, batch, CPP_OPT, R_OUT, MID, v16_mid != 0);
   from_cf(v, A);
}

void ref_monolithic_cfg(int N, int batch, int R_OUT, int MID, int v16_mid, float* A, const float* b_dr)
{
   const size_t n = (size_t)N * batch;
   std::vector<cf> v = to_cf(A, n);
   conv_monolithic_cfg(v, to_cf(b_dr, n), N, batch, CPP_OPT, R_OUT, MID, v16_mid != 0);
   from_cf(v, A);
}

void ref_fft2_f64(double* x, int n, int sign)
{
   std::vector<cd> v(n);
   for(int i = 0; i < n; i++) v[i] = cd(x[2 * i], x[2 * i + 1]);
   fft2_f64(v, sign);
   for(int i = 0; i < n; i++) { x[2 * i] = v[i].real(); x[2 * i + 1] = v[i].imag(); }
}

// ---- seeded inputs of the reference's tests ------------------------------

// test(): verify_kernel.cpp:1277-1286
void ref_gen_test(int N, int CPB, int batch, float* a, float* b)
{
   std::mt19937 rng(N * 131 + CPB);
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   const float invN = 1.0f / (float)N;
   // the reference's own expressions: the order in which the compiler draws
   // the two constructor arguments is part of the recipe
   for(size_t i = 0; i < (size_t)N * batch; i++) {
      const cf av = cf(d(rng), d(rng));
      const cf bv = cf(d(rng) * invN, d(rng) * invN);
      a[2 * i] = av.real(); a[2 * i + 1] = av.imag();
      b[2 * i] = bv.real(); b[2 * i + 1] = bv.imag();
   }
}

// the raw d(rng) stream of std::uniform_real_distribution<float>(-1, 1) over
// std::mt19937(seed), to pin the oracle's generator
void ref_uniform_stream(unsigned seed, int count, float* out)
{
   std::mt19937 rng(seed);
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   for(int i = 0; i < count; i++) out[i] = d(rng);
}

// test_bfp(): verify_kernel.cpp:1142-1149
void ref_gen_bfp(int N, int seed, float* a, float* b)
{
   std::mt19937 rng(seed * 991 + N);
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   const float invN = 1.0f / (float)N;
   for(int i = 0; i < N; i++) {
      const cf av = cf(d(rng), d(rng));
      const cf bv = cf(d(rng) * invN, d(rng) * invN);
      a[2 * i] = av.real(); a[2 * i + 1] = av.imag();
      b[2 * i] = bv.real(); b[2 * i + 1] = bv.imag();
   }
}

// test_r2(): verify_kernel.cpp:620-639 -- signals, the real filter's taps and
// its fp64 spectrum /N in the radix-8 chain order, rounded to fp32
void ref_gen_r2(int N, int batch, float* xr, float* yr, float* h_taps, float* b_dr)
{
   int LEAD, NR8; factorise(N, LEAD, NR8);
   std::mt19937 rng(N * 77 + 5);
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   const size_t n = (size_t)N * batch;
   std::vector<cd> h(N);
   for(size_t i = 0; i < n; i++) { xr[i] = d(rng); yr[i] = d(rng); }
   for(int i = 0; i < N; i++) { h[i] = cd((double)d(rng), 0.0); h_taps[i] = (float)h[i].real(); }
   std::vector<cd> H;
   ref_dft(h, H, -1);
   for(int t = 0; t < batch; t++)
      for(int i = 0; i < N; i++) {
         const cd v = H[mixedrev(i, LEAD, NR8)] / (double)N;
         b_dr[2 * ((size_t)t * N + i)] = (float)v.real();
         b_dr[2 * ((size_t)t * N + i) + 1] = (float)v.imag();
      }
}

// test_2d(): verify_kernel.cpp:727-737
void ref_gen_2d(int H, int W, int batch, float* a, float* b)
{
   std::mt19937 rng(H * 131 + W);
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   const float invN = 1.0f / (float)(H * W);
   for(size_t i = 0; i < (size_t)H * W * batch; i++) {
      const cf av = cf(d(rng), d(rng));
      const cf bv = cf(d(rng) * invN, d(rng) * invN);
      a[2 * i] = av.real(); a[2 * i + 1] = av.imag();
      b[2 * i] = bv.real(); b[2 * i + 1] = bv.imag();
   }
}

// test_large_cfg(): verify_kernel.cpp:487-496
void ref_gen_large_cfg(int N, int batch, int R_OUT, int MID, float* a, float* b)
{
   std::mt19937 rng(N ^ (R_OUT * 7919) ^ (MID * 104729));
   std::uniform_real_distribution<float> d(-1.0f, 1.0f);
   const float invN = 1.0f / (float)N;
   for(size_t i = 0; i < (size_t)N * batch; i++) {
      const cf av = cf(d(rng), d(rng));
      const cf bv = cf(d(rng) * invN, d(rng) * invN);
      a[2 * i] = av.real(); a[2 * i + 1] = av.imag();
      b[2 * i] = bv.real(); b[2 * i + 1] = bv.imag();
   }
}

}  // extern "C"
