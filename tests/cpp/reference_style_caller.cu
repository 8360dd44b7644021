// A reference-style caller of the C++ policy-struct layer (include/fufft_b200.hpp):
// the call sites of bench_fufft.cu rewritten against fufft_b200.  Built by
// tests/test_cpp_layer.py; on a GPU it runs every entry point once on a small
// batch and writes the results for the test to compare with the oracle.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "fufft_b200.hpp"

using namespace fufft_b200;

#define OK(x) do { fufft_status s_ = (x); if(s_ != FUFFT_OK) { \
   fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, fufft_status_string(s_)); return 1; } } while(0)

static int dump(const char* dir, const char* name, const void* d, size_t bytes)
{
   std::vector<char> h(bytes);
   if(cudaMemcpy(h.data(), d, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
   char path[512];
   snprintf(path, sizeof path, "%s/%s.bin", dir, name);
   FILE* f = fopen(path, "wb");
   if(!f) return 1;
   fwrite(h.data(), 1, bytes, f);
   fclose(f);
   return 0;
}

static int load(const char* dir, const char* name, void* d, size_t bytes)
{
   std::vector<char> h(bytes);
   char path[512];
   snprintf(path, sizeof path, "%s/%s.bin", dir, name);
   FILE* f = fopen(path, "rb");
   if(!f || fread(h.data(), 1, bytes, f) != bytes) return 1;
   fclose(f);
   return cudaMemcpy(d, h.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess;
}

int main(int argc, char** argv)
{
   if(argc < 2) { fprintf(stderr, "usage: %s <dir with a.bin b8.bin b16.bin bp16.bin>\n", argv[0]); return 2; }
   const char* dir = argv[1];
   constexpr int N = 4096, L8 = 1, NR8 = 4, L16 = 1, NR16 = 3, CPB = 1;
   const long long batch = 3;
   const size_t bytes = (size_t)N * batch * sizeof(float2);
   float2 *a, *b8, *b16, *bp16, *out;
   for(float2** p : {&a, &b8, &b16, &bp16, &out})
      if(cudaMalloc(p, bytes) != cudaSuccess) return 1;
   if(load(dir, "a", a, bytes) || load(dir, "b8", b8, bytes) || load(dir, "b16", b16, bytes) ||
      load(dir, "bp16", bp16, bytes)) return 1;
   OK((fufft_pipeline_ip<N, L8, NR8, CPB>(a, out, MidMultiply{b8}, nullptr, batch)));
   if(dump(dir, "out_ip", out, bytes)) return 1;
   OK((fufft_pipeline_ip<N, L8, NR8, CPB>(a, out, MidConjMultiply{b8}, nullptr, batch)));
   if(dump(dir, "out_ip_conj", out, bytes)) return 1;
   OK((fufft_pipeline_v16<N, L16, NR16, CPB>(a, out, MidMultiply{b16}, nullptr, batch)));
   if(dump(dir, "out_v16", out, bytes)) return 1;
   OK((fufft_pipeline_v16f<N, L16, NR16, CPB>(a, bp16, out, nullptr, batch)));
   if(dump(dir, "out_v16f", out, bytes)) return 1;
   OK((fufft_c2c<N, 4, CPB>(a, out, nullptr, batch)));   // Mode A: natural-order forward DFT
   if(dump(dir, "out_c2c", out, bytes)) return 1;
   if(cudaDeviceSynchronize() != cudaSuccess) return 1;
   printf("ok\n");
   return 0;
}
