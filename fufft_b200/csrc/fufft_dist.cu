// fufft_dist.cu -- the rank-local outer pass of the distributed single-signal
// convolution.  An n-point transform is viewed as [W][n/W] over W ranks; rank
// g holds columns col0 .. col0+cols-1 of every row (row k at x + k*cols).
// The first DIF pass of radix W at stride n/W has one butterfly group per
// column, so each rank runs it on its own columns with no communication;
// afterwards block (row) k belongs to rank k (one all-to-all), which runs the
// rest of the convolution on n/W points; an all-to-all back and the DIT pass
// finish it.  No reference counterpart: the reference is single-GPU
// (README.md:112); the pass is the flat pass of fufft.cuh:1113-1140 with the
// groups of one rank.
#include <cstring>

#include "fufft_internal.cuh"

namespace fufft {

// W_n^j for j < n <= 2^36 from two exact dyadic sincospif arguments:
// j = jh * 4096 + jl  ->  W_{n/4096}^{jh} * W_n^{jl}
__device__ __forceinline__ float2 twiddle_exact(long long j, long long n)
{
   const long long jh = j >> 12, jl = j & 4095;
   float s1, c1, s2, c2;
   sincospif(-2.0f * (float)jl / (float)n, &s2, &c2);
   if(jh == 0) return make_float2(c2, s2);
   sincospif(-2.0f * (float)jh / (float)(n >> 12), &s1, &c1);
   return cmul(make_float2(c1, s1), make_float2(c2, s2));
}

// the W ranks' block buffers, mapped into this process (peer memory over
// NVLink, this rank's own buffer at its own index)
struct PeerBlocks {
   float2* p[8];
};

// MODE LOCAL: in place on this rank's rows.  PUSH (forward): the outputs of
// row k go straight into rank k's block buffer at this rank's column offset --
// the all-to-all fused into the pass as NVLink stores.  PULL (inverse): the
// inputs of row k come straight from rank k's block buffer (NVLink loads),
// the outputs land in this rank's rows.
enum class DistMode { LOCAL, PUSH, PULL };

template<int W, int S, DistMode MODE>
__global__ void __launch_bounds__(256) dist_pass_kernel(float2* __restrict__ x, long long cols, long long col0,
                                                        long long n, PeerBlocks peers)
{
   for(long long jl = (long long)blockIdx.x * blockDim.x + threadIdx.x; jl < cols;
       jl += (long long)gridDim.x * blockDim.x) {
      float2 u[W], w[W];
#pragma unroll
      for(int k = 0; k < W; ++k) {
         if constexpr(MODE == DistMode::PULL) u[k] = peers.p[k][col0 + jl];
         else u[k] = ld_stream(x + k * cols + jl);
      }
      const long long j = col0 + jl;
      if(j) {
         twiddle_powers<W>(twiddle_exact(j, n), w);
      } else {
#pragma unroll
         for(int k = 1; k < W; ++k) w[k] = make_float2(1.0f, 0.0f);
      }
      if constexpr(S > 0) {
#pragma unroll
         for(int k = 1; k < W; ++k) u[k] = cmulc(u[k], w[k]);
      }
      dft<W, S>(u);
      if constexpr(S < 0) {
#pragma unroll
         for(int k = 1; k < W; ++k) u[k] = cmul(u[k], w[k]);
      }
#pragma unroll
      for(int k = 0; k < W; ++k) {
         if constexpr(MODE == DistMode::PUSH) peers.p[k][col0 + jl] = u[k];
         else st_stream(x + k * cols + jl, u[k]);
      }
   }
}

}  // namespace fufft

using namespace fufft;
using namespace fufft::host;

namespace {

template<DistMode MODE>
fufft_status dist_launch(float* x_local, const uint64_t* peer_blocks, int world, int64_t cols, int64_t col0,
                         int64_t n, int sign, fufft_stream_t stream)
{
   if(!x_local) return FUFFT_ERR_INVALID_ARG;
   if(world != 2 && world != 4 && world != 8) return FUFFT_ERR_UNSUPPORTED;
   if(sign != -1 && sign != 1) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(n) || n > (1LL << 36) || cols <= 0 || col0 < 0 || col0 + cols > n / world) return FUFFT_ERR_INVALID_SIZE;
   if(!aligned(x_local, 8)) return FUFFT_ERR_MISALIGNED;
   PeerBlocks peers{};
   if constexpr(MODE != DistMode::LOCAL) {
      if(!peer_blocks) return FUFFT_ERR_INVALID_ARG;
      for(int k = 0; k < world; ++k) {
         if(!peer_blocks[k]) return FUFFT_ERR_PEER_UNAVAILABLE;
         if(peer_blocks[k] % 8) return FUFFT_ERR_MISALIGNED;
         peers.p[k] = reinterpret_cast<float2*>(peer_blocks[k]);
      }
   }
   int dev = 0;
   fufft_status s = check(cudaGetDevice(&dev));
   if(s != FUFFT_OK) return s;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   const long long blocks = std::min<long long>((cols + 255) / 256, (long long)sm_count(dev) * 8);
   float2* x = reinterpret_cast<float2*>(x_local);
#define FUFFT_DP(WW)                                                                                       \
   if(world == WW) {                                                                                       \
      if(sign < 0) dist_pass_kernel<WW, -1, MODE><<<(unsigned)blocks, 256, 0, st>>>(x, cols, col0, n, peers); \
      else dist_pass_kernel<WW, +1, MODE><<<(unsigned)blocks, 256, 0, st>>>(x, cols, col0, n, peers);        \
   }
   FUFFT_DP(2) FUFFT_DP(4) FUFFT_DP(8)
#undef FUFFT_DP
   count_launch();
   return check(cudaGetLastError());
}

}  // namespace

extern "C" {

fufft_status fufft_dist_pass(float* x_local, int world, int64_t cols, int64_t col0, int64_t n, int sign,
                             fufft_stream_t stream)
{
   return dist_launch<DistMode::LOCAL>(x_local, nullptr, world, cols, col0, n, sign, stream);
}

fufft_status fufft_dist_pass_push(const float* x_local, const uint64_t* peer_blocks, int world, int rank,
                                  int64_t cols, int64_t n, fufft_stream_t stream)
{
   if(rank < 0 || rank >= world) return FUFFT_ERR_INVALID_ARG;
   return dist_launch<DistMode::PUSH>(const_cast<float*>(x_local), peer_blocks, world, cols, rank * cols, n, -1,
                                      stream);
}

fufft_status fufft_dist_pass_pull(float* x_local, const uint64_t* peer_blocks, int world, int rank, int64_t cols,
                                  int64_t n, fufft_stream_t stream)
{
   if(rank < 0 || rank >= world) return FUFFT_ERR_INVALID_ARG;
   return dist_launch<DistMode::PULL>(x_local, peer_blocks, world, cols, rank * cols, n, +1, stream);
}

// ---- device buffers other processes of the node can map (CUDA IPC) --------
fufft_status fufft_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle)
{
   if(!bytes || !dev_ptr || !ipc_handle) return FUFFT_ERR_INVALID_ARG;
   static_assert(sizeof(cudaIpcMemHandle_t) == FUFFT_IPC_HANDLE_BYTES, "IPC handle size");
   void* p = nullptr;
   fufft_status s = check(cudaMalloc(&p, bytes));
   if(s != FUFFT_OK) return s;
   cudaIpcMemHandle_t h;
   if((s = check(cudaIpcGetMemHandle(&h, p))) != FUFFT_OK) {
      cudaFree(p);
      return s;
   }
   memcpy(ipc_handle, &h, sizeof(h));
   *dev_ptr = p;
   return FUFFT_OK;
}

fufft_status fufft_peer_open(const void* ipc_handle, void** dev_ptr)
{
   if(!ipc_handle || !dev_ptr) return FUFFT_ERR_INVALID_ARG;
   cudaIpcMemHandle_t h;
   memcpy(&h, ipc_handle, sizeof(h));
   void* p = nullptr;
   const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
   if(e != cudaSuccess) {
      cuda_fail(e);
      return FUFFT_ERR_PEER_UNAVAILABLE;
   }
   *dev_ptr = p;
   return FUFFT_OK;
}

fufft_status fufft_peer_close(void* dev_ptr)
{
   if(!dev_ptr) return FUFFT_ERR_INVALID_ARG;
   return check(cudaIpcCloseMemHandle(dev_ptr));
}

fufft_status fufft_peer_free(void* dev_ptr)
{
   if(!dev_ptr) return FUFFT_ERR_INVALID_ARG;
   return check(cudaFree(dev_ptr));
}

}  // extern "C"
