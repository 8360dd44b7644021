// fufft_cluster.cu -- launches of the cluster-fused convolution
// (fufft_cluster.cuh): 1-D n = 16384 / 32768 / 65536 on the radix-16 chain,
// the four-step with one outer level (n = r_out * mid), and 2-D images
// beyond one CTA (128x128 .. 256x256, 128x512).
#include "fufft_cluster.cuh"
#include "fufft_internal.cuh"

namespace fufft {
namespace host {

template<class Inner, int C, int OUT_L, int OUT_SHIFT, Mid MID, Flt FLT, bool BFP = false>
static fufft_status launch_cluster(const ConvArgs& args, cudaStream_t st, int device)
{
   using K = ClusterConv<Inner, C, OUT_L, OUT_SHIFT, MID, FLT, BFP>;
   auto kern = conv_cluster_kernel<Inner, C, OUT_L, OUT_SHIFT, MID, FLT, BFP>;
   static std::atomic<uint64_t> configured{0}, usable{0};
   static std::atomic<int> wave[64];   // clusters resident at once
   const uint64_t bit = 1ull << (device & 63);
   cudaLaunchConfig_t cfg = {};
   cudaLaunchAttribute attr[1];
   attr[0].id = cudaLaunchAttributeClusterDimension;
   attr[0].val.clusterDim.x = C;
   attr[0].val.clusterDim.y = 1;
   attr[0].val.clusterDim.z = 1;
   cfg.blockDim = dim3(K::THREADS);
   cfg.dynamicSmemBytes = K::SMEM;
   cfg.stream = st;
   cfg.attrs = attr;
   cfg.numAttrs = 1;
   if(!(configured.load(std::memory_order_acquire) & bit)) {
      fufft_status s = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM));
      if(s != FUFFT_OK) return s;
      if(C > 8) {
         s = check(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
         if(s != FUFFT_OK) return s;
      }
      cfg.gridDim = dim3(C);
      int nclusters = 0;
      if(cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) != cudaSuccess) {
         cudaGetLastError();
         nclusters = 0;
      }
      if(nclusters > 0) usable.fetch_or(bit);
      wave[device & 63].store(nclusters);
      configured.fetch_or(bit, std::memory_order_acq_rel);
   }
   if(!(usable.load() & bit)) return FUFFT_ERR_UNSUPPORTED;
   cfg.gridDim = dim3((unsigned)(args.batch * C));
#ifndef FUFFT_CLUSTER_L2_PREFETCH
#define FUFFT_CLUSTER_L2_PREFETCH 1
#endif
   // L2 prefetch one cluster wave ahead, for launches of eight waves or more;
   // the bulk prefetches want 16-byte aligned rows
   ConvArgs a2 = args;
   const int w = wave[device & 63].load();
   const int eb = BFP ? 4 : 8;
   if(FUFFT_CLUSTER_L2_PREFETCH && w > 0 && args.batch >= 8LL * w && aligned(args.a, 16) &&
      (K::B / C) * eb % 16 == 0 && (MID == Mid::NONE || (aligned(args.b, 16) && args.filter_stride % 4 == 0)))
      a2.prefetch_ahead = w;
   fufft_status s = check(cudaLaunchKernelEx(&cfg, kern, a2));
   if(s == FUFFT_OK) count_launch();
   return s;
}

// register-boundary-ordered filters are read coalesced from global memory at
// the boundary (Flt::BP_DIRECT) rather than copied to shared memory first: the
// copy's B * 8 bytes would leave room for only two CTAs of B = 4096 per SM
#ifndef FUFFT_CLUSTER_BP_DIRECT
#define FUFFT_CLUSTER_BP_DIRECT 1
#endif
constexpr Flt CLUSTER_BP = FUFFT_CLUSTER_BP_DIRECT ? Flt::BP_DIRECT : Flt::SMEM;

template<class Inner, int C, int OUT_L, int OUT_SHIFT, bool BFP = false>
static fufft_status cluster_mid(fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   switch(mid) {
   case FUFFT_MID_NONE: return launch_cluster<Inner, C, OUT_L, OUT_SHIFT, Mid::NONE, Flt::NONE, BFP>(a, st, dev);
   case FUFFT_MID_MULTIPLY:
      return bperm ? launch_cluster<Inner, C, OUT_L, OUT_SHIFT, Mid::MUL, CLUSTER_BP, BFP>(a, st, dev)
                   : launch_cluster<Inner, C, OUT_L, OUT_SHIFT, Mid::MUL, Flt::GLOBAL, BFP>(a, st, dev);
   case FUFFT_MID_CONJ_MULTIPLY:
      return bperm ? launch_cluster<Inner, C, OUT_L, OUT_SHIFT, Mid::CONJ, CLUSTER_BP, BFP>(a, st, dev)
                   : launch_cluster<Inner, C, OUT_L, OUT_SHIFT, Mid::CONJ, Flt::GLOBAL, BFP>(a, st, dev);
   }
   return FUFFT_ERR_INVALID_ARG;
}

// 1-D on the radix-16 chain [C, 16, 16, 16]
fufft_status cluster_conv1d(int n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   switch(n) {
   case 16384: return cluster_mid<Chain<4096, 16>, 4, 16384, 0>(mid, bperm, a, st, dev);
   case 32768: return cluster_mid<Chain<4096, 16>, 8, 32768, 0>(mid, bperm, a, st, dev);
   case 65536: return cluster_mid<Chain<4096, 16>, 16, 65536, 0>(mid, bperm, a, st, dev);
   }
   return FUFFT_ERR_UNSUPPORTED;
}

// four-step with one outer level: chain [r_out] ++ chain(mid, 16)
fufft_status cluster_large(int r_out, int mid_n, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st,
                           int dev)
{
   if(r_out == 16 && mid_n == 2048) return cluster_mid<Chain<2048, 16>, 16, 32768, 0>(mid, bperm, a, st, dev);
   if(r_out == 8 && mid_n == 2048) return cluster_mid<Chain<2048, 16>, 8, 16384, 0>(mid, bperm, a, st, dev);
   if(r_out == 16 && mid_n == 4096) return cluster_mid<Chain<4096, 16>, 16, 65536, 0>(mid, bperm, a, st, dev);
   if(r_out == 8 && mid_n == 4096) return cluster_mid<Chain<4096, 16>, 8, 32768, 0>(mid, bperm, a, st, dev);
   return FUFFT_ERR_UNSUPPORTED;
}

// the same four-step shapes with int16-BFP signal, filter and result
fufft_status cluster_large_bfp(int r_out, int mid_n, fufft_midop mid, bool bperm, const ConvArgs& a,
                               cudaStream_t st, int dev)
{
   if(r_out == 16 && mid_n == 2048) return cluster_mid<Chain<2048, 16>, 16, 32768, 0, true>(mid, bperm, a, st, dev);
   if(r_out == 8 && mid_n == 2048) return cluster_mid<Chain<2048, 16>, 8, 16384, 0, true>(mid, bperm, a, st, dev);
   if(r_out == 16 && mid_n == 4096) return cluster_mid<Chain<4096, 16>, 16, 65536, 0, true>(mid, bperm, a, st, dev);
   if(r_out == 8 && mid_n == 4096) return cluster_mid<Chain<4096, 16>, 8, 32768, 0, true>(mid, bperm, a, st, dev);
   return FUFFT_ERR_UNSUPPORTED;
}

// 2-D: outer = the first column pass (radix C, per-column stride m = H/C)
fufft_status cluster_conv2d(int h, int w, fufft_midop mid, bool bperm, const ConvArgs& a, cudaStream_t st, int dev)
{
   if(h == 128 && w == 128) return cluster_mid<Chain2<16, 128, 16>, 8, 128, 7>(mid, bperm, a, st, dev);
   if(h == 256 && w == 128) return cluster_mid<Chain2<16, 128, 16>, 16, 256, 7>(mid, bperm, a, st, dev);
   if(h == 128 && w == 256) return cluster_mid<Chain2<16, 256, 16>, 8, 128, 8>(mid, bperm, a, st, dev);
   if(h == 256 && w == 256) return cluster_mid<Chain2<16, 256, 16>, 16, 256, 8>(mid, bperm, a, st, dev);
   if(h == 128 && w == 512) return cluster_mid<Chain2<16, 512, 16>, 8, 128, 9>(mid, bperm, a, st, dev);
   return FUFFT_ERR_UNSUPPORTED;
}

bool cluster_conv2d_shape(int h, int w)
{
   return (h == 128 && (w == 128 || w == 256 || w == 512)) || (h == 256 && (w == 128 || w == 256));
}

}  // namespace host
}  // namespace fufft
