// fufft_stream.cuh -- persistent, TMA-pipelined form of the fused
// convolution for fp32 and int16-BFP storage.
//
// Each CTA stays resident and walks its share of the batch (group g =
// blockIdx.x, +gridDim.x, ...; a group is CPB transforms).  While it computes
// group g it already has the signal of the next group in flight:
//   * the signal arrives by 2-D TMA tensor loads (128-byte rows,
//     SWIZZLE_128B) into one of two stage buffers; the hardware swizzle is
//     the exchange swizzle (Swz128), so for fp32 the stage buffer becomes the
//     exchange buffer in place and the first DIF pass reads it conflict-free;
//   * the filter has one buffer, reloaded by TMA for the next group as soon
//     as every thread has passed the register boundary (after the first
//     inverse exchange), so its latency hides under half a transform of work
//     on each side;
//   * the result leaves from registers with coalesced streaming stores.
// HBM latency is therefore never on the critical path of a CTA; what is left
// is the butterfly arithmetic and the shared-memory exchanges.
#pragma once
#include "fufft_conv.cuh"

namespace fufft {

// word (4-byte) index -> slot under the same 128-byte swizzle
__device__ __forceinline__ int swz128w(int e) { return e ^ (((e >> 5) & 7) << 2); }

template<int N, int R, int CPB, bool BFP, Mid MID, bool FLIN>
struct StreamKernel {
   using C = Chain<N, R>;
   static constexpr int T = C::T;
   static constexpr int THREADS = CPB * T;
   static constexpr int EB = BFP ? 4 : 8;                       // staged bytes per point
   static constexpr bool HAS_F = MID != Mid::NONE;
   static constexpr size_t STAGE = (size_t)CPB * N * EB;
   static constexpr size_t XB = BFP ? (size_t)CPB * N * 8 : 0;   // BFP: separate fp32 exchange buffer
   static constexpr size_t FB = HAS_F ? (size_t)CPB * N * EB : 0;
   static constexpr size_t SMEM = 2 * STAGE + XB + FB + 1024;    // + slack to align the base to 1 KB
   static constexpr int ROWS_SLOT = N * EB / 128;                // 128-byte rows per transform
   static constexpr int SIG_ROWS = CPB * ROWS_SLOT;              // rows per group (contiguous)
   static constexpr int SIG_BOX = SIG_ROWS < 256 ? SIG_ROWS : 256;
   static constexpr int FLT_BOX = ROWS_SLOT < 256 ? ROWS_SLOT : 256;
   static_assert(N * EB >= 128, "one transform must fill at least one 128-byte row");
   static_assert(STAGE % 1024 == 0 && XB % 1024 == 0, "1 KB aligned buffers (swizzle period)");

   // one thread: the signal rows of group g into stage buffer `dst`
   __device__ __forceinline__ static void issue_signal(const CUtensorMap* tm, long long g, void* dst, uint64_t* bar)
   {
      mbar_expect_tx(bar, (uint32_t)(SIG_ROWS * 128));
#pragma unroll 1
      for(int r = 0; r < SIG_ROWS; r += SIG_BOX)
         tma_load_2d(static_cast<unsigned char*>(dst) + (size_t)r * 128, tm, 0, (int)(g * SIG_ROWS + r), bar);
   }
   // one thread: each slot's filter (rows of transform t start at t*fstride_rows)
   __device__ __forceinline__ static void issue_filter(const CUtensorMap* tm, long long g, long long fstride_rows,
                                                       void* dst, uint64_t* bar)
   {
      mbar_expect_tx(bar, (uint32_t)(CPB * ROWS_SLOT * 128));
#pragma unroll 1
      for(int s = 0; s < CPB; ++s)
#pragma unroll 1
         for(int r = 0; r < ROWS_SLOT; r += FLT_BOX)
            tma_load_2d(static_cast<unsigned char*>(dst) + ((size_t)s * ROWS_SLOT + r) * 128, tm, 0,
                        (int)((g * CPB + s) * fstride_rows + r), bar);
   }

   template<int p>
   __device__ __forceinline__ static void fwd_step(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                   const float2* tw)
   {
      sched_fence();
      if constexpr(p > 0) {
         xstore<C, p - 1, Swz128>(X, off, x, lane);
         slot_sync<T, CPB>(slot);
         xload<C, p, Swz128>(X, off, x, lane);
      }
      butterflies<C, p, -1>(x, lane, tw);
   }
   template<int p, class Hook>
   __device__ __forceinline__ static void inv_step(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                   const float2* tw, Hook& hook)
   {
      sched_fence();
      if constexpr(p < C::NP - 1) {
         xstore<C, p + 1, Swz128>(X, off, x, lane);
         slot_sync<T, CPB>(slot);
         if constexpr(p == C::NP - 2) hook();   // first inverse exchange: everyone is past the boundary
         xload<C, p, Swz128>(X, off, x, lane);
      }
      butterflies<C, p, +1>(x, lane, tw);
   }
   template<int... ps>
   __device__ __forceinline__ static void fwd_all(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                  const float2* tw, std::integer_sequence<int, ps...>)
   {
      (fwd_step<ps>(X, off, x, lane, slot, tw), ...);
   }
   template<class Hook, int... ps>
   __device__ __forceinline__ static void inv_all(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                  const float2* tw, Hook& hook, std::integer_sequence<int, ps...>)
   {
      (inv_step<C::NP - 1 - ps>(X, off, x, lane, slot, tw, hook), ...);
   }

   __device__ __forceinline__ static void run(const CUtensorMap* tm_a, const CUtensorMap* tm_b, const ConvArgs& args,
                                              long long ngroups)
   {
      extern __shared__ unsigned char smem_dyn[];
      __shared__ uint64_t bar_s[2], bar_f;
      __shared__ float warp_max[THREADS / 32 > 0 ? THREADS / 32 : 1];
      unsigned char* base = reinterpret_cast<unsigned char*>(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
      unsigned char* stage[2] = {base, base + STAGE};
      float2* Xb = reinterpret_cast<float2*>(base + 2 * STAGE);
      unsigned char* F = base + 2 * STAGE + XB;

      const int tid = threadIdx.x;
      const int slot = tid / T, lane = tid % T;
      const int off = slot * N;
      const long long fstride_rows = args.filter_stride * EB / 128;

      if(tid == 0) {
         prefetch_tmap(tm_a);
         if constexpr(HAS_F) prefetch_tmap(tm_b);
         mbar_init(&bar_s[0], 1);
         mbar_init(&bar_s[1], 1);
         mbar_init(&bar_f, 1);
         fence_mbar_init();
      }
      __syncthreads();
      if(tid == 0 && (long long)blockIdx.x < ngroups) {
         issue_signal(tm_a, blockIdx.x, stage[0], &bar_s[0]);
         if constexpr(HAS_F) issue_filter(tm_b, blockIdx.x, fstride_rows, F, &bar_f);
      }

      int it = 0;
#pragma unroll 1
      for(long long g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
         const int st = it & 1;
         const long long gnext = g + gridDim.x;
         // the other stage buffer was last touched (as exchange buffer) by this
         // CTA's threads in the previous group: order those generic accesses
         // before the TMA that refills it
         fence_proxy_async_smem();
         __syncthreads();
         if(tid == 0) {
            if(gnext < ngroups) issue_signal(tm_a, gnext, stage[st ^ 1], &bar_s[st ^ 1]);
            if constexpr(HAS_F && C::NP == 1)
               if(it > 0) issue_filter(tm_b, g, fstride_rows, F, &bar_f);
         }
         const long long tr = g * CPB + slot;
         const bool active = tr < args.batch;
         const size_t gbase = (size_t)tr * N;
         float2* X = BFP ? Xb : reinterpret_cast<float2*>(stage[st]);

         mbar_wait(&bar_s[st], (it >> 1) & 1, args.status);

         // ---- first DIF pass from the staged signal
         float2 x[R];
         constexpr int r0 = C::radix(0), G0 = R / r0;
         float sa = 1.0f;
         if constexpr(BFP) sa = active ? __ldg(args.a_scale + tr) : 0.0f;
#pragma unroll
         for(int s = 0; s < G0; ++s)
#pragma unroll
            for(int k = 0; k < r0; ++k) {
               const int e = off + lane + T * (s + G0 * k);
               if constexpr(BFP)
                  x[s * r0 + k] = bfp_dequant(reinterpret_cast<const uint32_t*>(stage[st])[swz128w(e)], sa);
               else
                  x[s * r0 + k] = reinterpret_cast<const float2*>(stage[st])[Swz128::map(e)];
            }
         fwd_all(X, off, x, lane, slot, args.tw, std::make_integer_sequence<int, C::NP>{});

         // ---- register boundary
         if constexpr(HAS_F) {
            mbar_wait(&bar_f, it & 1, args.status);
            float2 f[R];
            if constexpr(BFP) {
               const uint32_t* Fw = reinterpret_cast<const uint32_t*>(F);
               const float sb = active ? __ldg(args.b_scale + (args.filter_stride ? tr : 0)) : 0.0f;
               if constexpr(FLIN) {
#pragma unroll
                  for(int k = 0; k < R; k += 4) {
                     const uint4 w = *reinterpret_cast<const uint4*>(Fw + swz128w(off + R * lane + k));
                     f[k] = bfp_dequant(w.x, sb); f[k + 1] = bfp_dequant(w.y, sb);
                     f[k + 2] = bfp_dequant(w.z, sb); f[k + 3] = bfp_dequant(w.w, sb);
                  }
               } else {
#pragma unroll
                  for(int k = 0; k < R; ++k) f[k] = bfp_dequant(Fw[swz128w(off + lane + k * T)], sb);
               }
            } else {
               const float2* Ff = reinterpret_cast<const float2*>(F);
               if constexpr(FLIN) {
#pragma unroll
                  for(int k = 0; k < R; k += 2) {
                     const float4 v = *reinterpret_cast<const float4*>(Ff + Swz128::map(off + R * lane + k));
                     f[k] = make_float2(v.x, v.y);
                     f[k + 1] = make_float2(v.z, v.w);
                  }
               } else {
#pragma unroll
                  for(int k = 0; k < R; ++k) f[k] = Ff[Swz128::map(off + lane + k * T)];
               }
            }
#pragma unroll
            for(int k = 0; k < R; ++k) x[k] = (MID == Mid::MUL) ? cmul(x[k], f[k]) : cmulc(x[k], f[k]);
         }

         // refill the filter buffer for the next group once every thread of
         // the CTA has read it (called right after the first inverse exchange
         // barrier; with CPB > 1 that barrier covers one transform only, so a
         // CTA-wide barrier is added)
         auto refill = [&]() {
            if constexpr(HAS_F) {
               if constexpr(CPB > 1) __syncthreads();
               if(tid == 0 && gnext < ngroups) issue_filter(tm_b, gnext, fstride_rows, F, &bar_f);
            }
         };
         inv_all(X, off, x, lane, slot, args.tw, refill, std::make_integer_sequence<int, C::NP>{});

         // ---- last DIT pass straight to HBM
         if constexpr(BFP) {
            float m = 0.0f;
#pragma unroll
            for(int i = 0; i < R; ++i) m = fmaxf(m, fmaxf(fabsf(x[i].x), fabsf(x[i].y)));
            if constexpr(T >= 32) {
#pragma unroll
               for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
               if((tid & 31) == 0) warp_max[tid >> 5] = m;
               slot_sync<T, CPB>(slot);
               m = 0.0f;
#pragma unroll
               for(int w = 0; w < T / 32; ++w) m = fmaxf(m, warp_max[slot * (T / 32) + w]);
            } else {
#pragma unroll
               for(int o = T / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            }
            const float mx = fmaxf(m, 1e-30f);
            const float inv = 32767.0f / mx;
            if(active) {
               uint32_t* o = static_cast<uint32_t*>(args.out);
#pragma unroll
               for(int s = 0; s < G0; ++s)
#pragma unroll
                  for(int k = 0; k < r0; ++k)
                     st_stream(o + gbase + lane + (size_t)T * (s + G0 * k), bfp_quant(x[s * r0 + k], inv));
               if(lane == 0) args.out_scale[tr] = mx / 32767.0f;
            }
         } else if(active) {
#pragma unroll
            for(int s = 0; s < G0; ++s)
#pragma unroll
               for(int k = 0; k < r0; ++k)
                  st_stream(static_cast<float2*>(args.out) + gbase + lane + (size_t)T * (s + G0 * k), x[s * r0 + k]);
         }
      }
   }
};

// two resident 256-thread CTAs per SM (128 registers per thread)
template<int N, int R, int CPB, bool BFP, Mid MID, bool FLIN>
__global__ void __launch_bounds__(CPB * (N / R), (CPB * (N / R) <= 256 ? 2 : 1))
conv_stream_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const ConvArgs args, long long ngroups)
{
   StreamKernel<N, R, CPB, BFP, MID, FLIN>::run(&tm_a, &tm_b, args, ngroups);
}

}  // namespace fufft
