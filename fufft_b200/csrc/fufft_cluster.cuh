// fufft_cluster.cuh -- fused convolution of transforms larger than one SM's
// shared memory, in one kernel and three HBM passes, on a thread-block
// cluster of C CTAs exchanging through distributed shared memory (DSMEM).
//
// The transform of NT = C * B points is seen as C rows of B points (row q =
// positions q*B .. q*B + B-1).  Its radix chain starts with one pass of
// radix C at stride B (the four-step's outer level), which mixes only the C
// points of one column; the rest of the chain works inside rows.  So:
//   1. CTA c loads columns c*B/C .. (c+1)*B/C - 1 of all rows straight from
//      HBM (coalesced) and runs the radix-C DIF pass on them in registers;
//   2. forward exchange: the value of row q goes to CTA q's buffer X by an
//      asynchronous remote store (st.async) that counts its bytes on CTA q's
//      mbarrier -- CTA q waits for its row's bytes, not for the whole cluster;
//   3. CTA q runs the fused one-CTA convolution on its B points (the engine of
//      fufft_conv.cuh: DIF chain, filter block q at the register boundary,
//      DIT chain); the results stay in registers;
//   4. return exchange: each result goes by st.async to the CTA owning its
//      column, into that CTA's buffer Y (a third buffer, so no CTA has to wait
//      for its peers to finish with X or with the filter), counted on a second
//      mbarrier; radix-C DIT pass in registers, coalesced stores.
// Each buffer is written once per kernel, so the only cluster barrier is the
// one at start-up: a relaxed arrive after the mbarriers are initialised
// (fence.mbarrier_init), waited on before the first remote store, which makes
// sure every CTA of the cluster runs and can count bytes before any is sent.
// After the return exchange no CTA touches a peer's memory, and every CTA has
// received all bytes addressed to it before it leaves.
// The filter of the whole transform is in the chain order [C] ++ inner chain;
// its block q is exactly the inner transform's own chain-ordered filter.
// 1-D: N = 16384 (C 4), 32768 (C 8), 65536 (C 16) with B = 4096 and the
// radix-16 chain [C, 16, 16, 16] -- the mixedrev16 order of N;
// the four-step N = r_out * mid (the reference's N=32768 recipe: C = 16,
// B = 2048, chain [16, 8, 16, 16]);
// 2-D: the first column pass is the outer pass (per-column stride H/C,
// twiddle index = row position inside the column group).
// int16-BFP storage (BFP = true, the four-step N = r_out * mid of
// fufft_conv_large_bfp): taps, filter block and result are packed int16 pairs
// with one fp32 scale per transform; the output scale needs the abs-max of the
// whole transform, so each CTA sends its own maximum to every peer (a third
// st.async exchange of 4 bytes per peer) before quantising.
// Every bounded mbarrier wait returns (reporting a timeout in the status
// word), so every thread of every CTA reaches the start-up barrier's wait.
#pragma once
#include "fufft_conv.cuh"

namespace fufft {

__device__ __forceinline__ uint32_t cluster_ctarank()
{
   uint32_t r;
   asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
   return r;
}
__device__ __forceinline__ uint32_t cluster_id_x()
{
   uint32_t r;
   asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
   return r;
}
// split-phase forms: arrive early, wait late, with independent work between
__device__ __forceinline__ void cluster_arrive_relaxed()
{
   asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait()
{
   asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// shared::cta address of this CTA -> the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_remote(uint32_t local_addr, uint32_t rank)
{
   uint32_t r;
   asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
   return r;
}
// asynchronous remote store of 8 bytes, counted on the destination CTA's
// mbarrier `mbar` (a shared::cluster address in that CTA)
__device__ __forceinline__ void st_async(uint32_t addr, float2 v, uint32_t mbar)
{
   asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
                :: "r"(addr), "f"(v.x), "f"(v.y), "r"(mbar) : "memory");
}
// the same for 4 bytes
__device__ __forceinline__ void st_async(uint32_t addr, float v, uint32_t mbar)
{
   asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                :: "r"(addr), "r"(__float_as_uint(v)), "r"(mbar) : "memory");
}

// Inner: the one-CTA chain of a row (Chain2); C: outer radix = CTAs per
// cluster; OUT_L / OUT_SHIFT: the outer pass's twiddle W_{OUT_L}^{(col >> OUT_SHIFT) q}
template<class Inner, int C, int OUT_L, int OUT_SHIFT, Mid MID, Flt FLT, bool BFP = false>
struct ClusterConv {
   using I = Inner;
   static constexpr int B = I::N, R = I::R, T = I::T, G = R / C, NT = C * B;
   static constexpr int THREADS = T;
   static constexpr bool HAS_FILTER = MID != Mid::NONE;
   static constexpr int CB = B / C;   // columns per CTA
   static constexpr int FELEM = BFP ? 4 : 8;   // filter bytes per point
   static constexpr size_t X_BYTES = (size_t)B * sizeof(float2);
   static constexpr size_t F_BYTES = (HAS_FILTER && FLT == Flt::SMEM) ? (size_t)B * FELEM : 0;
   static constexpr size_t Y_BYTES = (size_t)B * sizeof(float2);
   static constexpr size_t SMEM = X_BYTES + F_BYTES + Y_BYTES;
   // bytes each exchange brings into a CTA from its C-1 peers
   static constexpr uint32_t XCHG_BYTES = (uint32_t)((C - 1) * CB * sizeof(float2));
   static_assert(C == 2 || C == 4 || C == 8 || C == 16, "outer radix");
   static_assert(R % C == 0 && (B / C) == G * T, "each thread holds G whole columns");

   template<int p>
   __device__ __forceinline__ static void fwd_step(float2* X, float2 (&x)[R], int lane, const float2* tw)
   {
      sched_fence();
      if constexpr(p > 0) {
         xstore<I, p - 1>(X, 0, x, lane);
         exchange_sync<I, p - 1, 1>(0);
         xload<I, p>(X, 0, x, lane);
      }
      butterflies<I, p, -1>(x, lane, tw);
   }
   template<int p>
   __device__ __forceinline__ static void inv_step(float2* X, float2 (&x)[R], int lane, const float2* tw)
   {
      sched_fence();
      if constexpr(p < I::NP - 1) {
         xstore<I, p + 1>(X, 0, x, lane);
         exchange_sync<I, p, 1>(0);
         xload<I, p>(X, 0, x, lane);
      }
      butterflies<I, p, +1>(x, lane, tw);
   }
   template<int... ps>
   __device__ __forceinline__ static void fwd_all(float2* X, float2 (&x)[R], int lane, const float2* tw,
                                                  std::integer_sequence<int, ps...>)
   {
      (fwd_step<ps>(X, x, lane, tw), ...);
   }
   template<int... ps>
   __device__ __forceinline__ static void inv_all(float2* X, float2 (&x)[R], int lane, const float2* tw,
                                                  std::integer_sequence<int, ps...>)
   {
      (inv_step<I::NP - 1 - ps>(X, x, lane, tw), ...);
   }

   // the outer radix-C pass on this thread's G columns, DIF (S=-1) or DIT (S=+1)
   template<int S>
   __device__ __forceinline__ static void outer(float2 (&x)[R], int c, int lane, const float2* tw)
   {
#pragma unroll
      for(int s = 0; s < G; ++s) {
         float2* u = x + s * C;
         const int col = c * (B / C) + lane + T * s;
         const int j = col >> OUT_SHIFT;
         float2 w[C];
         if constexpr(OUT_L > C) twiddle_powers<C>(__ldca(tw + tw_offset(OUT_L) + (j & (OUT_L / C - 1))), w);
         if constexpr(S > 0 && OUT_L > C) {
#pragma unroll
            for(int q = 1; q < C; ++q) u[q] = cmulc(u[q], w[q]);
         }
         dft<C, S>(u);
         if constexpr(S < 0 && OUT_L > C) {
#pragma unroll
            for(int q = 1; q < C; ++q) u[q] = cmul(u[q], w[q]);
         }
      }
   }

   __device__ __forceinline__ static void run(const ConvArgs& args)
   {
      extern __shared__ __align__(1024) unsigned char smem_raw[];
      // filter copy; forward, return and (BFP) abs-max exchanges
      __shared__ uint64_t fbar, xbar[3];
      __shared__ float cmax[C], wmax[T / 32];
      float2* X = reinterpret_cast<float2*>(smem_raw);
      unsigned char* F = smem_raw + X_BYTES;
      float2* Y = reinterpret_cast<float2*>(smem_raw + X_BYTES + F_BYTES);
      const int lane = threadIdx.x;
      const int c = (int)cluster_ctarank();
      const long long tr = cluster_id_x();
      const size_t gbase = (size_t)tr * NT;

      // ---- mbarriers: initialised and armed (one arrival + the bytes the
      // peers will send) before this CTA announces itself to the cluster
      if(lane == 0) {
         if constexpr(HAS_FILTER && FLT == Flt::SMEM) mbar_init(&fbar, 1);
         mbar_init(&xbar[0], 1);
         mbar_init(&xbar[1], 1);
         if constexpr(BFP) mbar_init(&xbar[2], 1);
         fence_mbar_init();
         mbar_expect_tx(&xbar[0], XCHG_BYTES);
         mbar_expect_tx(&xbar[1], XCHG_BYTES);
         if constexpr(BFP) mbar_expect_tx(&xbar[2], (uint32_t)((C - 1) * sizeof(float)));
      }
      __syncthreads();
      cluster_arrive_relaxed();

      // ---- L2 prefetch: the column slice and filter block of the transform
      // this CTA's slot takes one cluster wave later
      if(lane == 0 && args.prefetch_ahead > 0 && tr + args.prefetch_ahead < args.batch) {
         constexpr uint32_t EB = BFP ? 4 : 8;
         const long long nt = tr + args.prefetch_ahead;
         const unsigned char* a = static_cast<const unsigned char*>(args.a);
#pragma unroll 1
         for(int q = 0; q < C; ++q)
            prefetch_l2_bulk(a + ((size_t)nt * NT + (size_t)q * B + (size_t)c * CB) * EB, (uint32_t)(CB * EB));
         if constexpr(HAS_FILTER)
            if(args.filter_stride != 0)
               prefetch_l2_bulk(static_cast<const unsigned char*>(args.b) +
                                   ((size_t)(nt * args.filter_stride) + (size_t)c * B) * FELEM,
                                (uint32_t)(B * FELEM));
      }

      // ---- this CTA's filter block (row c of the chain order), TMA bulk prefetch
      if constexpr(HAS_FILTER && FLT == Flt::SMEM) {
         if(lane == 0) {
            mbar_expect_tx(&fbar, (uint32_t)(B * FELEM));
            bulk_g2s(F, static_cast<const unsigned char*>(args.b) +
                            ((size_t)(tr * args.filter_stride) + (size_t)c * B) * FELEM,
                     (uint32_t)(B * FELEM), &fbar);
         }
      }

      // ---- 1. outer DIF pass on this CTA's columns, taps straight from HBM
      float2 x[R];
      float sa = 1.0f;
      if constexpr(BFP) sa = __ldg(args.a_scale + tr);
#pragma unroll
      for(int s = 0; s < G; ++s)
#pragma unroll
         for(int q = 0; q < C; ++q) {
            const size_t gi = gbase + (size_t)q * B + c * CB + lane + T * s;
            if constexpr(BFP) x[s * C + q] = bfp_dequant(ld_stream(static_cast<const uint32_t*>(args.a) + gi), sa);
            else x[s * C + q] = ld_stream(static_cast<const float2*>(args.a) + gi);
         }
      outer<-1>(x, c, lane, args.tw);
      cluster_wait();   // every CTA of the cluster runs, its mbarriers armed

      // ---- 2. forward exchange: (row q, column col) -> X of CTA q at col
      {
         const uint32_t xb = smem_u32(X), mb = smem_u32(&xbar[0]);
#pragma unroll
         for(int q = 0; q < C; ++q) {
            const uint32_t rx = map_remote(xb, q), rm = map_remote(mb, q);
#pragma unroll
            for(int s = 0; s < G; ++s) {
               const int col = c * CB + lane + T * s;
               if(q == c) X[col] = x[s * C + q];
               else st_async(rx + (uint32_t)(col * sizeof(float2)), x[s * C + q], rm);
            }
         }
      }
      mbar_wait<true>(&xbar[0], 0, args.status);
      __syncthreads();   // this CTA's own share, written by plain stores

      // ---- 3. the fused one-CTA convolution of row c
      {
         constexpr int r0 = I::radix(0), G0 = R / r0;
#pragma unroll
         for(int s = 0; s < G0; ++s)
#pragma unroll
            for(int k = 0; k < r0; ++k) x[s * r0 + k] = X[lane + T * (s + G0 * k)];
      }
      fwd_all(X, x, lane, args.tw, std::make_integer_sequence<int, I::NP>{});
      if constexpr(HAS_FILTER) {
         float2 f[R];
         float sb = 1.0f;
         if constexpr(BFP) sb = __ldg(args.b_scale + (args.filter_stride ? tr : 0));
         const size_t fbase = (size_t)(tr * args.filter_stride) + (size_t)c * B;
         if constexpr(FLT == Flt::SMEM) {
            mbar_wait(&fbar, 0, args.status);
#pragma unroll
            for(int k = 0; k < R; ++k) {
               if constexpr(BFP) f[k] = bfp_dequant(reinterpret_cast<const uint32_t*>(F)[lane + k * T], sb);
               else f[k] = reinterpret_cast<const float2*>(F)[lane + k * T];
            }
         } else if constexpr(FLT == Flt::BP_DIRECT) {
            // the same register-boundary order read coalesced from global
            // memory: no shared-memory copy, so more CTAs fit on an SM
#pragma unroll
            for(int k = 0; k < R; ++k) {
               if constexpr(BFP)
                  f[k] = bfp_dequant(__ldg(static_cast<const uint32_t*>(args.b) + fbase + lane + k * T), sb);
               else f[k] = __ldg(static_cast<const float2*>(args.b) + fbase + lane + k * T);
            }
         } else if constexpr(BFP) {
            const uint4* fp = reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(args.b) + fbase +
                                                             (size_t)lane * R);
#pragma unroll
            for(int k = 0; k < R; k += 4) {
               const uint4 w = __ldg(fp + k / 4);
               f[k] = bfp_dequant(w.x, sb);
               f[k + 1] = bfp_dequant(w.y, sb);
               f[k + 2] = bfp_dequant(w.z, sb);
               f[k + 3] = bfp_dequant(w.w, sb);
            }
         } else {
            const float4* fp = reinterpret_cast<const float4*>(static_cast<const float2*>(args.b) + fbase +
                                                               (size_t)lane * R);
#pragma unroll
            for(int k = 0; k < R; k += 2) {
               const float4 v = __ldg(fp + k / 2);
               f[k] = make_float2(v.x, v.y);
               f[k + 1] = make_float2(v.z, v.w);
            }
         }
#pragma unroll
         for(int k = 0; k < R; ++k) x[k] = (MID == Mid::MUL) ? cmul(x[k], f[k]) : cmulc(x[k], f[k]);
      }
      inv_all(X, x, lane, args.tw, std::make_integer_sequence<int, I::NP>{});

      // ---- 4. return exchange: row position p -> Y of its column's owner
      // o = p / CB, at [row c][p % CB]
      {
         constexpr int r0 = I::radix(0), G0 = R / r0;
         const uint32_t yb = smem_u32(Y), mb = smem_u32(&xbar[1]);
#pragma unroll
         for(int s = 0; s < G0; ++s)
#pragma unroll
            for(int k = 0; k < r0; ++k) {
               const int p = lane + T * (s + G0 * k);
               const int o = p / CB, idx = c * CB + (p % CB);
               if(o == c) Y[idx] = x[s * r0 + k];
               else st_async(map_remote(yb, o) + (uint32_t)(idx * sizeof(float2)), x[s * r0 + k],
                             map_remote(mb, o));
            }
      }
      mbar_wait<true>(&xbar[1], 0, args.status);
      __syncthreads();

      // ---- 5. this CTA's columns of every row, outer DIT pass, store
#pragma unroll
      for(int s = 0; s < G; ++s)
#pragma unroll
         for(int q = 0; q < C; ++q) x[s * C + q] = Y[q * CB + lane + T * s];
      outer<+1>(x, c, lane, args.tw);
      if constexpr(BFP) {
         // ---- 6. abs-max of the whole transform: this CTA's share, then one
         // 4-byte st.async to every peer; quantise with the cluster maximum
         float m = 0.0f;
#pragma unroll
         for(int i = 0; i < R; ++i) m = fmaxf(m, fmaxf(fabsf(x[i].x), fabsf(x[i].y)));
#pragma unroll
         for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
         if((lane & 31) == 0) wmax[lane >> 5] = m;
         __syncthreads();
         if(lane == 0) {
#pragma unroll
            for(int w = 1; w < T / 32; ++w) m = fmaxf(m, wmax[w]);
            const uint32_t cb = smem_u32(&cmax[c]), mb = smem_u32(&xbar[2]);
            cmax[c] = m;
#pragma unroll
            for(int q = 0; q < C; ++q)
               if(q != c) st_async(map_remote(cb, q), m, map_remote(mb, q));
         }
         mbar_wait<true>(&xbar[2], 0, args.status);
         __syncthreads();
         m = 0.0f;
#pragma unroll
         for(int q = 0; q < C; ++q) m = fmaxf(m, cmax[q]);
         const float mx = fmaxf(m, 1e-30f);
         const float inv = 32767.0f / mx;
         uint32_t* o = static_cast<uint32_t*>(args.out);
#pragma unroll
         for(int s = 0; s < G; ++s)
#pragma unroll
            for(int q = 0; q < C; ++q)
               st_stream(o + gbase + (size_t)q * B + c * CB + lane + T * s, bfp_quant(x[s * C + q], inv));
         if(c == 0 && lane == 0) args.out_scale[tr] = mx / 32767.0f;
      } else {
#pragma unroll
         for(int s = 0; s < G; ++s)
#pragma unroll
            for(int q = 0; q < C; ++q)
               st_stream(static_cast<float2*>(args.out) + gbase + (size_t)q * B + c * CB + lane + T * s,
                         x[s * C + q]);
      }
   }
};

// 768 resident threads per SM (three CTAs of 256, six of 128; 80 registers):
// the load, exchange and compute phases of one cluster barely overlap, so
// more resident clusters hide them better (+8-20% over 512 on the 1-D,
// four-step and 2-D shapes; 1024 spills and is slower)
#ifndef FUFFT_CLUSTER_RESIDENT
#define FUFFT_CLUSTER_RESIDENT 768
#endif
template<class Inner, int C, int OUT_L, int OUT_SHIFT, Mid MID, Flt FLT, bool BFP>
__global__ void __launch_bounds__(Inner::T, min_blocks<Inner::T, FUFFT_CLUSTER_RESIDENT>())
conv_cluster_kernel(const ConvArgs args)
{
   ClusterConv<Inner, C, OUT_L, OUT_SHIFT, MID, FLT, BFP>::run(args);
}

}  // namespace fufft
