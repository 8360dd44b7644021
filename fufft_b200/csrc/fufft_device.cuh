// fufft_device.cuh -- device building blocks of the fused FFT-convolution
// kernels for sm_100a: complex fp32 arithmetic, small DFT butterflies, the
// twiddle tables, the shared-memory swizzle, and the TMA bulk-copy /
// mbarrier primitives (inline PTX).
//
// Conventions (the ones the reference's C++ entry points expose, fufft.cuh):
//   * forward transforms use W_N = exp(-2 pi i / N) (sign -1), inverse +1,
//     unnormalised; the 1/N is folded into the filter spectrum by the caller;
//   * a radix-r DIF pass at stride M over group (b, j) reads taps
//     b*r*M + j + k*M, runs a natural-order DFT_r, then multiplies output k by
//     W_{rM}^{jk}; the DIT pass multiplies by the conjugate first, then runs
//     the inverse DFT_r (fufft.cuh:460-502, :723-750).
#pragma once
#include <cuda.h>   // CUtensorMap
#include <cuda_runtime.h>
#include <stdint.h>

namespace fufft {

// ---------------------------------------------------------------------------
// complex fp32 on float2 = (re, im)
// ---------------------------------------------------------------------------
// sm_100 packed fp32 pair arithmetic: one instruction per complex add/sub
// (per-lane IEEE add, bit-identical to the scalar form).  Measured on B200:
// +5..10% on the fused convolution, which is issue-bound, not FMA-pipe-bound.
__device__ __forceinline__ float2 cadd(float2 a, float2 b)
{
   float2 r;
   asm("{\n\t.reg .b64 ra, rb, rr;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
       "add.rn.f32x2 rr, ra, rb;\n\tmov.b64 {%0, %1}, rr;\n\t}"
       : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
   return r;
}
__device__ __forceinline__ float2 csub(float2 a, float2 b)
{
   float2 r;
   asm("{\n\t.reg .b64 ra, rb, rr;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
       "sub.rn.f32x2 rr, ra, rb;\n\tmov.b64 {%0, %1}, rr;\n\t}"
       : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
   return r;
}
// lane-wise product of two fp32 pairs (mul.rn.f32x2: one instruction, each
// lane rounded as the scalar product)
__device__ __forceinline__ float2 fmul2(float2 a, float2 b)
{
   float2 r;
   asm("{\n\t.reg .b64 ra, rb, rr;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
       "mul.rn.f32x2 rr, ra, rb;\n\tmov.b64 {%0, %1}, rr;\n\t}"
       : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
   return r;
}
// a * w, two fused products (same rounding shape as the reference's cmul,
// fufft.cuh:243-261)
__device__ __forceinline__ float2 cmul(float2 a, float2 w)
{
   return make_float2(fmaf(a.x, w.x, -a.y * w.y), fmaf(a.x, w.y, a.y * w.x));
}
// a * conj(w)  (fufft.cuh:644-648, MidConjMultiply)
__device__ __forceinline__ float2 cmulc(float2 a, float2 w)
{
   return make_float2(fmaf(a.x, w.x, a.y * w.y), fmaf(a.y, w.x, -a.x * w.y));
}

// Exact constants of the 16th roots of unity (rounded once from the exact values).
#define FUFFT_K_R2  0.70710678118654752440f   // cos(pi/4)
#define FUFFT_K_C16 0.92387953251128673848f   // cos(pi/8)
#define FUFFT_K_S16 0.38268343236508977173f   // sin(pi/8)

// a * W_4^1 in direction S (S = -1 forward: -i, S = +1 inverse: +i); free
template<int S> __device__ __forceinline__ float2 rot4(float2 a)
{
   return S < 0 ? make_float2(a.y, -a.x) : make_float2(-a.y, a.x);
}
// a * W_8^1 = a * (1 + S i)/sqrt2 : two adds, one packed multiply (the
// assembler may fuse that multiply into the butterfly add that consumes it:
// one rounding fewer, same or better accuracy)
template<int S> __device__ __forceinline__ float2 rot8(float2 a)
{
   return S < 0 ? fmul2(make_float2(a.x + a.y, a.y - a.x), make_float2(FUFFT_K_R2, FUFFT_K_R2))
                : fmul2(make_float2(a.x - a.y, a.x + a.y), make_float2(FUFFT_K_R2, FUFFT_K_R2));
}
// a * W_8^3 = a * (-1 + S i)/sqrt2
template<int S> __device__ __forceinline__ float2 rot8_3(float2 a)
{
   return S < 0 ? fmul2(make_float2(a.y - a.x, a.x + a.y), make_float2(FUFFT_K_R2, -FUFFT_K_R2))
                : fmul2(make_float2(a.x + a.y, a.x - a.y), make_float2(-FUFFT_K_R2, FUFFT_K_R2));
}
// a * W_16^e for the exponents the 4x4 radix-16 needs
template<int E, int S> __device__ __forceinline__ float2 rot16(float2 a)
{
   if constexpr(E == 0) return a;
   else if constexpr(E == 2) return rot8<S>(a);
   else if constexpr(E == 4) return rot4<S>(a);
   else if constexpr(E == 6) return rot8_3<S>(a);
   else if constexpr(E == 1) return cmul(a, make_float2(FUFFT_K_C16, (float)S * FUFFT_K_S16));
   else if constexpr(E == 3) return cmul(a, make_float2(FUFFT_K_S16, (float)S * FUFFT_K_C16));
   else /* E == 9 */ return cmul(a, make_float2(-FUFFT_K_C16, -(float)S * FUFFT_K_S16));
}

// ---------------------------------------------------------------------------
// natural-order DFTs on registers, in place: x[k] <- sum_n x[n] W_r^{S n k}
// ---------------------------------------------------------------------------
template<int S> __device__ __forceinline__ void dft2(float2* x)
{
   const float2 t = x[0];
   x[0] = cadd(t, x[1]);
   x[1] = csub(t, x[1]);
}

template<int S> __device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3)
{
   const float2 t0 = cadd(a0, a2), t1 = csub(a0, a2);
   const float2 t2 = cadd(a1, a3), t3 = rot4<S>(csub(a1, a3));
   a0 = cadd(t0, t2); a2 = csub(t0, t2);
   a1 = cadd(t1, t3); a3 = csub(t1, t3);
}
template<int S> __device__ __forceinline__ void dft4(float2* x) { dft4<S>(x[0], x[1], x[2], x[3]); }

// 8 = 2 x 4: DFT_4 over the even and the odd taps, W_8^k on the odd half,
// one radix-2 layer: X[k] = E[k] + W8^k O[k], X[k+4] = E[k] - W8^k O[k].
template<int S> __device__ __forceinline__ void dft8(float2* x)
{
   dft4<S>(x[0], x[2], x[4], x[6]);
   dft4<S>(x[1], x[3], x[5], x[7]);
   const float2 o1 = rot8<S>(x[3]), o2 = rot4<S>(x[5]), o3 = rot8_3<S>(x[7]);
   const float2 e0 = x[0], e1 = x[2], e2 = x[4], e3 = x[6], o0 = x[1];
   x[0] = cadd(e0, o0); x[4] = csub(e0, o0);
   x[1] = cadd(e1, o1); x[5] = csub(e1, o1);
   x[2] = cadd(e2, o2); x[6] = csub(e2, o2);
   x[3] = cadd(e3, o3); x[7] = csub(e3, o3);
}

// 16 = 4 x 4 with n = n1 + 4 n2, k = k2 + 4 k1:
//   Y[n1][k2] = DFT_4 over n2 of x[n1 + 4 n2];  Y[n1][k2] *= W16^{n1 k2};
//   X[k2 + 4 k1] = DFT_4 over n1 of Y[n1][k2].
template<int S> __device__ __forceinline__ void dft16(float2* x)
{
#pragma unroll
   for(int n1 = 0; n1 < 4; n1++) dft4<S>(x[n1], x[n1 + 4], x[n1 + 8], x[n1 + 12]);
   x[5] = rot16<1, S>(x[5]);  x[6] = rot16<2, S>(x[6]);  x[7] = rot16<3, S>(x[7]);
   x[9] = rot16<2, S>(x[9]);  x[10] = rot16<4, S>(x[10]); x[11] = rot16<6, S>(x[11]);
   x[13] = rot16<3, S>(x[13]); x[14] = rot16<6, S>(x[14]); x[15] = rot16<9, S>(x[15]);
   // Y[n1][k2] sits at x[n1 + 4 k2]; the radix-4 over n1 for fixed k2 uses
   // x[4k2 .. 4k2+3] and leaves X[k2 + 4 k1] at x[4 k2 + k1]
#pragma unroll
   for(int k2 = 0; k2 < 4; k2++) dft4<S>(x[4 * k2], x[4 * k2 + 1], x[4 * k2 + 2], x[4 * k2 + 3]);
   float2 y[16];
#pragma unroll
   for(int i = 0; i < 16; i++) y[i] = x[i];
#pragma unroll
   for(int k2 = 0; k2 < 4; k2++)
#pragma unroll
      for(int k1 = 0; k1 < 4; k1++) x[k2 + 4 * k1] = y[4 * k2 + k1];
}

template<int R, int S> __device__ __forceinline__ void dft(float2* x)
{
   static_assert(R == 2 || R == 4 || R == 8 || R == 16, "radix");
   if constexpr(R == 2) dft2<S>(x);
   else if constexpr(R == 4) dft4<S>(x);
   else if constexpr(R == 8) dft8<S>(x);
   else dft16<S>(x);
}

// ---------------------------------------------------------------------------
// twiddle table: for every power of two L <= 2^16 the L values
// W_L^j = exp(-2 pi i j / L), j < L, from fp64 sincospi rounded once to fp32
// (tw_offset(L) = L - 2).  A radix-r pass at stride M needs W_{rM}^{jk}, k < r:
// it loads the single value W_{rM}^j and forms the powers in registers
// (twiddle_powers), so the whole table a transform touches is a few KB and
// stays L1-resident.
// ---------------------------------------------------------------------------
constexpr int TW_LOG_MAX = 16;                       // largest L
__host__ __device__ constexpr int tw_offset(int L) { return L - 2; }
constexpr int TW_TOTAL = (2 << TW_LOG_MAX) - 2;

// w[k] = w1^k for k = 1 .. r-1 by a product tree of depth <= 4 (rounding
// error of the power grows with the depth, not with k)
template<int r>
__device__ __forceinline__ void twiddle_powers(float2 w1, float2* w)
{
   w[1] = w1;
   if constexpr(r > 2) w[2] = cmul(w1, w1);
   if constexpr(r > 3) w[3] = cmul(w[2], w1);
   if constexpr(r > 4) {
      w[4] = cmul(w[2], w[2]);
      w[5] = cmul(w[4], w1);
      w[6] = cmul(w[4], w[2]);
      w[7] = cmul(w[4], w[3]);
   }
   if constexpr(r > 8) {
      w[8] = cmul(w[4], w[4]);
#pragma unroll
      for(int k = 9; k < 16; ++k) w[k] = cmul(w[8], w[k - 8]);
   }
}

// ---------------------------------------------------------------------------
// shared-memory swizzle: XOR bits 1..3 of the float2 index with a function of
// bits 4..6/5..7.  A bijection (bits >= 4 are untouched), keeps adjacent
// pairs together (bit 0 untouched) so the register boundary moves 16 bytes at
// a time, and is 1-way on every exchange pattern of the radix-16 and radix-8
// engines (checked by tests/test_smem_audit.py).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int swz(int p) { return p ^ ((((p >> 4) ^ (p >> 5)) & 7) << 1); }

// ---------------------------------------------------------------------------
// TMA bulk copy + mbarrier (inline PTX, sm_90+ forms valid on sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
   asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init()
{
   asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
   asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes)
                : "memory");
}
// global -> shared bulk copy; dst, src 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
   asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// hint: bring `bytes` of global memory into L2 (no destination, no
// completion); src 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes)
{
   asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}
// 2-D tiled TMA load of box (x, y) of a tensor map into shared memory,
// completion on `bar`.  Every CTA loads its own tiles from this GPU's memory.  x is
// always 0 here (whole 128-byte rows), so the 16-byte rule on x holds.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar)
{
   asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%2, %3}], [%4];"
                :: "r"(smem_u32(dst)), "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm)
{
   asm volatile("prefetch.tensormap [%0];" :: "l"(tm) : "memory");
}
// orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) writes to the same memory
__device__ __forceinline__ void fence_proxy_async_smem()
{
   asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// CLUSTER = true: acquire at cluster scope, for phases completed by other
// CTAs' st.async stores (their complete_tx releases at cluster scope)
template<bool CLUSTER = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
   uint32_t ok;
   if constexpr(CLUSTER)
      asm volatile("{\n\t.reg .pred p;\n\t"
                   "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                   "selp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
   else
      asm volatile("{\n\t.reg .pred p;\n\t"
                   "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                   "selp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
   return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns()
{
   uint64_t t;
   asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
   return t;
}

// bits of the device status word the host reads through fufft_device_status()
constexpr unsigned STATUS_TMA_TIMEOUT = 1u;   // a bounded mbarrier wait gave up

// Bounded wait: gives up after `limit_ns` (2 s by default) and records it in
// the status word instead of spinning forever.
template<bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* status,
                                          uint64_t limit_ns = 2000000000ull)
{
   if(mbar_try_wait<CLUSTER>(bar, parity)) return true;
   const uint64_t t0 = globaltimer_ns();
   while(!mbar_try_wait<CLUSTER>(bar, parity)) {
      if(globaltimer_ns() - t0 > limit_ns) {
         atomicOr(status, STATUS_TMA_TIMEOUT);
         return false;
      }
   }
   return true;
}

// streaming global loads/stores: data read or written once, kept out of L1 so
// the twiddle tables stay resident
__device__ __forceinline__ float2 ld_stream(const float2* p) { return __ldcs(p); }
__device__ __forceinline__ uint32_t ld_stream(const uint32_t* p) { return __ldcs(reinterpret_cast<const unsigned int*>(p)); }
__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float2* p, float2 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(uint32_t* p, uint32_t v) { __stcs(reinterpret_cast<unsigned int*>(p), v); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

}  // namespace fufft
