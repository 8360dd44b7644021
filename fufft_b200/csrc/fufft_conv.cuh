// fufft_conv.cuh -- the fused one-block FFT convolution engine for sm_100a.
//
// One CTA runs CPB independent transforms of N points, T = N/R threads each,
// every thread holding R complex values in registers (R = 16: the V=16 form of
// fufft.cuh:763-800 / :1448-1497; R = 8: the radix-8 form of :930-1036).
// The radix chain is the reference's, so spectra come out in the same
// chain-reversed order and the filter layouts are interchangeable with it:
//     N = LEAD * R^NR, DIF passes [LEAD (if > 1), R, ..., R], strides
//     N/LEAD, N/(LEAD R), ..., 1; DIT in reverse.
//
// What is B200-specific:
//   * the first DIF pass reads its taps straight from HBM into registers
//     (thread `lane` needs a[lane + T*u], u < R: every warp load is one
//     coalesced 256-byte request), and the last DIT pass stores straight back
//     the same way -- no shared-memory staging of signal or result;
//   * the M == 1 passes of forward and inverse meet in registers: spectrum,
//     filter multiply and inverse butterfly never touch shared memory;
//   * the filter, in the register-boundary layout, is prefetched with one TMA
//     bulk copy per transform (cp.async.bulk + mbarrier) at kernel start, so
//     its HBM latency hides under the forward transform;
//   * exchanges between passes go through a swizzled shared buffer that is
//     1-way for every pattern (see swz()); 128-bit at the register boundary;
//   * twiddles come from fp64-accurate per-stride tables (L1-resident), not
//     from sincos recurrences;
//   * every wait is bounded (mbar_wait) and reports through the status word.
#pragma once
#include "fufft_device.cuh"

#include <utility>

namespace fufft {

// signal form entering / result form leaving the kernel.  SPEC: a spectrum in
// chain order (thread `lane` owns the R consecutive positions R*lane ..);
// SPEC_BP: the same spectrum in register-boundary order, position R*lane + k
// stored at lane + k*T (the bperm filter map) -- coalesced for every warp access
// Out::NAT: the spectrum in natural order (plain c2c transform, no inverse).
enum class In { C32, BFP, REAL2, SPEC, SPEC_BP, SPEC_R8, SPEC_R8BP };
enum class Out { C32, BFP, REAL2, SPEC, SPEC_BP, NAT, SPEC_R8, SPEC_R8BP };
enum class Mid { NONE, MUL, CONJ };        // pointwise operation between the transforms
// filter read: register-boundary layout staged by a TMA bulk copy (SMEM) or
// read straight from global memory (BP_DIRECT: coalesced, no shared memory),
// or chain order straight from global memory (GLOBAL), or chain order staged
// warp by warp through the free part of the exchange buffer (LIN_STAGED); a
// radix-16 engine reading a filter in the radix-8 chain order (R8_STAGED) or
// the radix-8 register-boundary order (R8BP_STAGED), staged the same way, or
// the register-boundary order read straight from global memory (R8BP_DIRECT)
enum class Flt { NONE, SMEM, GLOBAL, BP_DIRECT, LIN_STAGED, R8_STAGED, R8BP_STAGED, R8BP_DIRECT };

__host__ __device__ constexpr int ilog2c(long long n) { return n <= 1 ? 0 : 1 + ilog2c(n / 2); }

// radix chain of one dimension of length n under base radix R:
// [lead (if > 1), R, ..., R] with lead = 2^(log2 n mod log2 R)
__host__ __device__ constexpr int dim_passes(int n, int R)
{
   return n <= 1 ? 0 : ilog2c(n) / ilog2c(R) + ((ilog2c(n) % ilog2c(R)) ? 1 : 0);
}
__host__ __device__ constexpr int dim_radix(int n, int R, int q)
{
   return ((ilog2c(n) % ilog2c(R)) && q == 0) ? (1 << (ilog2c(n) % ilog2c(R))) : R;
}

// Pass plan of an H x W transform (H = 1: a 1-D transform of W points).
// Columns first: pass q of the H chain (radix r, per-column stride m) runs at
// flattened stride M = W*m with twiddles W_{r m}^{j2 k}, j2 = row position
// inside the group = (j >> log2 W) -- the column pass of fufft.cuh:1185-1207.
// Then the W chain along rows (stride M < W, twiddles W_{r M}^{j k}), whose
// last pass runs at M = 1 with radix R: the register boundary.  A 2-D DFT
// has no twiddles between its dimensions, so the two chains commute and the
// spectrum slot (r, c) holds frequency (rev_H(r), rev_W(c)).
template<int H_, int W_, int R_> struct Chain2 {
   static constexpr int H = H_, W = W_, R = R_, N = H_ * W_;
   static constexpr int T = N / R;
   static constexpr int NPC = dim_passes(H, R), NPR = dim_passes(W, R), NP = NPC + NPR;
   __host__ __device__ static constexpr int radix(int p)
   {
      return p < NPC ? dim_radix(H, R, p) : dim_radix(W, R, p - NPC);
   }
   __host__ __device__ static constexpr int dim_stride(int p)   // stride inside its own dimension
   {
      int m = p < NPC ? H : W;
      for(int q = (p < NPC ? 0 : NPC); q <= p; ++q) m /= radix(q);
      return m;
   }
   __host__ __device__ static constexpr int stride(int p) { return p < NPC ? W * dim_stride(p) : dim_stride(p); }
   __host__ __device__ static constexpr bool tw_on(int p) { return dim_stride(p) > 1; }
   __host__ __device__ static constexpr int tw_L(int p) { return radix(p) * dim_stride(p); }
   __host__ __device__ static constexpr int tw_shift(int p) { return p < NPC ? ilog2c(W) : 0; }
   static_assert((1 << ilog2c(H)) == H && (1 << ilog2c(W)) == W && (1 << ilog2c(R)) == R, "powers of two only");
   static_assert(W >= R, "the row chain must end in a full radix-R pass (the register boundary)");
};
template<int N, int R> using Chain = Chain2<1, N, R>;

struct ConvArgs {
   const void* a;          // signal: float2 (C32), packed int16 pairs (BFP), float xr (REAL2), spectrum (SPEC)
   const void* a2;         // REAL2: yr
   const float* a_scale;   // BFP: one scale per transform
   const void* b;          // filter spectrum (float2, or packed int16 pairs for BFP)
   const float* b_scale;   // BFP filter scales
   void* out;              // result (float2 / packed int16 / ur / spectrum)
   void* out2;             // REAL2: vr
   float* out_scale;       // BFP: one scale per transform
   long long filter_stride;  // elements between consecutive transforms' filters; 0 = one shared filter
   long long spec_stride;    // SPEC input: elements between consecutive transforms' spectra
   long long scale_div;      // BFP filter scale of transform t: b_scale[t / scale_div] (0, 1: per transform)
   long long grid_filters;   // SPEC input, > 0: transform t = s * grid_filters + f applies filter f to spectrum s
   int conj_io;              // Out::NAT: conjugate on load and store (the inverse transform)
   float spec_scale;         // spectrum outputs: multiply by this when nonzero (filter preparation: 1/n)
   long long prefetch_ahead; // > 0: each CTA asks L2 for the data of the CTA this many blocks later
   long long batch;
   const float2* tw;         // the device's twiddle tables (tw_offset layout)
   unsigned int* status;     // device status word (bounded-wait reports)
};

// ---------------------------------------------------------------------------
// per-pass index maps.  In pass p (radix r, stride M, G = R/r groups per
// thread) thread `lane` owns groups g = lane + s*T; group g = (b, j) =
// (g / M, g % M) holds taps b*r*M + j + k*M.  Register x[s*r + k] is tap k of
// group s.
// ---------------------------------------------------------------------------
template<class C, int p, class F>
__device__ __forceinline__ void visit(int lane, F&& f)
{
   constexpr int r = C::radix(p), M = C::stride(p), G = C::R / r, T = C::T;
#pragma unroll
   for(int s = 0; s < G; ++s) {
      const int g = lane + s * T;
      const int j = g & (M - 1);
      const int b = g >> ilog2c(M);
      const int base = b * r * M + j;
#pragma unroll
      for(int k = 0; k < r; ++k) f(s * r + k, base + k * M);
   }
}

// DIF (S = -1): butterfly, then W^{jk}.  DIT (S = +1): conj(W^{jk}), then butterfly.
// One table load (W_{rM}^j) per group; the powers are formed in registers.
template<class C, int p, int S>
__device__ __forceinline__ void butterflies(float2 (&x)[C::R], int lane, const float2* __restrict__ twt)
{
   constexpr int r = C::radix(p), M = C::stride(p), G = C::R / r, T = C::T;
#pragma unroll
   for(int s = 0; s < G; ++s) {
      float2* u = x + s * r;
      if constexpr(C::tw_on(p)) {
         const int j = ((lane + s * T) & (M - 1)) >> C::tw_shift(p);
         float2 w[r];
         twiddle_powers<r>(__ldca(twt + tw_offset(C::tw_L(p)) + j), w);
         if constexpr(S > 0) {
#pragma unroll
            for(int k = 1; k < r; ++k) u[k] = cmulc(u[k], w[k]);
         }
         dft<r, S>(u);
         if constexpr(S < 0) {
#pragma unroll
            for(int k = 1; k < r; ++k) u[k] = cmul(u[k], w[k]);
         }
      } else {
         dft<r, S>(u);
      }
   }
}

// Swizzle policies of the exchange buffer (float2 index -> float2 slot).
//   SwzEngine: swz() above, 1-way for every size of both engines.
//   Swz128:    exactly the TMA SWIZZLE_128B pattern (16-byte chunk bits 4..6
//              of the byte address XOR bits 7..9), so a buffer filled by a
//              swizzled TMA tensor load is already in exchange order; 1-way
//              for every pattern with n >= 256 (radix 16) / n >= 8 (radix 8).
// map(p) = p ^ term(p >> 4): the XOR term reads the bits 4 .. log2(PERIOD)-1
// of p and writes bits 1..3, so adding a multiple of PERIOD commutes with map.
struct SwzEngine {
   static constexpr int PERIOD = 256;
   __host__ __device__ static constexpr int term(int v) { return ((v ^ (v >> 1)) & 7) << 1; }
   __device__ __forceinline__ static int map(int p) { return swz(p); }
};
struct Swz128 {
   static constexpr int PERIOD = 128;
   __host__ __device__ static constexpr int term(int v) { return (v & 7) << 1; }
   __device__ __forceinline__ static int map(int p) { return p ^ (((p >> 4) & 7) << 1); }
};

#ifndef FUFFT_XADDR
#define FUFFT_XADDR 1
#endif
// swizzled slot of every position a thread touches in pass p: f(i, slot) for
// register i.  The swizzle is taken out of the per-element work where the
// pass structure allows: stride M a multiple of the period -> one map per
// group and constant offsets; stride 16 with the group base's bits 4..7 zero
// (radix-16 pass, whole 256-point blocks) -> one XOR with a per-k constant.
template<class C, int p, class SW, class F>
__device__ __forceinline__ void visit_slots(int off, int lane, F&& f)
{
   constexpr int r = C::radix(p), M = C::stride(p), G = C::R / r, T = C::T;
#pragma unroll
   for(int s = 0; s < G; ++s) {
      const int g = lane + s * T;
      const int j = g & (M - 1);
      const int b = g >> ilog2c(M);
      const int P = off + b * r * M + j;
      if constexpr(FUFFT_XADDR && M % SW::PERIOD == 0) {
         const int q = SW::map(P);
#pragma unroll
         for(int k = 0; k < r; ++k) f(s * r + k, q + k * M);
      } else if constexpr(FUFFT_XADDR && M == 16 && (r * M) % SW::PERIOD == 0 && C::N % SW::PERIOD == 0) {
#pragma unroll
         for(int k = 0; k < r; ++k) f(s * r + k, (P ^ SW::term(k)) + k * M);
      } else {
#pragma unroll
         for(int k = 0; k < r; ++k) f(s * r + k, SW::map(P + k * M));
      }
   }
}

// exchange through the swizzled shared buffer; `off` = slot * N
template<class C, int p, class SW = SwzEngine>
__device__ __forceinline__ void xstore(float2* X, int off, const float2 (&x)[C::R], int lane)
{
   if constexpr(C::stride(p) == 1) {
      // base's low log2(R) bits are zero: map(base + k) = (base ^ term(base >> 4)) ^ k
      const int base = off + lane * C::R;
      const int x0 = FUFFT_XADDR ? base ^ SW::term(base >> 4) : 0;
#pragma unroll
      for(int k = 0; k < C::R; k += 2) {
         const int q = FUFFT_XADDR ? (x0 ^ k) : SW::map(base + k);
         *reinterpret_cast<float4*>(X + q) = make_float4(x[k].x, x[k].y, x[k + 1].x, x[k + 1].y);
      }
   } else {
      visit_slots<C, p, SW>(off, lane, [&](int i, int q) { X[q] = x[i]; });
   }
}

template<class C, int p, class SW = SwzEngine>
__device__ __forceinline__ void xload(const float2* X, int off, float2 (&x)[C::R], int lane)
{
   if constexpr(C::stride(p) == 1) {
      const int base = off + lane * C::R;
      const int x0 = FUFFT_XADDR ? base ^ SW::term(base >> 4) : 0;
#pragma unroll
      for(int k = 0; k < C::R; k += 2) {
         const int q = FUFFT_XADDR ? (x0 ^ k) : SW::map(base + k);
         const float4 v = *reinterpret_cast<const float4*>(X + q);
         x[k] = make_float2(v.x, v.y);
         x[k + 1] = make_float2(v.z, v.w);
      }
   } else {
      visit_slots<C, p, SW>(off, lane, [&](int i, int q) { x[i] = X[q]; });
   }
}

// compiler-level ordering point between passes.  (The twiddle tables are
// read with coherent ld.global.ca rather than the read-only path: ptxas may
// move read-only loads across bar.sync, and hoisting every later pass's
// twiddles to the top of the kernel costs ~60 registers and spills.)
__device__ __forceinline__ void sched_fence() { asm volatile("" ::: "memory"); }


// The exchange between passes p and p+1 is warp-local when every position's
// owner in pass p and its owner in pass p+1 (lane of its butterfly group,
// visit() above) sit in the same warp.  Every thread writes exactly the
// positions it owns in the pass it read, so between two block-wide barriers
// each position is touched only by the threads of one warp along a run of
// warp-local exchanges, and __syncwarp orders them.  (Radix-16 chains: the
// last exchange of each direction moves data within 16-lane groups.)
template<class C, int p>
constexpr bool warp_local_exchange()
{
   if(C::T <= 32) return true;
   const int r0 = C::radix(p), M0 = C::stride(p), r1 = C::radix(p + 1), M1 = C::stride(p + 1);
   for(int P = 0; P < C::N; ++P) {
      const int g0 = (P / (r0 * M0)) * M0 + P % M0;
      const int g1 = (P / (r1 * M1)) * M1 + P % M1;
      if((g0 % C::T) / 32 != (g1 % C::T) / 32) return false;
   }
   return true;
}

#ifndef FUFFT_WARP_LOCAL_SYNC
#define FUFFT_WARP_LOCAL_SYNC 1
#endif
// barrier of the exchange between passes p and p+1
template<class C, int p, int CPB>
__device__ __forceinline__ void exchange_sync(int slot);

// barrier over the T threads of one transform
template<int T, int CPB>
__device__ __forceinline__ void slot_sync(int slot)
{
   if constexpr(T <= 32) __syncwarp();
   else if constexpr(CPB == 1) __syncthreads();
   else asm volatile("bar.sync %0, %1;" :: "r"(slot + 1), "n"(T) : "memory");
}

template<class C, int p, int CPB>
__device__ __forceinline__ void exchange_sync(int slot)
{
   if constexpr(FUFFT_WARP_LOCAL_SYNC && warp_local_exchange<C, p>()) __syncwarp();
   else slot_sync<C::T, CPB>(slot);
}

// int16 pair <-> fp32 complex, the reference's BFP element (fufft.cuh:1572-1612)
#ifndef FUFFT_DEQUANT_PTX
#define FUFFT_DEQUANT_PTX 1
#endif
#ifndef FUFFT_BFP_MAGIC_Q
#define FUFFT_BFP_MAGIC_Q 1
#endif
// (An integer-free dequantisation -- each half, sign-flipped, placed in the
// mantissa of 2^23 and the offset subtracted -- measured 1-3% slower than the
// two conversions: five issue slots against two.)
__device__ __forceinline__ float2 bfp_dequant(uint32_t w, float scale)
{
#if FUFFT_DEQUANT_PTX
   // the two int16 halves converted straight from the packed word
   float x, y;
   asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
       "cvt.rn.f32.s16 %0, lo;\n\tcvt.rn.f32.s16 %1, hi;\n\t}"
       : "=f"(x), "=f"(y) : "r"(w));
   return make_float2(x * scale, y * scale);
#else
   return make_float2((float)(short)(w & 0xffffu) * scale, (float)(short)(w >> 16) * scale);
#endif
}
// rint(clamp(v * inv, +-32767)) per component.  |v * inv| <= 32767 * (1 +
// 2^-23) because inv comes from the abs-max of the same values, so the
// explicit clamp of the reference's C++ form (fufft.cuh:1587-1589) changes
// nothing reachable.  The product is rounded to fp32 first, as in the
// reference's PTX form (fufft.cuh:1576-1584), then to the nearest integer,
// ties to even.  Default form: adding 1.5 * 2^23 to the product leaves that
// integer in the low mantissa bits (exact for |v * inv| < 2^22), whose low 16
// bits are its two's-complement int16 -- the same result as the s16
// conversion for every finite input, in two FMA-pipe operations instead of
// the conversion unit (+1-2% on the BFP kernels).  Non-finite products give
// 0 through the conversion and an unspecified value here.
__device__ __forceinline__ uint32_t bfp_quant(float2 v, float inv)
{
#if FUFFT_BFP_MAGIC_Q
   // scalar intrinsics on purpose: a packed f32x2 product followed by a packed
   // add may be fused into one f32x2 FMA by the assembler, which skips the
   // product's rounding and breaks bit-exactness with the reference quantiser
   const float fx = __fadd_rn(__fmul_rn(v.x, inv), 12582912.0f);
   const float fy = __fadd_rn(__fmul_rn(v.y, inv), 12582912.0f);
   return __byte_perm(__float_as_uint(fx), __float_as_uint(fy), 0x5410);
#else
   uint32_t r;
   asm("{\n\t.reg .s16 sx, sy;\n\t.reg .f32 fx, fy;\n\t"
       "mul.rn.f32 fx, %1, %3;\n\tmul.rn.f32 fy, %2, %3;\n\t"
       "cvt.rni.s16.f32 sx, fx;\n\tcvt.rni.s16.f32 sy, fy;\n\t"
       "mov.b32 %0, {sx, sy};\n\t}"
       : "=r"(r) : "f"(v.x), "f"(v.y), "f"(inv));
   return r;
#endif
}

// natural (frequency) index of chain position p of a 1-D chain: the digits
// of p, one per pass (pass 0 most significant), written back in reverse order
template<class C>
__device__ __forceinline__ int chain_natural(int p)
{
   int out = 0, pos = ilog2c(C::N), op = 0;
#pragma unroll
   for(int k = 0; k < C::NP; ++k) {
      const int w = ilog2c(C::radix(k));
      pos -= w;
      out |= ((p >> pos) & ((1 << w) - 1)) << op;
      op += w;
   }
   return out;
}
// the same for p = R*lane + k when the last pass has radix R: k is the last
// digit, so chain_natural(R*lane + k) = k*T + lane_natural(lane), with the
// lane's digits (passes 0 .. NP-2) reversed into the low bits
template<class C>
__device__ __forceinline__ int lane_natural(int lane)
{
   static_assert(C::radix(C::NP - 1) == C::R, "last pass of radix R");
   int out = 0, pos = ilog2c(C::T), op = 0;
#pragma unroll
   for(int k = 0; k < C::NP - 1; ++k) {
      const int w = ilog2c(C::radix(k));
      pos -= w;
      out |= ((lane >> pos) & ((1 << w) - 1)) << op;
      op += w;
   }
   return out;
}

// Programmatic dependent launch of the fused kernels (griddepcontrol): the
// next launch's CTAs are scheduled while this one drains, so back-to-back
// launches lose no launch latency.  Measured on B200, n = 1024 R16_BPERM, four
// or more input sets in turn (> 3x L2): batch 1024 10.6 -> 9.5 us, 4096 24.5 ->
// 22.4 us, 16384 71.9 -> 70.2 us per launch; no change for a single launch.
// ---------------------------------------------------------------------------
// A filter in another chain's layout.  Every layout of a power-of-two n is a
// permutation of the index bits: chain position -> natural frequency reverses
// the chain's digit groups (chain_natural), the register-boundary order moves
// the last digit to the top.  So the map from this engine's chain position p
// to the index q of the same frequency in the radix-8 layouts (the reference's
// mixedrev order, fufft.cuh:1757-1772 with the filter permuted as in
// verify_kernel.cpp:145-156, and its register-boundary order) is a bit
// permutation: q = OR of sigma(b) over the set bits b of p, all known at
// compile time.
// chain position p -> natural frequency for the 1-D chain of n points under
// base radix R (the dim_radix chain), and its inverse
__host__ __device__ constexpr int dim_nat(int p, int n, int R)
{
   int out = 0, pos = ilog2c(n), op = 0;
   for(int k = 0; k < dim_passes(n, R); ++k) {
      const int w = ilog2c(dim_radix(n, R, k));
      pos -= w;
      out |= ((p >> pos) & ((1 << w) - 1)) << op;
      op += w;
   }
   return out;
}
__host__ __device__ constexpr int dim_pos(int nu, int n, int R)
{
   int p = 0, pos = ilog2c(n), op = 0;
   for(int k = 0; k < dim_passes(n, R); ++k) {
      const int w = ilog2c(dim_radix(n, R, k));
      pos -= w;
      p |= ((nu >> op) & ((1 << w) - 1)) << pos;
      op += w;
   }
   return p;
}

// Staging plan of one warp's 512 filter values for the radix-16 engine (each
// lane holds chain positions 16*l + k of the warp's 512): the low 9 bits of p
// are the warp's own.  Bit B0 of p lands on bit 0 of q, so positions p and
// p | (1 << B0) are one 16-byte load.  Of the other 8 low bits, 5 index the
// lanes and 3 the loads of a lane, picked at compile time so that the
// exchange-slot stores of a load are free of bank conflicts and each group of
// lanes reads whole 32-byte sectors (bit 1 of q among the lane bits).
template<class C, bool BP> struct R8Perm {
   static constexpr int N = C::N, LB = ilog2c(N);
   // this chain's position -> radix-8 layout index.  2-D (H x W): each
   // dimension's digits are reversed on its own (slot (r, c) holds frequency
   // (rev_H(r), rev_W(c)) in both layouts)
   __host__ __device__ static constexpr int map(int p)
   {
      const int r = p / C::W, c = p % C::W;
      const int q = dim_pos(dim_nat(r, C::H, 16), C::H, 8) * C::W + dim_pos(dim_nat(c, C::W, 16), C::W, 8);
      return BP ? (q >> 3) + (q & 7) * (N / 8) : q;
   }
   __host__ __device__ static constexpr int sig(int b) { return ilog2c(map(1 << b)); }
   // do the five low lane bits (position bits 4..8) land on index bits 0 and 1?
   __host__ __device__ static constexpr bool lanes_cover_q01()
   {
      bool z = false, o = false;
      for(int b = 4; b < 9 && b < LB; ++b) {
         z = z || sig(b) == 0;
         o = o || sig(b) == 1;
      }
      return z && o;
   }
   __host__ __device__ static constexpr int slot(int p)   // float2 slot of local position p (swizzled float4 rows)
   {
      return 2 * ((p >> 1) ^ ((p >> 4) & 7)) + (p & 1);
   }
   struct Plan {
      int b0;
      int lane[5];
      int hi[3];
   };
   __host__ __device__ static constexpr int b0()
   {
      int r = -1;
      for(int b = 0; b < LB; ++b)
         if(sig(b) == 0) r = b;
      return r;
   }
   // bank-conflict degree (sum over the 16 stores of a lane of the worst bank pair's count)
   __host__ __device__ static constexpr int cost(const int (&lane)[5], const int (&hi)[3], int z)
   {
      int tot = 0;
      for(int i = 0; i < 8; ++i)
         for(int half = 0; half < 2; ++half) {
            int cnt[16] = {};
            int worst = 2;
            for(int l = 0; l < 32; ++l) {
               int p = half << z;
               for(int t = 0; t < 5; ++t) p |= ((l >> t) & 1) << lane[t];
               for(int t = 0; t < 3; ++t) p |= ((i >> t) & 1) << hi[t];
               const int c = ++cnt[slot(p) & 15];
               worst = c > worst ? c : worst;
            }
            tot += worst;
         }
      return tot;
   }
   __host__ __device__ static constexpr Plan plan()
   {
      Plan best{b0(), {0, 0, 0, 0, 0}, {0, 0, 0}};
      int free_[8] = {}, nf = 0;
      for(int b = 0; b < 9; ++b)
         if(b != best.b0) free_[nf++] = b;
      int best_cost = 1 << 30;
      for(int m = 0; m < 256; ++m) {   // 5 of the 8 free bits for the lanes
         int pc = 0;
         for(int t = 0; t < 8; ++t) pc += (m >> t) & 1;
         if(pc != 5) continue;
         int lane[5] = {}, hi[3] = {}, nl = 0, nh = 0;
         bool q1 = false;
         for(int t = 0; t < 8; ++t) {
            if((m >> t) & 1) {
               lane[nl++] = free_[t];
               q1 = q1 || sig(free_[t]) == 1;
            } else {
               hi[nh++] = free_[t];
            }
         }
         const int c = cost(lane, hi, best.b0) * 2 + (q1 ? 0 : 1);
         if(c < best_cost) {
            best_cost = c;
            for(int t = 0; t < 5; ++t) best.lane[t] = lane[t];
            for(int t = 0; t < 3; ++t) best.hi[t] = hi[t];
         }
      }
      return best;
   }
   // everything the kernel needs, as one constant (evaluated at compile time)
   struct Tables {
      int b0;
      int lane[5];       // local position bit of lane bit t
      int sig_lane[5];   // its layout-index bit
      int sig_w[8];      // layout-index bit of warp bit t (position bit 9 + t)
      int qh[8];         // layout-index bits of load i
      int s0[8], s1[8];  // exchange slots of load i's two values (XOR with the lane's own)
      int sig[16];       // layout-index bit of every position bit (direct reads)
      int mapk[16];      // layout index of positions 0..15 (register k of lane 0)
   };
   __host__ __device__ static constexpr Tables tables()
   {
      const Plan P = plan();
      Tables tb{};
      for(int b = 0; b < 16; ++b) tb.sig[b] = b < LB ? sig(b) : 0;
      for(int k = 0; k < 16; ++k) tb.mapk[k] = map(k);
      tb.b0 = P.b0;
      for(int t = 0; t < 5; ++t) {
         tb.lane[t] = P.lane[t];
         tb.sig_lane[t] = sig(P.lane[t]);
      }
      for(int t = 0; t < 8; ++t) tb.sig_w[t] = 9 + t < LB ? sig(9 + t) : 0;
      for(int i = 0; i < 8; ++i) {
         int hp = 0;
         for(int t = 0; t < 3; ++t) hp |= ((i >> t) & 1) << P.hi[t];
         int q = 0;
         for(int b = 0; b < LB; ++b)
            if((hp >> b) & 1) q |= 1 << sig(b);
         tb.qh[i] = q;
         tb.s0[i] = slot(hp);
         tb.s1[i] = slot(hp | (1 << P.b0));
      }
      return tb;
   }
   static_assert(LB >= 9 && b0() >= 0 && b0() < 9, "bit 0 of the layout index comes from a warp-local bit");
};

#ifndef FUFFT_SPEC_STAGED
#define FUFFT_SPEC_STAGED 1
#endif
#ifndef FUFFT_PDL
#define FUFFT_PDL 1
#endif
template<class C_, int CPB, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
struct ConvKernel {
   using C = C_;
   static constexpr int N = C::N, R = C::R;
   static constexpr int T = C::T;
   static constexpr int THREADS = CPB * T;
   // int16-BFP in and out: the transforms run on the raw mantissas and the
   // product of the input and filter scales enters only the output scale
   // (a convolution is linear), saving the multiplies of the dequantisation
   static constexpr bool FOLD = IN == In::BFP && OUT == Out::BFP;
   static constexpr bool SPEC_IN = IN == In::SPEC || IN == In::SPEC_BP || IN == In::SPEC_R8 || IN == In::SPEC_R8BP;
   static constexpr bool SPEC_OUT =
      OUT == Out::SPEC || OUT == Out::SPEC_BP || OUT == Out::SPEC_R8 || OUT == Out::SPEC_R8BP;
   // radix-16 chain-order spectra move through the warp's exchange slots
   // (coalesced 16-byte accesses) when a transform has whole warps of one
   // dimension: forward +50-68%, apply +26-35% at n = 512..4096 (B200,
   // interleaved A/B); radix-8 rows (64 bytes per thread) measured 4-13%
   // slower staged and keep the direct 16-byte loads
   static constexpr bool SPEC_ROWS = FUFFT_SPEC_STAGED && R == 16 && T >= 32 && C::H == 1;
   static constexpr bool HAS_FILTER = (MID != Mid::NONE) && !SPEC_OUT;
   static constexpr int FELEM = FBFP ? 4 : 8;
   static constexpr size_t X_BYTES = (size_t)CPB * N * sizeof(float2);
   static constexpr size_t F_BYTES = (HAS_FILTER && FLT == Flt::SMEM) ? (size_t)CPB * N * FELEM : 0;
   static constexpr size_t SMEM = X_BYTES + F_BYTES;

   // BFP filter scale of transform t
   __device__ __forceinline__ static float filter_scale(const ConvArgs& args, long long t, bool active)
   {
      return active ? __ldg(args.b_scale + (args.filter_stride ? (args.scale_div > 1 ? t / args.scale_div : t) : 0))
                    : 0.0f;
   }

   // element offset of transform t's filter.  Grid apply (one launch over every
   // spectrum x every filter): filter t % F; otherwise t * filter_stride.
   __device__ __forceinline__ static long long filter_off(const ConvArgs& args, long long t)
   {
      if constexpr(SPEC_IN)
         if(args.grid_filters > 0) return (t % args.grid_filters) * N;
      return t * args.filter_stride;
   }

   // ---- a warp's 32*R consecutive chain positions <-> each lane's R
   // consecutive ones, through the warp's own exchange slots Xw.  The last
   // pass (stride 1, radix R) gives warp w exactly the positions [32 R w,
   // +32 R), and the exchange into it is either warp-local or behind a
   // barrier of the transform's threads, so between warp w's last forward
   // read and its first inverse write no other warp touches those slots.
   // 16-byte slot q sits at q ^ ((q >> 3) & 7): conflict-free for the
   // coalesced side and for the row side.
   __device__ __forceinline__ static void rows_in(const float2* src, float2* Xw, int l, bool active, float2 (&v)[R])
   {
      constexpr int RV = R / 2;
      float4* S = reinterpret_cast<float4*>(Xw);
      const float4* g = reinterpret_cast<const float4*>(src);
      __syncwarp();
#pragma unroll
      for(int i = 0; i < RV; ++i) {
         const float4 w = active ? __ldg(g + l + 32 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
         S[32 * i + (l ^ (((l >> 3) + 4 * i) & 7))] = w;
      }
      __syncwarp();
#pragma unroll
      for(int i = 0; i < RV; ++i) {
         const int q = RV * l + i;
         const float4 w = S[q ^ ((q >> 3) & 7)];
         v[2 * i] = make_float2(w.x, w.y);
         v[2 * i + 1] = make_float2(w.z, w.w);
      }
      __syncwarp();
   }
   __device__ __forceinline__ static void rows_out(const float2 (&v)[R], float2* Xw, float2* dst, int l)
   {
      constexpr int RV = R / 2;
      float4* S = reinterpret_cast<float4*>(Xw);
      float4* g = reinterpret_cast<float4*>(dst);
      __syncwarp();
#pragma unroll
      for(int i = 0; i < RV; ++i) {
         const int q = RV * l + i;
         S[q ^ ((q >> 3) & 7)] = make_float4(v[2 * i].x, v[2 * i].y, v[2 * i + 1].x, v[2 * i + 1].y);
      }
      __syncwarp();
#pragma unroll
      for(int i = 0; i < RV; ++i) st_stream(g + l + 32 * i, S[32 * i + (l ^ (((l >> 3) + 4 * i) & 7))]);
      __syncwarp();
   }
   // ---- the same for a radix-8 layout (R8Perm): this warp's 512 positions
   // sit at q = map(512 w + local p) of the transform starting at `base`
   template<bool BP>
   __device__ __forceinline__ static void perm_in(const float2* base, float2* Xw, int lane, bool active,
                                                  float2 (&v)[R])
   {
      using PM = R8Perm<C, BP>;
      constexpr typename PM::Tables TB = PM::tables();
      const int w = lane >> 5, l = lane & 31;
      int pl = 0, ql = 0;
#pragma unroll
      for(int t = 0; t < 5; ++t) {
         pl |= ((l >> t) & 1) << TB.lane[t];
         ql |= ((l >> t) & 1) << TB.sig_lane[t];
      }
#pragma unroll
      for(int t = 0; t < PM::LB - 9; ++t) ql |= ((w >> t) & 1) << TB.sig_w[t];
      // ql and qh[i] have disjoint bits: one base pointer, constant offsets;
      // slot() is XOR-linear in p
      const float2* g = base + ql;
      const int sl = PM::slot(pl);
      __syncwarp();
#pragma unroll
      for(int i = 0; i < 8; ++i) {
         const float4 x = active ? __ldg(reinterpret_cast<const float4*>(g + TB.qh[i]))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
         Xw[sl ^ TB.s0[i]] = make_float2(x.x, x.y);
         Xw[sl ^ TB.s1[i]] = make_float2(x.z, x.w);
      }
      __syncwarp();
      const float4* S = reinterpret_cast<const float4*>(Xw);
#pragma unroll
      for(int i = 0; i < 8; ++i) {
         const int q = 8 * l + i;
         const float4 x = S[q ^ ((q >> 3) & 7)];
         v[2 * i] = make_float2(x.x, x.y);
         v[2 * i + 1] = make_float2(x.z, x.w);
      }
      __syncwarp();
   }
   template<bool BP>
   __device__ __forceinline__ static void perm_out(const float2 (&v)[R], float2* Xw, float2* base, int lane)
   {
      using PM = R8Perm<C, BP>;
      constexpr typename PM::Tables TB = PM::tables();
      const int w = lane >> 5, l = lane & 31;
      int pl = 0, ql = 0;
#pragma unroll
      for(int t = 0; t < 5; ++t) {
         pl |= ((l >> t) & 1) << TB.lane[t];
         ql |= ((l >> t) & 1) << TB.sig_lane[t];
      }
#pragma unroll
      for(int t = 0; t < PM::LB - 9; ++t) ql |= ((w >> t) & 1) << TB.sig_w[t];
      float4* S = reinterpret_cast<float4*>(Xw);
      __syncwarp();
#pragma unroll
      for(int i = 0; i < 8; ++i) {
         const int q = 8 * l + i;
         S[q ^ ((q >> 3) & 7)] = make_float4(v[2 * i].x, v[2 * i].y, v[2 * i + 1].x, v[2 * i + 1].y);
      }
      __syncwarp();
      float2* g = base + ql;
      const int sl = PM::slot(pl);
#pragma unroll
      for(int i = 0; i < 8; ++i) {
         const float2 a = Xw[sl ^ TB.s0[i]], b = Xw[sl ^ TB.s1[i]];
         st_stream(reinterpret_cast<float4*>(g + TB.qh[i]), make_float4(a.x, a.y, b.x, b.y));
      }
      __syncwarp();
   }

   template<int p>
   __device__ __forceinline__ static void fwd_step(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                   const float2* tw)
   {
      sched_fence();
      if constexpr(p > 0) {
         xstore<C, p - 1>(X, off, x, lane);
         exchange_sync<C, p - 1, CPB>(slot);
         xload<C, p>(X, off, x, lane);
      }
      butterflies<C, p, -1>(x, lane, tw);
   }
   template<int p>
   __device__ __forceinline__ static void inv_step(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                   const float2* tw)
   {
      // p runs NP-1 .. 0
      sched_fence();
      if constexpr(p < C::NP - 1) {
         xstore<C, p + 1>(X, off, x, lane);
         exchange_sync<C, p, CPB>(slot);
         xload<C, p>(X, off, x, lane);
      }
      butterflies<C, p, +1>(x, lane, tw);
   }
   template<int... ps>
   __device__ __forceinline__ static void fwd_all(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                  const float2* tw, std::integer_sequence<int, ps...>)
   {
      (fwd_step<ps>(X, off, x, lane, slot, tw), ...);
   }
   template<int... ps>
   __device__ __forceinline__ static void inv_all(float2* X, int off, float2 (&x)[R], int lane, int slot,
                                                  const float2* tw, std::integer_sequence<int, ps...>)
   {
      (inv_step<C::NP - 1 - ps>(X, off, x, lane, slot, tw), ...);
   }

   __device__ __forceinline__ static void run(const ConvArgs& args)
   {
#if FUFFT_PDL
      // launched with programmatic stream serialisation: wait until the
      // stream's previous kernel has finished and its writes are visible,
      // then let the stream's next kernel be scheduled into the slots this
      // grid frees (it waits here in turn)
      asm volatile("griddepcontrol.wait;" ::: "memory");
      asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
      extern __shared__ __align__(1024) unsigned char smem_raw[];
      __shared__ uint64_t fbar;
      __shared__ float warp_max[THREADS / 32 > 0 ? THREADS / 32 : 1];
      float2* X = reinterpret_cast<float2*>(smem_raw);
      unsigned char* F = smem_raw + X_BYTES;

      const int slot = threadIdx.x / T, lane = threadIdx.x % T;
      const long long tr0 = (long long)blockIdx.x * CPB;
      const long long tr = tr0 + slot;
      const bool active = tr < args.batch;
      const int off = slot * N;
      const size_t gbase = (size_t)tr * N;
      // grid apply: spectrum s = t / F.  Real-pair output rows: ur of pair s
      // and filter f at row 2*s*F + f = t + s*F, vr one block of F rows later
      long long spec_row = tr * args.spec_stride;
      size_t obase = gbase;
      if constexpr(SPEC_IN) {
         if(args.grid_filters > 0) {
            const long long sidx = tr / args.grid_filters;
            spec_row = sidx * N;
            if constexpr(OUT == Out::REAL2) obase = (size_t)(tr + sidx * args.grid_filters) * N;
         }
      }

      // ---- L2 prefetch of the CTA that takes this slot one wave later: its
      // signal and filter requests reach HBM while this CTA computes
      if constexpr(IN == In::C32) {
         if(threadIdx.x == 0 && args.prefetch_ahead > 0) {
            const long long nt0 = tr0 + args.prefetch_ahead * CPB;
            if(nt0 < args.batch) {
               const long long left = args.batch - nt0;
               const uint32_t cnt = (uint32_t)(left < CPB ? left : CPB);
               prefetch_l2_bulk(static_cast<const float2*>(args.a) + (size_t)nt0 * N, cnt * N * 8);
               if constexpr(HAS_FILTER)
                  if(args.filter_stride == N)
                     prefetch_l2_bulk(static_cast<const unsigned char*>(args.b) + (size_t)nt0 * N * FELEM,
                                      cnt * N * FELEM);
            }
         }
      }

      // ---- filter prefetch: one bulk copy per transform, completes on fbar
      if constexpr(HAS_FILTER && FLT == Flt::SMEM) {
         if(threadIdx.x == 0) {
            mbar_init(&fbar, 1);
            fence_mbar_init();
         }
         __syncthreads();
         if(threadIdx.x == 0) {
            const long long left = args.batch - tr0;
            const int nact = left < CPB ? (int)left : CPB;
            mbar_expect_tx(&fbar, (uint32_t)(nact * N * FELEM));
            const unsigned char* fb = static_cast<const unsigned char*>(args.b);
            for(int s = 0; s < nact; ++s)
               bulk_g2s(F + (size_t)s * N * FELEM, fb + (size_t)filter_off(args, tr0 + s) * FELEM,
                        (uint32_t)(N * FELEM), &fbar);
         }
      }

      float2 x[R];

      if constexpr(!SPEC_IN) {
         // ---- first DIF pass straight from HBM: x[s*r + k] = a[lane + T*(s + G*k)]
         constexpr int r0 = C::radix(0), G0 = R / r0;
         float sa = 1.0f;
         if constexpr(IN == In::BFP && !FOLD) sa = active ? __ldg(args.a_scale + tr) : 0.0f;
#pragma unroll
         for(int s = 0; s < G0; ++s)
#pragma unroll
            for(int k = 0; k < r0; ++k) {
               const size_t gi = gbase + lane + (size_t)T * (s + G0 * k);
               float2 v = make_float2(0.f, 0.f);
               if(active) {
                  if constexpr(IN == In::C32) {
                     v = ld_stream(static_cast<const float2*>(args.a) + gi);
                     if constexpr(OUT == Out::NAT)
                        if(args.conj_io) v.y = -v.y;
                  }
                  else if constexpr(IN == In::BFP)
                     v = bfp_dequant(ld_stream(static_cast<const uint32_t*>(args.a) + gi), sa);
                  else v = make_float2(ld_stream(static_cast<const float*>(args.a) + gi),
                                       ld_stream(static_cast<const float*>(args.a2) + gi));
               }
               x[s * r0 + k] = v;
            }
         fwd_all(X, off, x, lane, slot, args.tw, std::make_integer_sequence<int, C::NP>{});
      } else {
         // ---- split apply: the spectrum enters at the boundary.  Default
         // cache policy: a spectrum is usually reused (one spectrum, many
         // filters), and an evict-first load would push it out of L2
         const float2* sp = static_cast<const float2*>(args.a) + (size_t)spec_row;
         if constexpr(IN == In::SPEC_BP) {
#pragma unroll
            for(int k = 0; k < R; ++k) x[k] = active ? __ldg(sp + lane + k * T) : make_float2(0.f, 0.f);
         } else if constexpr(IN == In::SPEC_R8 || IN == In::SPEC_R8BP) {
            static_assert(R == 16 && T >= 32 && C::H == 1, "radix-16 engine, whole warps per transform");
            perm_in<IN == In::SPEC_R8BP>(sp, X + off + 512 * (lane >> 5), lane, active, x);
         } else if constexpr(SPEC_ROWS) {
            rows_in(sp + 32 * R * (lane >> 5), X + off + 32 * R * (lane >> 5), lane & 31, active, x);
         } else {
            const float4* sp4 = reinterpret_cast<const float4*>(sp + (size_t)lane * R);
#pragma unroll
            for(int k = 0; k < R; k += 2) {
               float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
               if(active) v = __ldg(sp4 + k / 2);
               x[k] = make_float2(v.x, v.y);
               x[k + 1] = make_float2(v.z, v.w);
            }
         }
      }

      // ---- register boundary: x[k] is the spectrum at chain position R*lane + k
      if constexpr(OUT == Out::NAT) {
         // natural order: scatter through the exchange buffer, store coalesced
         static_assert(C::NPC == 0, "natural-order output of 1-D chains");
         sched_fence();
         slot_sync<T, CPB>(slot);   // every thread is past its last read of X
         {
            const int nl = off + lane_natural<C>(lane);
            if constexpr(T % SwzEngine::PERIOD == 0) {
               const int q = SwzEngine::map(nl);   // k*T leaves the swizzle's bits alone
#pragma unroll
               for(int k = 0; k < R; ++k) X[q + k * T] = x[k];
            } else {
#pragma unroll
               for(int k = 0; k < R; ++k) X[SwzEngine::map(nl + k * T)] = x[k];
            }
         }
         slot_sync<T, CPB>(slot);
         if(active) {
            const float sgn = args.conj_io ? -1.0f : 1.0f;
#pragma unroll
            for(int u = 0; u < R; ++u) {
               const float2 v = X[SwzEngine::map(off + lane + T * u)];
               st_stream(static_cast<float2*>(args.out) + gbase + lane + T * u, make_float2(v.x, sgn * v.y));
            }
         }
         return;
      } else if constexpr(SPEC_OUT) {
         if(args.spec_scale != 0.0f) {
#pragma unroll
            for(int k = 0; k < R; ++k) x[k] = make_float2(x[k].x * args.spec_scale, x[k].y * args.spec_scale);
         }
         if(active) {
            if constexpr(OUT == Out::SPEC_BP) {
               float2* sp = static_cast<float2*>(args.out) + gbase;
#pragma unroll
               for(int k = 0; k < R; ++k) st_stream(sp + lane + k * T, x[k]);
            } else if constexpr(OUT == Out::SPEC_R8 || OUT == Out::SPEC_R8BP) {
               static_assert(R == 16 && T >= 32 && C::H == 1, "radix-16 engine, whole warps per transform");
               perm_out<OUT == Out::SPEC_R8BP>(x, X + off + 512 * (lane >> 5),
                                               static_cast<float2*>(args.out) + gbase, lane);
            } else if constexpr(SPEC_ROWS) {
               rows_out(x, X + off + 32 * R * (lane >> 5),
                        static_cast<float2*>(args.out) + gbase + 32 * R * (lane >> 5), lane & 31);
            } else {
               float4* sp = reinterpret_cast<float4*>(static_cast<float2*>(args.out) + gbase + (size_t)lane * R);
#pragma unroll
               for(int k = 0; k < R; k += 2)
                  st_stream(sp + k / 2, make_float4(x[k].x, x[k].y, x[k + 1].x, x[k + 1].y));
            }
         }
         return;
      } else {
         if constexpr(MID != Mid::NONE) {
            float2 f[R];
            if constexpr(FLT == Flt::BP_DIRECT) {
               static_assert(!FBFP, "fp32 filters only");
               const float2* fb = static_cast<const float2*>(args.b) + (size_t)filter_off(args, tr) + lane;
#pragma unroll
               for(int k = 0; k < R; ++k) f[k] = active ? __ldg(fb + k * T) : make_float2(0.f, 0.f);
            } else if constexpr(FLT == Flt::LIN_STAGED) {
               // chain-order filter (the reference's mixedrev16 / mixedrev
               // layouts): lane needs the R consecutive values at R*lane --
               // staged warp by warp through its own exchange slots (rows_in)
               static_assert(!FBFP && T >= 32, "fp32, at least one warp per transform");
               const int w = lane >> 5;
               rows_in(static_cast<const float2*>(args.b) + (size_t)filter_off(args, tr) + 32 * R * w,
                       X + off + 32 * R * w, lane & 31, active, f);
            } else if constexpr(FLT == Flt::R8BP_DIRECT) {
               // the radix-8 register-boundary filter read straight from
               // global memory: q = map(16 lane + k) splits into a lane part
               // and a constant per k (map is a bit permutation), and the low
               // lane bits land on bits 0 and 1 of q, so every four lanes read
               // one whole 32-byte sector per load
               // (shapes whose low lane bits miss those bits stage instead)
               static_assert(!FBFP && T >= 32 && R == 16, "fp32 radix-16 engine, at least one warp per transform");
               using PM = R8Perm<C, true>;
               if constexpr(PM::lanes_cover_q01()) {
                  constexpr typename PM::Tables TB = PM::tables();   // evaluated at compile time
                  int ql = 0;
#pragma unroll
                  for(int t = 0; t + 4 < PM::LB; ++t) ql |= ((lane >> t) & 1) << TB.sig[4 + t];
                  const float2* fb = static_cast<const float2*>(args.b) + (size_t)filter_off(args, tr) + ql;
#pragma unroll
                  for(int k = 0; k < R; ++k) f[k] = active ? __ldg(fb + TB.mapk[k]) : make_float2(0.f, 0.f);
               } else {
                  perm_in<true>(static_cast<const float2*>(args.b) + (size_t)filter_off(args, tr),
                                X + off + 512 * (lane >> 5), lane, active, f);
               }
            } else if constexpr(FLT == Flt::R8_STAGED || FLT == Flt::R8BP_STAGED) {
               // a filter in a radix-8 layout: the warp's 512 values sit at
               // q = map(512 w + local p), a bit permutation (perm_in)
               static_assert(!FBFP && T >= 32 && R == 16, "fp32 radix-16 engine, at least one warp per transform");
               perm_in<FLT == Flt::R8BP_STAGED>(static_cast<const float2*>(args.b) + (size_t)filter_off(args, tr),
                                                X + off + 512 * (lane >> 5), lane, active, f);
            } else if constexpr(FLT == Flt::SMEM) {
               mbar_wait(&fbar, 0, args.status);
               if constexpr(FBFP) {
                  const uint32_t* Fs = reinterpret_cast<const uint32_t*>(F) + off;
                  const float sb = FOLD ? 1.0f : filter_scale(args, tr, active);
#pragma unroll
                  for(int k = 0; k < R; ++k) f[k] = bfp_dequant(Fs[lane + k * T], sb);
               } else {
                  const float2* Fs = reinterpret_cast<const float2*>(F) + off;
#pragma unroll
                  for(int k = 0; k < R; ++k) f[k] = Fs[lane + k * T];
               }
            } else {
               const size_t fbase = (size_t)filter_off(args, tr) + (size_t)lane * R;
               if constexpr(FBFP) {
                  const float sb = FOLD ? 1.0f : filter_scale(args, tr, active);
                  const uint4* fp = reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(args.b) + fbase);
#pragma unroll
                  for(int k = 0; k < R; k += 4) {
                     uint4 w = make_uint4(0, 0, 0, 0);
                     if(active) w = __ldg(fp + k / 4);
                     f[k] = bfp_dequant(w.x, sb); f[k + 1] = bfp_dequant(w.y, sb);
                     f[k + 2] = bfp_dequant(w.z, sb); f[k + 3] = bfp_dequant(w.w, sb);
                  }
               } else {
                  const float4* fp = reinterpret_cast<const float4*>(static_cast<const float2*>(args.b) + fbase);
#pragma unroll
                  for(int k = 0; k < R; k += 2) {
                     float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                     if(active) v = __ldg(fp + k / 2);
                     f[k] = make_float2(v.x, v.y);
                     f[k + 1] = make_float2(v.z, v.w);
                  }
               }
            }
#pragma unroll
            for(int k = 0; k < R; ++k) x[k] = (MID == Mid::MUL) ? cmul(x[k], f[k]) : cmulc(x[k], f[k]);
         }

         inv_all(X, off, x, lane, slot, args.tw, std::make_integer_sequence<int, C::NP>{});

         // ---- last DIT pass straight to HBM at the first pass's positions
         constexpr int r0 = C::radix(0), G0 = R / r0;
         if constexpr(OUT == Out::BFP) {
            float m = 0.0f;
#pragma unroll
            for(int i = 0; i < R; ++i) m = fmaxf(m, fmaxf(fabsf(x[i].x), fabsf(x[i].y)));
            if constexpr(T >= 32) {
#pragma unroll
               for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
               if((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
               slot_sync<T, CPB>(slot);
               m = 0.0f;
#pragma unroll
               for(int w = 0; w < T / 32; ++w) m = fmaxf(m, warp_max[slot * (T / 32) + w]);
            } else {
#pragma unroll
               for(int o = T / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            }
            // m is the abs-max of the raw result; the true one is m * fold
            float fold = active ? __ldg(args.a_scale + tr) : 0.0f;
            if constexpr(HAS_FILTER && FBFP) fold *= filter_scale(args, tr, active);
            const float mx = fmaxf(m * fold, 1e-30f);
            const float inv = (32767.0f / mx) * fold;
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
               for(int k = 0; k < r0; ++k) {
                  const size_t gi = obase + lane + (size_t)T * (s + G0 * k);
                  const float2 v = x[s * r0 + k];
                  if constexpr(OUT == Out::C32) st_stream(static_cast<float2*>(args.out) + gi, v);
                  else {
                     st_stream(static_cast<float*>(args.out) + gi, v.x);
                     st_stream(static_cast<float*>(args.out2) + gi, v.y);
                  }
               }
         }
      }
   }
};

// occupancy target in resident threads per SM.  fp32: 512 (two 256-thread
// CTAs, up to 128 registers per thread, no spills).  int16-BFP: 1024 (64
// registers): the BFP kernel moves half the bytes and is bound by issue and
// latency, and four CTAs per SM measured 10-20% faster at N = 512..4096;
// fp32 measured 3-9% slower at 768 or 1024 with the filter tile in shared
// memory (see resident_for below for the one fp32 case that runs 768).
#ifndef FUFFT_RESIDENT_THREADS
#define FUFFT_RESIDENT_THREADS 512
#endif
#ifndef FUFFT_RESIDENT_THREADS_BFP
#define FUFFT_RESIDENT_THREADS_BFP 1024
#endif
template<int THREADS, int RESIDENT = FUFFT_RESIDENT_THREADS> constexpr int min_blocks()
{
   return THREADS >= RESIDENT ? 1 : RESIDENT / THREADS;
}

// natural-order output (one transform direction, no filter): three CTAs per
// SM, as the spectrum-output kernels reach on their own (~80 registers)
#ifndef FUFFT_RESIDENT_THREADS_APPLY
#define FUFFT_RESIDENT_THREADS_APPLY 1024
#endif
template<In IN, Out OUT> constexpr int resident_threads()
{
   return IN == In::BFP ? FUFFT_RESIDENT_THREADS_BFP
        : OUT == Out::NAT ? 768
        : IN == In::SPEC_BP ? FUFFT_RESIDENT_THREADS_APPLY
                            : FUFFT_RESIDENT_THREADS;
}

// 1-D radix-16 fp32 convolution (complex or two-for-one real) of n >= 2048
// with the register-boundary filter read straight from global memory (no
// 32 KB shared-memory filter tile per CTA): three CTAs of 256 threads per SM
// at <= 80 registers, no spills.  Against two CTAs with the filter tile:
// +8-9% at n = 4096 and +4-6% at 2048 for the complex convolution, +6-8% at
// 4096 for the two-for-one real one (B200, 1 GiB batches).  At n <= 1024,
// and for the natural-order kernels, 768 threads measured 2-7% slower, so
// they keep their targets.
#ifndef FUFFT_RESIDENT_THREADS_CONV_DIRECT
#define FUFFT_RESIDENT_THREADS_CONV_DIRECT 768
#endif
#ifndef FUFFT_CONV_DIRECT_MIN_N
#define FUFFT_CONV_DIRECT_MIN_N 2048
#endif
constexpr int CONV_DIRECT_MIN_N = FUFFT_CONV_DIRECT_MIN_N;
// n = 1024 launches of a few waves (up to CONV_DIRECT_SMALL_POINTS points) read
// the register-boundary filter directly at three CTAs per SM too: back-to-back
// 4096-transform launches 22.3 -> 21.3 us (B200, four input sets in turn);
// at 2^24 points even, at 1 GiB 1% slower, so larger launches keep the tile
constexpr int CONV_DIRECT_SMALL_N = 1024;
constexpr long long CONV_DIRECT_SMALL_POINTS = 1LL << 23;
// fp32 radix-8 convolution of n >= 2048 (one transform per CTA, 256 or 512
// threads): two or more CTAs per SM at <= 64 registers.  At the 512-thread
// target one 512-thread CTA of 67 registers filled the SM: 16 warps, issue
// 44% (ncu, n = 4096).
#ifndef FUFFT_RESIDENT_THREADS_R8
#define FUFFT_RESIDENT_THREADS_R8 1024
#endif
template<class C, In IN, Out OUT, Flt FLT> constexpr int resident_for()
{
   return (((IN == In::C32 && OUT == Out::C32) || (IN == In::REAL2 && OUT == Out::REAL2)) &&
           (FLT == Flt::BP_DIRECT || FLT == Flt::LIN_STAGED || FLT == Flt::R8_STAGED || FLT == Flt::R8BP_STAGED ||
            FLT == Flt::R8BP_DIRECT) &&
           C::R == 16 && (C::N >= CONV_DIRECT_MIN_N || (FLT == Flt::BP_DIRECT && C::N == CONV_DIRECT_SMALL_N)))
             ? FUFFT_RESIDENT_THREADS_CONV_DIRECT
        : (IN == In::C32 && OUT == Out::C32 && C::H == 1 && C::R == 8 && C::N >= CONV_DIRECT_MIN_N)
             ? FUFFT_RESIDENT_THREADS_R8
             : resident_threads<IN, OUT>();
}

template<class C, int CPB, In IN, Out OUT, Mid MID, Flt FLT, bool FBFP>
__global__ void __launch_bounds__(CPB * C::T, min_blocks<CPB * C::T, resident_for<C, IN, OUT, FLT>()>())
conv_kernel(const ConvArgs args)
{
   ConvKernel<C, CPB, IN, OUT, MID, FLT, FBFP>::run(args);
}

}  // namespace fufft
