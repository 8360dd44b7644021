// fufft_large.cu -- four-step convolution for N beyond one kernel
// (bench_fufft.cu:391-492 run_large, fufft.cuh:1081-1140):
//
//   LOUT outer DIF passes of radix r_out over HBM (strides N/r_out .. MID)
//   -> the fused one-kernel convolution on every MID-point chunk (the chunks
//      pose as batch items; after the outer passes every remaining butterfly
//      group lives inside one chunk)
//   -> LOUT outer DIT passes (strides MID .. N/r_out).
// The filter arrives in the chain order of the whole radix sequence
// [r_out] x LOUT ++ middle chain, so each chunk sees its own chain-ordered
// slice (optionally in the middle's register-boundary layout).
//
// The outer pass: one thread per butterfly group (R taps at stride M),
// consecutive threads take consecutive j so every tap load and store is one
// coalesced 256-byte warp access; the group twiddle W_{RM}^j comes from
// sincospif on an exact argument (2j/(RM) is a dyadic fraction) and its powers
// from the register product tree.  int16-BFP variants dequantise on the way
// in (first pass) and reduce the per-transform abs-max on the way out (last
// pass) for the requantisation.
#include "fufft_internal.cuh"

namespace fufft {

enum class OuterMode { F32, BFP_IN, F32_ABSMAX };

struct OuterArgs {
   const void* src;           // fp32 complex, or packed int16 pairs (BFP_IN)
   float2* dst;
   const float* scale;        // BFP_IN: one scale per transform
   unsigned int* absmax;      // F32_ABSMAX: per-transform max |re|,|im| (fp32 bits)
   long long ngroups;         // batch * n / R
   long long n;               // transform size
   int M;                     // stride of this pass (a power of two)
   int logM, logn;
};

template<int R, int S, OuterMode MODE>
__global__ void __launch_bounds__(256) outer_pass_kernel(const OuterArgs args)
{
   const long long M = args.M;
   const float inv_rm = 1.0f / (float)(R * M);
   for(long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < args.ngroups;
       g += (long long)gridDim.x * blockDim.x) {
      const long long j = g & (M - 1), b = g >> args.logM;
      const long long base = b * R * M + j;
      float2 u[R];
      if constexpr(MODE == OuterMode::BFP_IN) {
         const float sc = __ldg(args.scale + (base >> args.logn));
         const uint32_t* w = static_cast<const uint32_t*>(args.src);
#pragma unroll
         for(int k = 0; k < R; ++k) u[k] = bfp_dequant(ld_stream(w + base + k * M), sc);
      } else {
         const float2* x = static_cast<const float2*>(args.src);
#pragma unroll
         for(int k = 0; k < R; ++k) u[k] = ld_stream(x + base + k * M);
      }
      float2 w[R];
      if(j) {
         float sn, cs;
         sincospif(-2.0f * (float)j * inv_rm, &sn, &cs);
         twiddle_powers<R>(make_float2(cs, sn), w);
      } else {
#pragma unroll
         for(int k = 1; k < R; ++k) w[k] = make_float2(1.0f, 0.0f);
      }
      if constexpr(S > 0) {
#pragma unroll
         for(int k = 1; k < R; ++k) u[k] = cmulc(u[k], w[k]);
      }
      dft<R, S>(u);
      if constexpr(S < 0) {
#pragma unroll
         for(int k = 1; k < R; ++k) u[k] = cmul(u[k], w[k]);
      }
#pragma unroll
      for(int k = 0; k < R; ++k) st_stream(args.dst + base + k * M, u[k]);
      if constexpr(MODE == OuterMode::F32_ABSMAX) {
         // a warp's groups belong to one transform (n/R is a multiple of 32)
         float m = 0.0f;
#pragma unroll
         for(int k = 0; k < R; ++k) m = fmaxf(m, fmaxf(fabsf(u[k].x), fabsf(u[k].y)));
#pragma unroll
         for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
         if((threadIdx.x & 31) == 0) atomicMax(args.absmax + (base >> args.logn), __float_as_uint(m));
      }
   }
}

// powers w[k] = W^{jk} of the group twiddle W^j = exp(-2 pi i j / L), from an
// exact sincospif argument (2j/L is a dyadic fraction) and the product tree
template<int R>
__device__ __forceinline__ void outer_twiddles(long long j, float inv_l, float2 (&w)[R])
{
   if(j) {
      float sn, cs;
      sincospif(-2.0f * (float)j * inv_l, &sn, &cs);
      twiddle_powers<R>(make_float2(cs, sn), w);
   } else {
#pragma unroll
      for(int k = 1; k < R; ++k) w[k] = make_float2(1.0f, 0.0f);
   }
}

// DIF (S = -1): butterfly then W^{jk}; DIT (S = +1): conj(W^{jk}) then butterfly
template<int R, int S>
__device__ __forceinline__ void outer_butterfly(float2 (&u)[R], long long j, float inv_l)
{
   float2 w[R];
   outer_twiddles<R>(j, inv_l, w);
   if constexpr(S > 0) {
#pragma unroll
      for(int k = 1; k < R; ++k) u[k] = cmulc(u[k], w[k]);
   }
   dft<R, S>(u);
   if constexpr(S < 0) {
#pragma unroll
      for(int k = 1; k < R; ++k) u[k] = cmul(u[k], w[k]);
   }
}

// Two consecutive outer levels in one HBM round trip: level A at stride M
// (args.M) and level B at stride Mb = M / R.  Positions
//     b*R*M + j' + k2*Mb + k1*M,   k1, k2 < R,  j' < Mb
// of one block b and one j' form a closed R x R sub-problem: level A runs
// over k1 (group j = j' + k2*Mb, twiddle W_{RM}^{j k1}), level B over k2
// (group j', twiddle W_M^{j' k2}).  A CTA of 256 threads takes J = 256/R
// consecutive j' (128 or 256 contiguous bytes per row: coalesced), does one
// level in registers (thread = (k2, j') for A, (k1, j') for B), exchanges
// through a shared tile [k1][k2][j'] (conflict-free both ways: 32 consecutive
// slots per warp access) and does the other level.  DIF: A then B; DIT: B
// then A.  In place is safe: a CTA reads its whole tile before it writes.
template<int R, int S, OuterMode MODE>
__global__ void __launch_bounds__(256) outer2_pass_kernel(const OuterArgs args)
{
   constexpr int J = 256 / R;
   __shared__ float2 tile[R * R * J];
   const long long M = args.M, Mb = M / R;
   const float inv_a = 1.0f / (float)(R * M), inv_b = 1.0f / (float)M;
   const long long tiles_per_block = Mb / J;
   const long long ntiles = args.ngroups / (R * J);      // ngroups = batch * n / R
   const int q = threadIdx.x / J, jj = threadIdx.x % J;
   for(long long t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const long long b = t / tiles_per_block, jp = (t % tiles_per_block) * J + jj;
      const long long base = b * R * M + jp;
      float2 u[R];
      if constexpr(S < 0) {
         // level A, thread (k2 = q): taps k1 at base + q*Mb + k1*M
         const long long pa = base + q * Mb;
         if constexpr(MODE == OuterMode::BFP_IN) {
            const float sc = __ldg(args.scale + (base >> args.logn));
            const uint32_t* w = static_cast<const uint32_t*>(args.src);
#pragma unroll
            for(int k = 0; k < R; ++k) u[k] = bfp_dequant(ld_stream(w + pa + k * M), sc);
         } else {
            const float2* x = static_cast<const float2*>(args.src);
#pragma unroll
            for(int k = 0; k < R; ++k) u[k] = ld_stream(x + pa + k * M);
         }
         outer_butterfly<R, S>(u, jp + q * Mb, inv_a);
#pragma unroll
         for(int k = 0; k < R; ++k) tile[(k * R + q) * J + jj] = u[k];
         __syncthreads();
         // level B, thread (k1 = q): taps k2
#pragma unroll
         for(int k = 0; k < R; ++k) u[k] = tile[(q * R + k) * J + jj];
         outer_butterfly<R, S>(u, jp, inv_b);
         const long long pb = base + q * M;
#pragma unroll
         for(int k = 0; k < R; ++k) st_stream(args.dst + pb + k * Mb, u[k]);
      } else {
         // level B first, thread (k1 = q): taps k2 at base + q*M + k2*Mb
         const float2* x = static_cast<const float2*>(args.src);
         const long long pb = base + q * M;
#pragma unroll
         for(int k = 0; k < R; ++k) u[k] = ld_stream(x + pb + k * Mb);
         outer_butterfly<R, S>(u, jp, inv_b);
#pragma unroll
         for(int k = 0; k < R; ++k) tile[(q * R + k) * J + jj] = u[k];
         __syncthreads();
         // level A, thread (k2 = q): taps k1
#pragma unroll
         for(int k = 0; k < R; ++k) u[k] = tile[(k * R + q) * J + jj];
         outer_butterfly<R, S>(u, jp + q * Mb, inv_a);
         const long long pa = base + q * Mb;
#pragma unroll
         for(int k = 0; k < R; ++k) st_stream(args.dst + pa + k * M, u[k]);
         if constexpr(MODE == OuterMode::F32_ABSMAX) {
            // the whole tile lies in one transform (R*M <= n)
            float m = 0.0f;
#pragma unroll
            for(int k = 0; k < R; ++k) m = fmaxf(m, fmaxf(fabsf(u[k].x), fabsf(u[k].y)));
#pragma unroll
            for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if((threadIdx.x & 31) == 0) atomicMax(args.absmax + (base >> args.logn), __float_as_uint(m));
         }
      }
      __syncthreads();   // the next tile reuses the shared tile
   }
}

namespace host {

template<int R, int S, OuterMode MODE>
static fufft_status outer(OuterArgs a, cudaStream_t st, int device)
{
   a.logM = ilog2c(a.M);
   a.logn = ilog2c(a.n);
   const long long blocks_needed = (a.ngroups + 255) / 256;
   const long long cap = (long long)sm_count(device) * 8;
   outer_pass_kernel<R, S, MODE><<<(unsigned)(blocks_needed < cap ? blocks_needed : cap), 256, 0, st>>>(a);
   count_launch();
   return check(cudaGetLastError());
}

template<int S, OuterMode MODE>
static fufft_status outer_r(int r, const OuterArgs& a, cudaStream_t st, int device)
{
   return r == 8 ? outer<8, S, MODE>(a, st, device) : outer<16, S, MODE>(a, st, device);
}

// levels at strides a.M and a.M / R in one launch (outer2_pass_kernel)
template<int R, int S, OuterMode MODE>
static fufft_status outer2(OuterArgs a, cudaStream_t st, int device)
{
   a.logM = ilog2c(a.M);
   a.logn = ilog2c(a.n);
   const long long tiles = a.ngroups / 256;
   const long long cap = (long long)sm_count(device) * 8;
   outer2_pass_kernel<R, S, MODE><<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, st>>>(a);
   count_launch();
   return check(cudaGetLastError());
}

#ifndef FUFFT_OUTER_FUSE
#define FUFFT_OUTER_FUSE 1
#endif
// The outer levels of one direction, fused two by two where possible (a pair
// needs the inner stride M/R >= 256/R columns).  DIF (S = -1): strides
// m_top, m_top/R, ..., R*mid... down to mid, pairs from the top; the first
// launch may dequantise int16 input (first_mode BFP_IN).  DIT (S = +1):
// strides mid, mid*R, ..., pairs from the bottom; the last launch may reduce
// the per-transform abs-max (last_mode F32_ABSMAX).
template<int S>
static fufft_status outer_levels(int r, OuterArgs a, long long mid, int lout, bool bfp_in, bool absmax,
                                 float2* ws_after_first, cudaStream_t st, int device)
{
   const long long n = a.n;
   fufft_status s = FUFFT_OK;
   if constexpr(S < 0) {
      long long M = n / r;
      for(int l = 0; l < lout;) {
         const bool first = l == 0;
         const bool pair = FUFFT_OUTER_FUSE && l + 1 < lout && M / r >= 256 / r;
         a.M = (int)M;
         if(pair) {
            if(first && bfp_in)
               s = r == 8 ? outer2<8, -1, OuterMode::BFP_IN>(a, st, device) : outer2<16, -1, OuterMode::BFP_IN>(a, st, device);
            else
               s = r == 8 ? outer2<8, -1, OuterMode::F32>(a, st, device) : outer2<16, -1, OuterMode::F32>(a, st, device);
            M /= (long long)r * r;
            l += 2;
         } else {
            s = (first && bfp_in) ? outer_r<-1, OuterMode::BFP_IN>(r, a, st, device)
                                  : outer_r<-1, OuterMode::F32>(r, a, st, device);
            M /= r;
            l += 1;
         }
         if(s != FUFFT_OK) return s;
         if(first && ws_after_first) a.src = ws_after_first;   // later passes read the fp32 workspace
      }
   } else {
      long long M = mid;
      for(int l = 0; l < lout;) {
         const bool pair = FUFFT_OUTER_FUSE && l + 1 < lout && M >= 256 / r;
         const bool last = l + (pair ? 2 : 1) == lout;
         if(pair) {
            a.M = (int)(M * r);
            if(last && absmax)
               s = r == 8 ? outer2<8, 1, OuterMode::F32_ABSMAX>(a, st, device)
                          : outer2<16, 1, OuterMode::F32_ABSMAX>(a, st, device);
            else
               s = r == 8 ? outer2<8, 1, OuterMode::F32>(a, st, device) : outer2<16, 1, OuterMode::F32>(a, st, device);
            M *= (long long)r * r;
            l += 2;
         } else {
            a.M = (int)M;
            s = (last && absmax) ? outer_r<+1, OuterMode::F32_ABSMAX>(r, a, st, device)
                                 : outer_r<+1, OuterMode::F32>(r, a, st, device);
            M *= r;
            l += 1;
         }
         if(s != FUFFT_OK) return s;
      }
   }
   return FUFFT_OK;
}

}  // namespace host
}  // namespace fufft

using namespace fufft;
using namespace fufft::host;

namespace {

// N = r_out^LOUT * mid with mid a one-kernel size of the layout's radix
fufft_status check_plan(long long n, int r_out, int mid, fufft_layout layout, int* lout)
{
   const int R = layout_radix(layout);
   if(!R) return FUFFT_ERR_INVALID_ARG;
   if(r_out != 8 && r_out != 16) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(n) || !pow2(mid) || mid < 256 || mid > max_n(R) || n <= mid || n % mid) return FUFFT_ERR_INVALID_SIZE;
   long long q = n / mid;
   int l = 0;
   while(q > 1) {
      if(q % r_out) return FUFFT_ERR_INVALID_SIZE;   // n/mid must be a power of r_out
      q /= r_out;
      ++l;
   }
   if(n > (1LL << 31)) return FUFFT_ERR_INVALID_SIZE;
   *lout = l;
   return FUFFT_OK;
}

// the middle: the fused one-kernel convolution over the mid-point chunks
fufft_status run_middle(float2* buf, const void* b, const float* b_scale, long long chunks, int mid,
                        long long chunks_per_transform, fufft_layout layout, fufft_midop midop, bool bfp_filter,
                        const DeviceCtx& c, cudaStream_t st)
{
   ConvArgs args{};
   args.tw = c.tw;
   args.status = c.status;
   args.batch = chunks;
   args.a = buf;
   args.out = buf;
   args.b = b;
   args.b_scale = b_scale;
   args.filter_stride = mid;
   args.scale_div = chunks_per_transform;
   const int R = layout_radix(layout);
   const bool bperm = layout_bperm(layout);
   if(bfp_filter)
      return (R == 8 ? family_mid_bfpfilter_r8 : family_mid_bfpfilter_r16)(mid, midop, bperm, args, st, c.device);
   return (R == 8 ? family_conv_f32_r8 : family_conv_f32_r16)(mid, midop, bperm, args, st, c.device);
}

}  // namespace

extern "C" {

fufft_status fufft_large_plan(int64_t n, fufft_layout layout, int* r_out, int* mid)
{
   const int R = layout_radix(layout);
   if(!R || !r_out || !mid) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(n) || n <= max_n(R)) return FUFFT_ERR_INVALID_SIZE;
   // radix-16 outer levels first (fewest HBM passes), then radix 8
   for(int ro : {16, 8})
      for(long long m = max_n(R); m >= 256; m /= 2) {
         int l;
         if(check_plan(n, ro, (int)m, layout, &l) == FUFFT_OK) {
            *r_out = ro;
            *mid = (int)m;
            return FUFFT_OK;
         }
      }
   return FUFFT_ERR_INVALID_SIZE;
}

fufft_status fufft_conv_large_f32(float* buf, const float* b, int64_t n, int64_t batch, int r_out, int mid,
                                  fufft_layout layout, fufft_midop midop, fufft_stream_t stream)
{
   int lout = 0;
   fufft_status s = check_plan(n, r_out, mid, layout, &lout);
   if(s != FUFFT_OK) return s;
   if(batch < 0 || batch * n > (1LL << 40)) return FUFFT_ERR_INVALID_BATCH;
   if(batch == 0) return FUFFT_OK;
   if(!buf) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(buf, 16)) return FUFFT_ERR_MISALIGNED;
   if(midop < FUFFT_MID_NONE || midop > FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   if(midop != FUFFT_MID_NONE && (!b || !aligned(b, 16))) return b ? FUFFT_ERR_MISALIGNED : FUFFT_ERR_INVALID_ARG;
   DeviceCtx c;
   if((s = device_ctx(&c)) != FUFFT_OK) return s;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   float2* x = reinterpret_cast<float2*>(buf);
   if(lout == 1 && layout_radix(layout) == 16) {
      // one outer level: the cluster-fused kernel does the whole four-step in
      // one launch and 3 HBM passes (it reads every input of a transform
      // before its first cluster barrier and writes after its last, so in
      // place is safe); fall through to the multi-kernel form if the device
      // cannot host the cluster
      ConvArgs ca{};
      ca.tw = c.tw;
      ca.status = c.status;
      ca.batch = batch;
      ca.a = buf;
      ca.out = buf;
      ca.b = b;
      ca.filter_stride = n;
      s = cluster_large(r_out, mid, midop, layout_bperm(layout), ca, st, c.device);
      if(s != FUFFT_ERR_UNSUPPORTED) return s;
   }
   OuterArgs oa{};
   oa.dst = x;
   oa.src = x;
   oa.n = n;
   oa.ngroups = batch * n / r_out;
   if((s = outer_levels<-1>(r_out, oa, mid, lout, false, false, nullptr, st, c.device)) != FUFFT_OK) return s;
   if((s = run_middle(x, b, nullptr, batch * n / mid, mid, n / mid, layout, midop, false, c, st)) != FUFFT_OK)
      return s;
   return outer_levels<+1>(r_out, oa, mid, lout, false, false, nullptr, st, c.device);
}

size_t fufft_conv_large_bfp_workspace(int64_t n, int64_t batch)
{
   return n > 0 && batch > 0 ? (size_t)n * (size_t)batch * sizeof(float2) : 0;
}

}  // extern "C"

namespace fufft {
namespace host {

// argument checks of the int16-BFP four-step, in the order
// fufft_conv_large_bfp applies them; the workspace is checked only when
// check_workspace is set.  FUFFT_OK with *nothing_to_do set: batch 0.
fufft_status validate_large_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq, const float* b_scale,
                                const int16_t* oq, const float* o_scale, int64_t n, int64_t batch, int r_out,
                                int mid, fufft_layout layout, fufft_midop midop, bool check_workspace,
                                const void* workspace, size_t workspace_bytes, int* lout, bool* nothing_to_do)
{
   *nothing_to_do = false;
   fufft_status s = check_plan(n, r_out, mid, layout, lout);
   if(s != FUFFT_OK) return s;
   if(batch < 0 || batch * n > (1LL << 40)) return FUFFT_ERR_INVALID_BATCH;
   if(batch == 0) {
      *nothing_to_do = true;
      return FUFFT_OK;
   }
   if(!aq || !a_scale || !oq || !o_scale || (check_workspace && !workspace)) return FUFFT_ERR_INVALID_ARG;
   if(check_workspace && workspace_bytes < fufft_conv_large_bfp_workspace(n, batch)) return FUFFT_ERR_INVALID_ARG;
   if((check_workspace && !aligned(workspace, 16)) || !aligned(aq, 4) || !aligned(oq, 4))
      return FUFFT_ERR_MISALIGNED;
   if(midop < FUFFT_MID_NONE || midop > FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   if(midop != FUFFT_MID_NONE && (!bq || !b_scale)) return FUFFT_ERR_INVALID_ARG;
   if(midop != FUFFT_MID_NONE && !aligned(bq, 16)) return FUFFT_ERR_MISALIGNED;
   return FUFFT_OK;
}

}  // namespace host
}  // namespace fufft

extern "C" {

fufft_status fufft_conv_large_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq, const float* b_scale,
                                  int16_t* oq, float* o_scale, int64_t n, int64_t batch, int r_out, int mid,
                                  fufft_layout layout, fufft_midop midop, void* workspace,
                                  size_t workspace_bytes, fufft_stream_t stream)
{
   int lout = 0;
   bool nothing = false;
   fufft_status s = validate_large_bfp(aq, a_scale, bq, b_scale, oq, o_scale, n, batch, r_out, mid, layout, midop,
                                       true, workspace, workspace_bytes, &lout, &nothing);
   if(s != FUFFT_OK || nothing) return s;
   DeviceCtx c;
   if((s = device_ctx(&c)) != FUFFT_OK) return s;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   if(lout == 1 && layout_radix(layout) == 16) {
      // one outer level: the whole BFP four-step in one cluster kernel, 12 B
      // per point of HBM traffic and no use of the workspace (each CTA reads
      // the positions it later writes, so oq may alias aq); multi-kernel form
      // below if the device cannot host the cluster
      ConvArgs ca{};
      ca.tw = c.tw;
      ca.status = c.status;
      ca.batch = batch;
      ca.a = aq;
      ca.a_scale = a_scale;
      ca.b = bq;
      ca.b_scale = b_scale;
      ca.out = oq;
      ca.out_scale = o_scale;
      ca.filter_stride = n;
      s = cluster_large_bfp(r_out, mid, midop, layout_bperm(layout), ca, st, c.device);
      if(s != FUFFT_ERR_UNSUPPORTED) return s;
   }
   float2* ws = static_cast<float2*>(workspace);
   OuterArgs oa{};
   oa.n = n;
   oa.ngroups = batch * n / r_out;
   // the first DIF launch dequantises into the fp32 workspace
   oa.src = aq;
   oa.dst = ws;
   oa.scale = a_scale;
   if((s = outer_levels<-1>(r_out, oa, mid, lout, true, false, ws, st, c.device)) != FUFFT_OK) return s;
   if((s = run_middle(ws, bq, b_scale, batch * n / mid, mid, n / mid, layout, midop, true, c, st)) != FUFFT_OK)
      return s;
   // inverse passes; the last launch also reduces the per-transform abs-max into o_scale
   if((s = check(cudaMemsetAsync(o_scale, 0, sizeof(float) * batch, st))) != FUFFT_OK) return s;
   oa.src = ws;
   oa.absmax = reinterpret_cast<unsigned int*>(o_scale);
   if((s = outer_levels<+1>(r_out, oa, mid, lout, false, true, nullptr, st, c.device)) != FUFFT_OK) return s;
   return bfp_requantize(ws, o_scale, reinterpret_cast<uint32_t*>(oq), n, batch, st);
}

}  // extern "C"
