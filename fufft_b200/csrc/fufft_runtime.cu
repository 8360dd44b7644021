// fufft_runtime.cu -- per-device state, index maps, filter preparation and
// the int16 block-floating-point pack/unpack kernels of the C ABI.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "fufft_internal.cuh"

namespace fufft {

// twiddle tables (tw_offset layout) and the status word, one copy per device
__device__ float2 g_twiddle[TW_TOTAL];
__device__ unsigned int g_status;

// fill the table: entry L - 2 + j = exp(-2 pi i j / L) from fp64 sincospi,
// rounded once to fp32
__global__ void twiddle_init_kernel()
{
   for(int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < TW_TOTAL; idx += gridDim.x * blockDim.x) {
      int L = 2;
      while(tw_offset(2 * L) <= idx) L *= 2;   // largest L with L - 2 <= idx
      const int j = idx - tw_offset(L);
      double s, c;
      sincospi(-2.0 * (double)j / (double)L, &s, &c);
      g_twiddle[idx] = make_float2((float)c, (float)s);
   }
}

// self-test of the bounded waits: an mbarrier that nothing will complete,
// waited on with a short limit by one thread, which must give up, record
// STATUS_TMA_TIMEOUT and return like every waiting kernel of the library
__global__ void wait_timeout_selftest_kernel(unsigned int* status, uint32_t limit_us)
{
   __shared__ uint64_t bar;
   if(threadIdx.x == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
      mbar_wait(&bar, 0, status, (uint64_t)limit_us * 1000ull);
   }
}

namespace host {

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

struct DevState {
   std::once_flag once;
   fufft_status init_status = FUFFT_OK;
   const float2* tw = nullptr;
   unsigned int* status = nullptr;
};
constexpr int MAX_DEVICES = 64;
DevState g_dev[MAX_DEVICES];

fufft_status init_device(DevState& d)
{
   void* p = nullptr;
   fufft_status s = check(cudaGetSymbolAddress(&p, g_twiddle));
   if(s != FUFFT_OK) return s;
   d.tw = static_cast<const float2*>(p);
   s = check(cudaGetSymbolAddress(&p, g_status));
   if(s != FUFFT_OK) return s;
   d.status = static_cast<unsigned int*>(p);
   // a private stream keeps the one-time build off the caller's streams
   cudaStream_t st;
   s = check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
   if(s != FUFFT_OK) return s;
   twiddle_init_kernel<<<256, 256, 0, st>>>();
   s = check(cudaGetLastError());
   if(s == FUFFT_OK) s = check(cudaMemsetAsync(d.status, 0, sizeof(unsigned int), st));
   if(s == FUFFT_OK) s = check(cudaStreamSynchronize(st));
   cudaStreamDestroy(st);
   return s;
}
}  // namespace

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder()
{
   static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
   static std::once_flag once;
   std::call_once(once, [] {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
         q == cudaDriverEntryPointSuccess)
         fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
   });
   return fn;
}
std::atomic<int> g_sms[MAX_DEVICES];
}  // namespace

fufft_status encode_rows_tmap(CUtensorMap* tm, const void* base, unsigned long long bytes, int box_rows, bool words)
{
   auto fn = tmap_encoder();
   if(!fn) return FUFFT_ERR_UNSUPPORTED;
   if(bytes % 128 || !aligned(base, 16) || box_rows < 1 || box_rows > 256) return FUFFT_ERR_MISALIGNED;
   cuuint64_t dims[2] = {32, bytes / 128};
   cuuint64_t strides[1] = {128};
   cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
   cuuint32_t estr[2] = {1, 1};
   const CUresult r = fn(tm, words ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
   if(r != CUDA_SUCCESS) {
      t_last_error = "cuTensorMapEncodeTiled failed";
      return FUFFT_ERR_CUDA;
   }
   return FUFFT_OK;
}

int sm_count(int device)
{
   int v = g_sms[device & 63].load();
   if(!v) {
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
      if(v <= 0) v = 1;
      g_sms[device & 63].store(v);
   }
   return v;
}

fufft_status cuda_fail(cudaError_t e)
{
   t_last_error = cudaGetErrorString(e);
   return FUFFT_ERR_CUDA;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

fufft_status device_ctx(DeviceCtx* out)
{
   int dev = 0;
   fufft_status s = check(cudaGetDevice(&dev));
   if(s != FUFFT_OK) return s;
   if(dev < 0 || dev >= MAX_DEVICES) return FUFFT_ERR_UNSUPPORTED;
   DevState& d = g_dev[dev];
   std::call_once(d.once, [&] { d.init_status = init_device(d); });
   if(d.init_status != FUFFT_OK) return d.init_status;
   out->tw = d.tw;
   out->status = d.status;
   out->device = dev;
   return FUFFT_OK;
}

}  // namespace host

// ---------------------------------------------------------------------------
// filter permutation: natural-order spectrum -> chain order / register
// boundary order, per transform
// ---------------------------------------------------------------------------
__host__ __device__ inline long long chain_rev_dev(long long idx, const int* w, int p, int m)
{
   long long out = 0;
   int pos = m, op = 0;
   // digit k (width w[k], MSB-first in idx) lands at the mirrored position
   for(int k = 0; k < p; k++) {
      pos -= w[k];
      const long long d = (idx >> pos) & ((1LL << w[k]) - 1);
      out |= d << op;
      op += w[k];
   }
   return out;
}

struct PermPlan {
   long long blk = 0;  // > 0: register-boundary order applies per block of blk points
   int w[32];          // row-dimension (W) chain: bit-group widths in pass order
   int p = 0, m = 0;
   int wh[32];         // column-dimension (H) chain; ph = 0 for 1-D
   int ph = 0, mh = 0;
   int v = 1;          // register-boundary width (1 = plain chain order)
   int T = 1;
};

static fufft_status dim_plan(int n, int R, int* w, int* p, int* m)
{
   int rad[32];
   const int nrad = n > 1 ? fufft_chain(n, R, rad) : 0;
   if(nrad < 0) return FUFFT_ERR_INVALID_SIZE;
   *p = nrad;
   *m = 0;
   for(int k = 0; k < nrad; k++) {
      int lw = 0;
      while((1 << lw) < rad[k]) lw++;
      w[k] = lw;
      *m += lw;
   }
   return FUFFT_OK;
}

static fufft_status make_perm_plan2(int h, int wd, fufft_layout layout, PermPlan* pl)
{
   const int R = host::layout_radix(layout);
   if(!R) return FUFFT_ERR_INVALID_ARG;
   fufft_status s = dim_plan(wd, R, pl->w, &pl->p, &pl->m);
   if(s != FUFFT_OK) return s;
   s = dim_plan(h, R, pl->wh, &pl->ph, &pl->mh);
   if(s != FUFFT_OK) return s;
   pl->v = host::layout_bperm(layout) ? R : 1;
   pl->T = h * wd / pl->v;
   // transforms beyond one CTA run as a cluster of C CTAs, C = the first radix
   // of the chain; each CTA's block of n/C points is its own register boundary
   if(pl->v > 1 && (long long)h * wd > host::MAX_N_R16 && R == 16) {
      int rad[32];
      const int first = h > 1 ? (fufft_chain(h, R, rad), rad[0]) : (fufft_chain(wd, R, rad), rad[0]);
      pl->blk = (long long)h * wd / first;
      pl->T = (int)(pl->blk / pl->v);
   }
   return FUFFT_OK;
}

static fufft_status make_perm_plan(int n, fufft_layout layout, PermPlan* pl)
{
   return make_perm_plan2(1, n, layout, pl);
}

// destination position i -> natural spectrum index.  chain[r*W + c] =
// spectrum[rev_H(r)*W + rev_W(c)]; bperm[L + k*T] = chain[v*L + k]
__host__ __device__ inline long long perm_src(long long i, const PermPlan& pl)
{
   long long c = i;
   if(pl.v > 1) {
      const long long off = pl.blk > 0 ? (i / pl.blk) * pl.blk : 0, ii = i - off;
      const long long L = ii % pl.T, k = ii / pl.T;
      c = off + pl.v * L + k;
   }
   const long long row = c >> pl.m, col = c & ((1LL << pl.m) - 1);
   return (chain_rev_dev(row, pl.wh, pl.ph, pl.mh) << pl.m) | chain_rev_dev(col, pl.w, pl.p, pl.m);
}

__global__ void filter_permute_kernel(const float2* __restrict__ in, float2* __restrict__ out, int n,
                                      long long total, PermPlan pl)
{
   for(long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
      const long long t = g / n, i = g % n;
      out[g] = in[t * n + perm_src(i, pl)];
   }
}

// ---------------------------------------------------------------------------
// int16 BFP pack / unpack.  Even n <= 8192: one pass (bfp_pack_onepass_kernel
// below).  Otherwise three short launches, so any n works:
//   1) per-transform abs-max into the scale array (atomicMax on the fp32
//      bits, which order like the values for x >= 0);
//   2) quantise with inv = 32767 / max(mx, 1e-30);
//   3) scale = max(mx, 1e-30) / 32767.
// Same operations and roundings as the reference's host quantiser.
// ---------------------------------------------------------------------------
constexpr int BFP_CHUNK = 2048;   // points per block of the abs-max pass

__global__ void bfp_absmax_kernel(const float2* __restrict__ x, unsigned int* __restrict__ mx_bits, int n,
                                  int blocks_per_tr)
{
   const long long t = blockIdx.x / blocks_per_tr;
   const long long lo = (long long)(blockIdx.x % blocks_per_tr) * BFP_CHUNK;
   const long long hi = lo + BFP_CHUNK < n ? lo + BFP_CHUNK : n;
   float m = 0.0f;
   for(long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const float2 v = x[t * n + i];
      m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
   }
   for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
   if((threadIdx.x & 31) == 0) atomicMax(mx_bits + t, __float_as_uint(m));
}

__global__ void bfp_quant_kernel(const float2* __restrict__ x, const float* __restrict__ mxv,
                                 uint32_t* __restrict__ q, long long n, long long total)
{
   for(long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
      const float mx = fmaxf(mxv[g / n], 1e-30f);
      const float inv = 32767.0f / mx;
      q[g] = bfp_quant(x[g], inv);
   }
}

// One pass for transforms that fit one CTA (even n <= 2 * 256 * P): every
// thread holds P pairs of points in registers, the CTA reduces the abs-max,
// then quantises the values it already holds -- 12 bytes per point of HBM
// traffic instead of the 20 of the abs-max pass + quantise pass above, and
// the same operations on the same fp32 values, so the same mantissas and
// scale.
template<int P>
__global__ void __launch_bounds__(256) bfp_pack_onepass_kernel(const float4* __restrict__ x, uint2* __restrict__ q,
                                                               float* __restrict__ scale, int half)
{
   __shared__ float wmax[8];
   const long long t = blockIdx.x;
   const float4* xt = x + t * half;
   float4 v[P];
   float m = 0.0f;
#pragma unroll
   for(int k = 0; k < P; ++k) {
      const int i = threadIdx.x + 256 * k;
      v[k] = i < half ? __ldcs(xt + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
   }
#pragma unroll
   for(int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
   if((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
   __syncthreads();
#pragma unroll
   for(int w = 0; w < 8; ++w) m = fmaxf(m, wmax[w]);
   const float mx = fmaxf(m, 1e-30f);
   const float inv = 32767.0f / mx;
   uint2* qt = q + t * half;
#pragma unroll
   for(int k = 0; k < P; ++k) {
      const int i = threadIdx.x + 256 * k;
      if(i < half)
         __stcs(qt + i, make_uint2(bfp_quant(make_float2(v[k].x, v[k].y), inv),
                                   bfp_quant(make_float2(v[k].z, v[k].w), inv)));
   }
   if(threadIdx.x == 0) scale[t] = mx / 32767.0f;
}

// the one-pass form for even n <= 8192 on aligned buffers; false: not taken
static bool bfp_pack_onepass(const float* x, int16_t* q, float* scale, int n, long long batch, cudaStream_t st)
{
   if(n % 2 || n > 8192 || !host::aligned(x, 16) || !host::aligned(q, 8) || batch > 0x7fffffffLL) return false;
   const int half = n / 2, p = (half + 255) / 256;
   const float4* xv = reinterpret_cast<const float4*>(x);
   uint2* qv = reinterpret_cast<uint2*>(q);
   const unsigned g = (unsigned)batch;
   if(p <= 1) bfp_pack_onepass_kernel<1><<<g, 256, 0, st>>>(xv, qv, scale, half);
   else if(p <= 2) bfp_pack_onepass_kernel<2><<<g, 256, 0, st>>>(xv, qv, scale, half);
   else if(p <= 4) bfp_pack_onepass_kernel<4><<<g, 256, 0, st>>>(xv, qv, scale, half);
   else if(p <= 8) bfp_pack_onepass_kernel<8><<<g, 256, 0, st>>>(xv, qv, scale, half);
   else bfp_pack_onepass_kernel<16><<<g, 256, 0, st>>>(xv, qv, scale, half);
   host::count_launch();
   return true;
}

__global__ void bfp_scale_kernel(float* __restrict__ s, long long batch)
{
   const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
   if(t < batch) s[t] = fmaxf(s[t], 1e-30f) / 32767.0f;
}

__global__ void bfp_unpack_kernel(const uint32_t* __restrict__ q, const float* __restrict__ s,
                                  float2* __restrict__ x, int n, long long total)
{
   for(long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x)
      x[g] = bfp_dequant(q[g], s[g / n]);
}

namespace host {
fufft_status bfp_requantize(const float2* x, float* scale, uint32_t* q, long long n, long long batch, cudaStream_t st)
{
   const long long total = n * batch;
   const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
   bfp_quant_kernel<<<blocks, 256, 0, st>>>(x, scale, q, n, total);
   bfp_scale_kernel<<<(unsigned)((batch + 255) / 256), 256, 0, st>>>(scale, batch);
   count_launch();
   count_launch();
   return check(cudaGetLastError());
}
}  // namespace host

}  // namespace fufft

using namespace fufft;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* fufft_status_string(fufft_status s)
{
   switch(s) {
   case FUFFT_OK: return "ok";
   case FUFFT_ERR_INVALID_SIZE: return "invalid size: n must be a supported power of two";
   case FUFFT_ERR_INVALID_BATCH: return "invalid batch";
   case FUFFT_ERR_MISALIGNED: return "misaligned pointer or stride";
   case FUFFT_ERR_CUDA: return "CUDA error (see fufft_last_cuda_error)";
   case FUFFT_ERR_TIMEOUT: return "a bounded device wait timed out";
   case FUFFT_ERR_PEER_UNAVAILABLE: return "peer device unavailable";
   case FUFFT_ERR_INVALID_ARG: return "invalid argument";
   case FUFFT_ERR_UNSUPPORTED: return "unsupported by this build";
   }
   return "unknown status";
}

const char* fufft_last_cuda_error(void) { return host::t_last_error.c_str(); }

int fufft_max_n(fufft_layout layout)
{
   const int R = host::layout_radix(layout);
   return R == 16 ? host::MAX_N_CLUSTER : host::max_n(R);
}

fufft_status fufft_init(void)
{
   host::DeviceCtx c;
   return host::device_ctx(&c);
}

fufft_status fufft_device_status(uint32_t* status_out, fufft_stream_t stream)
{
   if(!status_out) return FUFFT_ERR_INVALID_ARG;
   host::DeviceCtx c;
   fufft_status s = host::device_ctx(&c);
   if(s != FUFFT_OK) return s;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   unsigned int v = 0;
   s = host::check(cudaMemcpyAsync(&v, c.status, sizeof(v), cudaMemcpyDeviceToHost, st));
   if(s == FUFFT_OK) s = host::check(cudaMemsetAsync(c.status, 0, sizeof(unsigned int), st));
   if(s == FUFFT_OK) s = host::check(cudaStreamSynchronize(st));
   *status_out = v;
   return s;
}

uint64_t fufft_launch_count(void) { return host::g_launches.load(); }

fufft_status fufft_selftest_wait_timeout(uint32_t limit_us, fufft_stream_t stream)
{
   if(limit_us == 0 || limit_us > 1000000) return FUFFT_ERR_INVALID_ARG;
   host::DeviceCtx c;
   fufft_status s = host::device_ctx(&c);
   if(s != FUFFT_OK) return s;
   wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(c.status, limit_us);
   return host::check(cudaGetLastError());
}

int fufft_chain(int n, int radix, int* radices_out)
{
   if(!host::pow2(n) || !host::pow2(radix) || radix < 2 || !radices_out) return -1;
   int m = 0, rb = 0;
   while((1 << m) < n) m++;
   while((1 << rb) < radix) rb++;
   const int nr = m / rb, lead = 1 << (m % rb);
   int p = 0;
   if(lead > 1) radices_out[p++] = lead;
   for(int i = 0; i < nr && p < 32; i++) radices_out[p++] = radix;
   return p;
}

int64_t fufft_chain_rev(int64_t idx, const int* radices, int nrad)
{
   if(!radices || nrad < 0 || nrad > 32) return -1;
   int w[32], m = 0;
   for(int k = 0; k < nrad; k++) {
      int lw = 0;
      while((1 << lw) < radices[k]) lw++;
      w[k] = lw;
      m += lw;
   }
   return chain_rev_dev(idx, w, nrad, m);
}

fufft_status fufft_filter_permute_host(const float* spec_natural, float* out, int n, int batch,
                                       fufft_layout layout)
{
   if(!spec_natural || !out || spec_natural == out) return FUFFT_ERR_INVALID_ARG;
   if(batch < 0) return FUFFT_ERR_INVALID_BATCH;
   if(!host::pow2(n)) return FUFFT_ERR_INVALID_SIZE;
   PermPlan pl;
   fufft_status s = make_perm_plan(n, layout, &pl);
   if(s != FUFFT_OK) return s;
   if(pl.v > 1 && n % pl.v) return FUFFT_ERR_INVALID_SIZE;
   const float2* in = reinterpret_cast<const float2*>(spec_natural);
   float2* o = reinterpret_cast<float2*>(out);
   for(long long i = 0; i < n; i++) {
      const long long src = perm_src(i, pl);
      for(long long t = 0; t < batch; t++) o[t * n + i] = in[t * n + src];
   }
   return FUFFT_OK;
}

fufft_status fufft_filter_permute(const float* spec_natural, float* out, int n, int batch,
                                  fufft_layout layout, fufft_stream_t stream)
{
   if(!spec_natural || !out || spec_natural == out) return FUFFT_ERR_INVALID_ARG;
   if(batch < 0) return FUFFT_ERR_INVALID_BATCH;
   if(!host::pow2(n)) return FUFFT_ERR_INVALID_SIZE;
   if(!host::aligned(spec_natural, 8) || !host::aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   PermPlan pl;
   fufft_status s = make_perm_plan(n, layout, &pl);
   if(s != FUFFT_OK) return s;
   if(pl.v > 1 && n % pl.v) return FUFFT_ERR_INVALID_SIZE;
   if(batch == 0) return FUFFT_OK;
   const long long total = (long long)n * batch;
   const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
   filter_permute_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float2*>(spec_natural), reinterpret_cast<float2*>(out), n, total, pl);
   host::count_launch();
   return host::check(cudaGetLastError());
}

fufft_status fufft_filter_permute2d(const float* spec_natural, float* out, int h, int w, int batch,
                                    fufft_layout layout, int on_host, fufft_stream_t stream)
{
   if(!spec_natural || !out || spec_natural == out) return FUFFT_ERR_INVALID_ARG;
   if(batch < 0) return FUFFT_ERR_INVALID_BATCH;
   if(!host::pow2(h) || !host::pow2(w)) return FUFFT_ERR_INVALID_SIZE;
   PermPlan pl;
   fufft_status s = make_perm_plan2(h, w, layout, &pl);
   if(s != FUFFT_OK) return s;
   const int n = h * w;
   if(pl.v > 1 && n % pl.v) return FUFFT_ERR_INVALID_SIZE;
   if(on_host) {
      const float2* in = reinterpret_cast<const float2*>(spec_natural);
      float2* o = reinterpret_cast<float2*>(out);
      for(long long i = 0; i < n; i++) {
         const long long src = perm_src(i, pl);
         for(long long t = 0; t < batch; t++) o[t * n + i] = in[t * n + src];
      }
      return FUFFT_OK;
   }
   if(!host::aligned(spec_natural, 8) || !host::aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   if(batch == 0) return FUFFT_OK;
   const long long total = (long long)n * batch;
   const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
   filter_permute_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float2*>(spec_natural), reinterpret_cast<float2*>(out), n, total, pl);
   host::count_launch();
   return host::check(cudaGetLastError());
}

fufft_status fufft_bfp_pack(const float* x, int16_t* q, float* scale, int n, int64_t batch,
                            fufft_stream_t stream)
{
   if(!x || !q || !scale) return FUFFT_ERR_INVALID_ARG;
   if(batch < 0) return FUFFT_ERR_INVALID_BATCH;
   if(n <= 0) return FUFFT_ERR_INVALID_SIZE;
   if(!host::aligned(x, 8) || !host::aligned(q, 4) || !host::aligned(scale, 4)) return FUFFT_ERR_MISALIGNED;
   if(batch == 0) return FUFFT_OK;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#ifndef FUFFT_BFP_PACK_ONEPASS
#define FUFFT_BFP_PACK_ONEPASS 1
#endif
   if(FUFFT_BFP_PACK_ONEPASS && bfp_pack_onepass(x, q, scale, n, batch, st)) return host::check(cudaGetLastError());
   fufft_status s = host::check(cudaMemsetAsync(scale, 0, sizeof(float) * batch, st));
   if(s != FUFFT_OK) return s;
   const int bpt = (n + BFP_CHUNK - 1) / BFP_CHUNK;
   bfp_absmax_kernel<<<(unsigned)(bpt * batch), 256, 0, st>>>(reinterpret_cast<const float2*>(x),
                                                            reinterpret_cast<unsigned int*>(scale), n, bpt);
   const long long total = (long long)n * batch;
   const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
   bfp_quant_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float2*>(x), scale,
                                            reinterpret_cast<uint32_t*>(q), n, total);
   bfp_scale_kernel<<<(unsigned)((batch + 255) / 256), 256, 0, st>>>(scale, batch);
   host::count_launch(); host::count_launch(); host::count_launch();
   return host::check(cudaGetLastError());
}

fufft_status fufft_bfp_unpack(const int16_t* q, const float* scale, float* x, int n, int64_t batch,
                              fufft_stream_t stream)
{
   if(!x || !q || !scale) return FUFFT_ERR_INVALID_ARG;
   if(batch < 0) return FUFFT_ERR_INVALID_BATCH;
   if(n <= 0) return FUFFT_ERR_INVALID_SIZE;
   if(!host::aligned(x, 8) || !host::aligned(q, 4) || !host::aligned(scale, 4)) return FUFFT_ERR_MISALIGNED;
   if(batch == 0) return FUFFT_OK;
   const long long total = (long long)n * batch;
   const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
   bfp_unpack_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(q), scale, reinterpret_cast<float2*>(x), n, total);
   host::count_launch();
   return host::check(cudaGetLastError());
}

}  // extern "C"
