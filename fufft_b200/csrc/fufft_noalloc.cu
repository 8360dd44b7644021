// fufft_noalloc.cu -- the int16-BFP four-step convolution for callers that
// cannot allocate device memory when they call the library.
//
// fufft_conv_large_bfp needs an fp32 workspace of 8 * n * batch bytes that the
// caller passes in.  Some callers have no way to provide one at call time:
// a host whose device memory is entirely reserved by its own pool allocator
// (an extra cudaMalloc would fail, or fragment memory the pool assumes it
// owns), or a latency-critical loop in which an allocation -- which may
// synchronise the whole device -- is not acceptable.  For them this file
// holds a fixed scratch area in the library's own device memory, reserved
// when the library is loaded, and an entry point that uses it instead.
//
// Limits and behaviour:
//   * the scratch is FUFFT_NOALLOC_SCRATCH_BYTES (16 MiB) on every GPU that
//     loads the library, held until the process exits; every request whose
//     8 * n * batch bytes exceed it is rejected with FUFFT_ERR_INVALID_SIZE,
//     also the one-outer-level radix-16 plans that run as one cluster kernel
//     without touching the scratch (the limit depends on the sizes only);
//   * arguments are checked in the same order, with the same status codes,
//     as fufft_conv_large_bfp; the scratch limit comes after those checks;
//   * all calls on a device share the one array, so calls that may overlap on
//     the GPU (different streams without ordering between them) race on it --
//     serialise them on one stream;
//   * the first successful call on each device looks up the array's device
//     address (cudaGetSymbolAddress, with that device current) and remembers
//     it; make that first call before any stream capture.  A lookup that
//     fails is not remembered: the next call tries again.  The remembered
//     address belongs to the device's current context; after cudaDeviceReset
//     the library must be reloaded before this entry point is used again;
//   * the array keeps the previous call's contents, and nothing in it needs
//     to start at zero: the first outer pass writes every workspace element
//     before anything reads it (the per-transform abs-max that must start at
//     zero lives in the caller's o_scale, cleared on the stream).
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "fufft_internal.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FUFFT_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[MAX_DEVICES] = {};   // device address per device, once looked up

// the host-side name of the array is not a device address: look the address
// up with the device current, and remember it only once the lookup succeeded
fufft_status scratch_of_current_device(void** out)
{
   int dev = 0;
   const cudaError_t e = cudaGetDevice(&dev);
   if(e != cudaSuccess) return fufft::host::cuda_fail(e);
   if(dev < 0 || dev >= MAX_DEVICES) return FUFFT_ERR_UNSUPPORTED;
   std::lock_guard<std::mutex> lock(g_scratch_mutex);
   if(!g_scratch_ptr[dev]) {
      void* p = nullptr;
      const cudaError_t le = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if(le != cudaSuccess) return fufft::host::cuda_fail(le);
      if(!p) return FUFFT_ERR_CUDA;
      g_scratch_ptr[dev] = p;
   }
   *out = g_scratch_ptr[dev];
   return FUFFT_OK;
}

}  // namespace

extern "C" fufft_status fufft_conv_large_bfp_noalloc(const int16_t* aq, const float* a_scale, const int16_t* bq,
                                                     const float* b_scale, int16_t* oq, float* o_scale, int64_t n,
                                                     int64_t batch, int r_out, int mid, fufft_layout layout,
                                                     fufft_midop mid_op, fufft_stream_t stream)
{
   int lout = 0;
   bool nothing = false;
   fufft_status s = fufft::host::validate_large_bfp(aq, a_scale, bq, b_scale, oq, o_scale, n, batch, r_out, mid,
                                                    layout, mid_op, false, nullptr, 0, &lout, &nothing);
   if(s != FUFFT_OK || nothing) return s;
   if(fufft_conv_large_bfp_workspace(n, batch) > FUFFT_NOALLOC_SCRATCH_BYTES) return FUFFT_ERR_INVALID_SIZE;
   void* scratch = nullptr;
   if((s = scratch_of_current_device(&scratch)) != FUFFT_OK) return s;
   return fufft_conv_large_bfp(aq, a_scale, bq, b_scale, oq, o_scale, n, batch, r_out, mid, layout, mid_op, scratch,
                               FUFFT_NOALLOC_SCRATCH_BYTES, stream);
}
