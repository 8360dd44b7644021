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
//     loads the library, held until the process exits; requests needing more
//     (8 * n * batch bytes) are rejected with FUFFT_ERR_INVALID_SIZE;
//   * all calls on a device share the one array, so calls that may overlap on
//     the GPU (different streams without ordering between them) race on it --
//     serialise them on one stream;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and remembers it; make
//     that first call before any stream capture;
//   * nothing in the array needs to start at zero: every workspace element is
//     written by the first outer pass before anything reads it.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "fufft_internal.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FUFFT_NOALLOC_SCRATCH_BYTES];

struct ScratchSlot {
   std::once_flag once;
   void* ptr = nullptr;
   cudaError_t err = cudaSuccess;
};
constexpr int MAX_DEVICES = 64;
ScratchSlot g_slots[MAX_DEVICES];

// the host-side name of the array is not a device address: look the address
// up once per device, with that device current
fufft_status scratch_of_current_device(void** out)
{
   int dev = 0;
   const cudaError_t e = cudaGetDevice(&dev);
   if(e != cudaSuccess) return fufft::host::cuda_fail(e);
   if(dev < 0 || dev >= MAX_DEVICES) return FUFFT_ERR_UNSUPPORTED;
   ScratchSlot& s = g_slots[dev];
   std::call_once(s.once, [&] { s.err = cudaGetSymbolAddress(&s.ptr, g_noalloc_scratch); });
   if(s.err != cudaSuccess) return fufft::host::cuda_fail(s.err);
   *out = s.ptr;
   return FUFFT_OK;
}

}  // namespace

extern "C" fufft_status fufft_conv_large_bfp_noalloc(const int16_t* aq, const float* a_scale, const int16_t* bq,
                                                     const float* b_scale, int16_t* oq, float* o_scale, int64_t n,
                                                     int64_t batch, int r_out, int mid, fufft_layout layout,
                                                     fufft_midop mid_op, fufft_stream_t stream)
{
   if(n <= 0 || batch < 0) return batch < 0 ? FUFFT_ERR_INVALID_BATCH : FUFFT_ERR_INVALID_SIZE;
   if(fufft_conv_large_bfp_workspace(n, batch) > FUFFT_NOALLOC_SCRATCH_BYTES) return FUFFT_ERR_INVALID_SIZE;
   void* scratch = nullptr;
   const fufft_status s = scratch_of_current_device(&scratch);
   if(s != FUFFT_OK) return s;
   return fufft_conv_large_bfp(aq, a_scale, bq, b_scale, oq, o_scale, n, batch, r_out, mid, layout, mid_op, scratch,
                               FUFFT_NOALLOC_SCRATCH_BYTES, stream);
}
