// fufft_host.cu -- fused convolution of data that lives in HOST memory.
//
// The reference's kernels take device pointers and leave the transfers to the
// caller (bench_fufft.cu:183-186 copies the whole batch in, :227 copies it
// out after the launches, one after the other).  Over PCIe that serial form
// is bound by the sum of both transfer directions.  fufft_conv_c2c_f32_host
// splits the batch
// into chunks of about 32 MiB and runs a three-stage pipeline on private
// streams of the device:
//   h2d stream:   signal (and filter) chunk i -> device slot i % 3
//   compute:      fused convolution of slot i in place (fufft_conv_c2c_f32)
//   d2h stream:   result chunk i -> host
// so the host->device and device->host directions of the link run at the
// same time, and the kernels hide under the copies.  A slot is reused only
// after its previous result has left (event `down`), the pipeline starts
// after the work already queued on the caller's stream and the caller's
// stream waits for its end, so the call behaves like any other asynchronous
// call on `stream`.  Device memory comes from the caller (workspace), none is
// allocated here.  Host buffers should be pinned (cudaHostAlloc /
// cudaHostRegister) for the copies to overlap.
#include <mutex>

#include "fufft_internal.cuh"

using namespace fufft;
using namespace fufft::host;

namespace {

constexpr int SLOTS = 3;
constexpr size_t CHUNK_BYTES = 32u << 20;
constexpr size_t ALIGN = 256;

size_t round_up(size_t v) { return (v + ALIGN - 1) / ALIGN * ALIGN; }

// transforms per chunk: about CHUNK_BYTES of signal, at least one transform
long long chunk_transforms(int n, long long batch)
{
   long long ct = (long long)(CHUNK_BYTES / ((size_t)n * sizeof(float2)));
   if(ct < 1) ct = 1;
   return ct < batch ? ct : batch;
}

#ifndef FUFFT_HOST_TWO_UPLOADS
#define FUFFT_HOST_TWO_UPLOADS 1
#endif
struct Pipe {
   std::mutex mu;
   bool ready = false;
   // h2d2 carries the filters so two copy engines share the upload direction
   cudaStream_t h2d = nullptr, h2d2 = nullptr, comp = nullptr, d2h = nullptr;
   cudaEvent_t start = nullptr, up[SLOTS] = {}, up2[SLOTS] = {}, done[SLOTS] = {}, down[SLOTS] = {};
};
constexpr int MAX_DEVICES = 64;
Pipe g_pipe[MAX_DEVICES];

fufft_status pipe_init(Pipe& p)
{
   fufft_status s;
   for(cudaStream_t* st : {&p.h2d, &p.h2d2, &p.comp, &p.d2h})
      if((s = check(cudaStreamCreateWithFlags(st, cudaStreamNonBlocking))) != FUFFT_OK) return s;
   if((s = check(cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming))) != FUFFT_OK) return s;
   for(int i = 0; i < SLOTS; ++i)
      for(cudaEvent_t* e : {&p.up[i], &p.up2[i], &p.done[i], &p.down[i]})
         if((s = check(cudaEventCreateWithFlags(e, cudaEventDisableTiming))) != FUFFT_OK) return s;
   p.ready = true;
   return FUFFT_OK;
}

struct Plan {
   long long ct;        // transforms per chunk
   size_t sig_bytes;    // one slot's signal / result region
   size_t flt_bytes;    // one slot's filter region (per-transform filters)
   size_t slot_bytes;
   size_t shared_bytes; // the single filter of filter_stride 0
   size_t total;
};

Plan make_plan(int n, long long batch, long long filter_stride)
{
   Plan p{};
   p.ct = chunk_transforms(n, batch);
   p.sig_bytes = round_up((size_t)p.ct * n * sizeof(float2));
   p.flt_bytes = filter_stride == n ? p.sig_bytes : 0;
   p.slot_bytes = p.sig_bytes + p.flt_bytes;
   p.shared_bytes = filter_stride == 0 ? round_up((size_t)n * sizeof(float2)) : 0;
   p.total = SLOTS * p.slot_bytes + p.shared_bytes;
   return p;
}

}  // namespace

extern "C" {

size_t fufft_conv_host_workspace(int n, int64_t batch, int64_t filter_stride)
{
   if(n <= 0 || batch <= 0) return 0;
   return make_plan(n, batch, filter_stride).total;
}

fufft_status fufft_conv_c2c_f32_host(const float* a, const float* b, float* out, int n, int64_t batch,
                                     fufft_layout layout, fufft_midop mid, int64_t filter_stride, void* workspace,
                                     size_t workspace_bytes, fufft_stream_t stream)
{
   if(!layout_radix(layout)) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(n) || n > fufft_max_n(layout)) return FUFFT_ERR_INVALID_SIZE;
   if(batch < 0 || batch > (int64_t)1 << 40) return FUFFT_ERR_INVALID_BATCH;
   if(mid < FUFFT_MID_NONE || mid > FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   const bool has_filter = mid != FUFFT_MID_NONE;
   if(has_filter && (!b || (filter_stride != 0 && filter_stride != n))) return FUFFT_ERR_INVALID_ARG;
   if(!has_filter) filter_stride = n;   // no filter region
   if(batch == 0) return FUFFT_OK;
   if(!a || !out || !workspace) return FUFFT_ERR_INVALID_ARG;
   const Plan plan = make_plan(n, batch, has_filter ? filter_stride : -1);
   if(workspace_bytes < plan.total) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(workspace, ALIGN)) return FUFFT_ERR_MISALIGNED;

   DeviceCtx ctx;
   fufft_status s = device_ctx(&ctx);
   if(s != FUFFT_OK) return s;
   Pipe& p = g_pipe[ctx.device];
   std::lock_guard<std::mutex> lock(p.mu);
   if(!p.ready && (s = pipe_init(p)) != FUFFT_OK) return s;

   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   unsigned char* ws = static_cast<unsigned char*>(workspace);
   const size_t pt = (size_t)n * sizeof(float2);   // bytes per transform
   const float* bdev = nullptr;
   // the pipeline starts after the work already queued on the caller's stream
   if((s = check(cudaEventRecord(p.start, st))) != FUFFT_OK) return s;
   for(cudaStream_t q : {p.h2d, p.h2d2, p.comp, p.d2h})
      if((s = check(cudaStreamWaitEvent(q, p.start, 0))) != FUFFT_OK) return s;
   const bool two = FUFFT_HOST_TWO_UPLOADS && has_filter && filter_stride == n;
   cudaStream_t fup = two ? p.h2d2 : p.h2d;
   if(has_filter && filter_stride == 0) {
      float* shared = reinterpret_cast<float*>(ws + SLOTS * plan.slot_bytes);
      if((s = check(cudaMemcpyAsync(shared, b, pt, cudaMemcpyHostToDevice, p.h2d))) != FUFFT_OK) return s;
      bdev = shared;
   }
   const long long nchunks = (batch + plan.ct - 1) / plan.ct;
   for(long long i = 0; i < nchunks; ++i) {
      const int slot = (int)(i % SLOTS);
      const long long t0 = i * plan.ct;
      const long long cnt = batch - t0 < plan.ct ? batch - t0 : plan.ct;
      float* sig = reinterpret_cast<float*>(ws + slot * plan.slot_bytes);
      float* flt = reinterpret_cast<float*>(ws + slot * plan.slot_bytes + plan.sig_bytes);
      const size_t bytes = (size_t)cnt * pt;
      // upload: the slot is free once its previous result has left
      if(i >= SLOTS && (s = check(cudaStreamWaitEvent(p.h2d, p.down[slot], 0))) != FUFFT_OK) return s;
      if(two && i >= SLOTS && (s = check(cudaStreamWaitEvent(fup, p.down[slot], 0))) != FUFFT_OK) return s;
      if((s = check(cudaMemcpyAsync(sig, a + (size_t)t0 * 2 * n, bytes, cudaMemcpyHostToDevice, p.h2d))) != FUFFT_OK)
         return s;
      if(has_filter && filter_stride == n) {
         if((s = check(cudaMemcpyAsync(flt, b + (size_t)t0 * 2 * n, bytes, cudaMemcpyHostToDevice, fup))) !=
            FUFFT_OK)
            return s;
      }
      if((s = check(cudaEventRecord(p.up[slot], p.h2d))) != FUFFT_OK) return s;
      if(two && (s = check(cudaEventRecord(p.up2[slot], fup))) != FUFFT_OK) return s;
      // convolve in place
      if((s = check(cudaStreamWaitEvent(p.comp, p.up[slot], 0))) != FUFFT_OK) return s;
      if(two && (s = check(cudaStreamWaitEvent(p.comp, p.up2[slot], 0))) != FUFFT_OK) return s;
      s = fufft_conv_c2c_f32(sig, has_filter ? (filter_stride == n ? flt : bdev) : nullptr, sig, n, cnt, layout, mid,
                             has_filter ? filter_stride : n, reinterpret_cast<fufft_stream_t>(p.comp));
      if(s != FUFFT_OK) return s;
      if((s = check(cudaEventRecord(p.done[slot], p.comp))) != FUFFT_OK) return s;
      // download
      if((s = check(cudaStreamWaitEvent(p.d2h, p.done[slot], 0))) != FUFFT_OK) return s;
      if((s = check(cudaMemcpyAsync(out + (size_t)t0 * 2 * n, sig, bytes, cudaMemcpyDeviceToHost, p.d2h))) !=
         FUFFT_OK)
         return s;
      if((s = check(cudaEventRecord(p.down[slot], p.d2h))) != FUFFT_OK) return s;
   }
   // the caller's stream continues after the last download (the d2h stream is in order)
   return check(cudaStreamWaitEvent(st, p.down[(nchunks - 1) % SLOTS], 0));
}

}  // extern "C"
