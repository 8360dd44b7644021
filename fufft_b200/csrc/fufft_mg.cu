// fufft_mg.cu -- one convolution job over several GPUs from one host thread
// (fufft_conv_multi_gpu).  The reference is single-GPU.  Its transforms are
// independent, so a batch splits across GPUs with no communication.  The one
// case that communicates -- a single signal spread over several GPUs -- reuses
// the fused outer passes of fufft_dist.cu, with the all-to-alls done as NVLink
// peer stores and loads.
//
// Single-signal phases, per rank r on its shard's stream:
//   0. wait for every shard stream's earlier work (a previous job may still
//      be reading the blocks);
//   1. push: rank r's share of the first DIF pass; row k is stored into rank
//      k's block (fufft_dist_pass_push);
//   2. wait for every rank's push, then convolve block r (one kernel, a cluster
//      kernel or the four-step, by the block size);
//   3. wait for every rank's block, then pull: the rows are loaded back from
//      the blocks and the last DIT pass writes the slice (fufft_dist_pass_pull);
//   4. wait for every rank's pull, so that work queued later on any stream may
//      reuse the blocks.
// Each wait is a cudaStreamWaitEvent on events recorded on the other shard
// streams.  The ordering lives in the streams and no kernel spins on another
// rank, so shards may also share a GPU.
#include <algorithm>
#include <mutex>

#include "fufft_internal.cuh"

using namespace fufft::host;

namespace {

constexpr int PHASES = 4;

// Events per shard index and phase.  Each is created on its shard's device,
// and recreated when a later job puts that shard index on another device.
struct MgEvents {
   std::mutex mu;
   int device[FUFFT_MG_MAX_SHARDS];
   cudaEvent_t ev[FUFFT_MG_MAX_SHARDS][PHASES];
   MgEvents()
   {
      for(int i = 0; i < FUFFT_MG_MAX_SHARDS; ++i) {
         device[i] = -1;
         for(int p = 0; p < PHASES; ++p) ev[i][p] = nullptr;
      }
   }
};
MgEvents g_events;

// restores the caller's current device on every return path
struct DeviceGuard {
   int saved = -1;
   DeviceGuard()
   {
      if(cudaGetDevice(&saved) != cudaSuccess) {
         cudaGetLastError();
         saved = -1;
      }
   }
   ~DeviceGuard()
   {
      if(saved >= 0) cudaSetDevice(saved);
   }
};

fufft_status shard_events(int i, int dev)
{
   if(g_events.device[i] == dev) return FUFFT_OK;
   fufft_status s;
   for(int p = 0; p < PHASES; ++p)
      if(g_events.ev[i][p]) {
         // an event is destroyed on the device it was created on
         cudaSetDevice(g_events.device[i]);
         cudaEventDestroy(g_events.ev[i][p]);
         g_events.ev[i][p] = nullptr;
      }
   g_events.device[i] = -1;
   if((s = check(cudaSetDevice(dev))) != FUFFT_OK) return s;
   for(int p = 0; p < PHASES; ++p)
      if((s = check(cudaEventCreateWithFlags(&g_events.ev[i][p], cudaEventDisableTiming))) != FUFFT_OK) return s;
   g_events.device[i] = dev;
   return FUFFT_OK;
}

// every shard stream waits for phase `p` of every other shard stream
fufft_status all_wait(const fufft_mg_desc& d, int p)
{
   fufft_status s;
   for(int i = 0; i < d.n_shards; ++i) {
      const fufft_mg_shard& sh = d.shards[i];
      if((s = check(cudaSetDevice(sh.device))) != FUFFT_OK) return s;
      if((s = check(cudaEventRecord(g_events.ev[i][p], reinterpret_cast<cudaStream_t>(sh.stream)))) != FUFFT_OK)
         return s;
   }
   for(int i = 0; i < d.n_shards; ++i) {
      const fufft_mg_shard& sh = d.shards[i];
      if((s = check(cudaSetDevice(sh.device))) != FUFFT_OK) return s;
      for(int j = 0; j < d.n_shards; ++j) {
         if(j == i) continue;
         s = check(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(sh.stream), g_events.ev[j][p], 0));
         if(s != FUFFT_OK) return s;
      }
   }
   return FUFFT_OK;
}

// peer access from every shard's GPU to every other distinct GPU of the job
fufft_status enable_peers(const fufft_mg_desc& d)
{
   static std::mutex mu;
   static uint64_t enabled[64] = {};   // bit j of enabled[i]: GPU i maps GPU j
   std::lock_guard<std::mutex> lock(mu);
   for(int i = 0; i < d.n_shards; ++i)
      for(int j = 0; j < d.n_shards; ++j) {
         const int a = d.shards[i].device, b = d.shards[j].device;
         const bool cached = a < 64 && b < 64;
         if(a == b || (cached && ((enabled[a] >> b) & 1))) continue;
         int can = 0;
         fufft_status s = check(cudaDeviceCanAccessPeer(&can, a, b));
         if(s != FUFFT_OK) return s;
         if(!can) return FUFFT_ERR_PEER_UNAVAILABLE;
         if((s = check(cudaSetDevice(a))) != FUFFT_OK) return s;
         const cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
         if(e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
         else if(e != cudaSuccess) return cuda_fail(e);
         if(cached) enabled[a] |= 1ull << b;
      }
   return FUFFT_OK;
}

struct BlockPlan {
   int64_t n_blk, cols;
   bool one_kernel;   // the block fits fufft_conv_c2c_f32 with the radix-16 chain
   int r_out, mid;    // else its four-step plan
};

fufft_status block_plan(int64_t n, int world, BlockPlan* p)
{
   if(world != 2 && world != 4 && world != 8) return FUFFT_ERR_UNSUPPORTED;
   if(!pow2(n) || n < (int64_t)world * world * 256 || n > (1LL << 36)) return FUFFT_ERR_INVALID_SIZE;
   p->n_blk = n / world;
   p->cols = p->n_blk / world;
   p->one_kernel = p->n_blk <= fufft_max_n(FUFFT_LAYOUT_R16);
   p->r_out = 0;
   p->mid = (int)std::min<int64_t>(p->n_blk, 1 << 30);
   if(!p->one_kernel) return fufft_large_plan(p->n_blk, FUFFT_LAYOUT_R16, &p->r_out, &p->mid);
   return FUFFT_OK;
}

fufft_status validate(const fufft_mg_desc* d, BlockPlan* plan)
{
   if(!d || !d->shards || d->n_shards < 1 || d->n_shards > FUFFT_MG_MAX_SHARDS) return FUFFT_ERR_INVALID_ARG;
   if(d->mode < FUFFT_MG_BATCH || d->mode > FUFFT_MG_SINGLE_SIGNAL) return FUFFT_ERR_INVALID_ARG;
   if(d->mid < FUFFT_MID_NONE || d->mid > FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   for(int i = 0; i < d->n_shards; ++i)
      if(d->shards[i].device < 0) return FUFFT_ERR_INVALID_ARG;
   if(d->mode != FUFFT_MG_SINGLE_SIGNAL) {
      if(!layout_radix(d->layout)) return FUFFT_ERR_INVALID_ARG;
      if(!pow2(d->n) || d->n > fufft_max_n(d->layout)) return FUFFT_ERR_INVALID_SIZE;
      for(int i = 0; i < d->n_shards; ++i)
         if(d->shards[i].batch < 0) return FUFFT_ERR_INVALID_BATCH;
      return FUFFT_OK;
   }
   if(d->n_shards != 2 && d->n_shards != 4 && d->n_shards != 8) return FUFFT_ERR_UNSUPPORTED;
   fufft_status s = block_plan(d->n, d->n_shards, plan);
   if(s != FUFFT_OK) return s;
   for(int i = 0; i < d->n_shards; ++i) {
      const fufft_mg_shard& sh = d->shards[i];
      if(!sh.out || !sh.workspace || (sh.a && sh.a != sh.out)) return FUFFT_ERR_INVALID_ARG;
      if(d->mid != FUFFT_MID_NONE && !sh.b) return FUFFT_ERR_INVALID_ARG;
      if(sh.workspace_bytes < (size_t)plan->n_blk * 8) return FUFFT_ERR_INVALID_ARG;
      if(!aligned(sh.out, 16) || !aligned(sh.workspace, 16) || (sh.b && !aligned(sh.b, 16)))
         return FUFFT_ERR_MISALIGNED;
   }
   return FUFFT_OK;
}

fufft_status run_batch(const fufft_mg_desc& d)
{
   for(int i = 0; i < d.n_shards; ++i) {
      const fufft_mg_shard& sh = d.shards[i];
      if(sh.batch == 0) continue;
      fufft_status s = check(cudaSetDevice(sh.device));
      if(s != FUFFT_OK) return s;
      if(d.mode == FUFFT_MG_BATCH)
         s = fufft_conv_c2c_f32(sh.a, sh.b, sh.out, (int)d.n, sh.batch, d.layout, d.mid, d.filter_stride, sh.stream);
      else
         s = fufft_conv_c2c_f32_host(sh.a, sh.b, sh.out, (int)d.n, sh.batch, d.layout, d.mid, d.filter_stride,
                                     sh.workspace, sh.workspace_bytes, sh.stream);
      if(s != FUFFT_OK) return s;
   }
   return FUFFT_OK;
}

fufft_status run_single(const fufft_mg_desc& d, const BlockPlan& plan)
{
   fufft_status s;
   if((s = enable_peers(d)) != FUFFT_OK) return s;
   std::lock_guard<std::mutex> lock(g_events.mu);
   for(int i = 0; i < d.n_shards; ++i)
      if((s = shard_events(i, d.shards[i].device)) != FUFFT_OK) return s;
   const int world = d.n_shards;
   uint64_t blocks[8];
   for(int i = 0; i < world; ++i) blocks[i] = reinterpret_cast<uint64_t>(d.shards[i].workspace);

   if((s = all_wait(d, 0)) != FUFFT_OK) return s;
   for(int r = 0; r < world; ++r) {
      const fufft_mg_shard& sh = d.shards[r];
      if((s = check(cudaSetDevice(sh.device))) != FUFFT_OK) return s;
      if((s = fufft_dist_pass_push(sh.out, blocks, world, r, plan.cols, d.n, sh.stream)) != FUFFT_OK) return s;
   }
   if((s = all_wait(d, 1)) != FUFFT_OK) return s;
   for(int r = 0; r < world; ++r) {
      const fufft_mg_shard& sh = d.shards[r];
      if((s = check(cudaSetDevice(sh.device))) != FUFFT_OK) return s;
      float* blk = static_cast<float*>(sh.workspace);
      if(plan.one_kernel)
         s = fufft_conv_c2c_f32(blk, sh.b, blk, (int)plan.n_blk, 1, FUFFT_LAYOUT_R16, d.mid, plan.n_blk, sh.stream);
      else
         s = fufft_conv_large_f32(blk, sh.b, plan.n_blk, 1, plan.r_out, plan.mid, FUFFT_LAYOUT_R16, d.mid,
                                  sh.stream);
      if(s != FUFFT_OK) return s;
   }
   if((s = all_wait(d, 2)) != FUFFT_OK) return s;
   for(int r = 0; r < world; ++r) {
      const fufft_mg_shard& sh = d.shards[r];
      if((s = check(cudaSetDevice(sh.device))) != FUFFT_OK) return s;
      if((s = fufft_dist_pass_pull(sh.out, blocks, world, r, plan.cols, d.n, sh.stream)) != FUFFT_OK) return s;
   }
   return all_wait(d, 3);
}

}  // namespace

extern "C" {

fufft_status fufft_conv_multi_gpu(const fufft_mg_desc* desc)
{
   BlockPlan plan{};
   fufft_status s = validate(desc, &plan);
   if(s != FUFFT_OK) return s;
   int count = 0;
   if((s = check(cudaGetDeviceCount(&count))) != FUFFT_OK) return s;
   for(int i = 0; i < desc->n_shards; ++i)
      if(desc->shards[i].device >= count) return FUFFT_ERR_INVALID_ARG;
   DeviceGuard guard;
   return desc->mode == FUFFT_MG_SINGLE_SIGNAL ? run_single(*desc, plan) : run_batch(*desc);
}

int fufft_mg_chain(int64_t n, int world, int* radices_out)
{
   BlockPlan plan{};
   if(!radices_out || block_plan(n, world, &plan) != FUFFT_OK) return -1;
   int len = 0;
   radices_out[len++] = world;
   if(plan.one_kernel) {
      const int k = fufft_chain((int)plan.n_blk, 16, radices_out + len);
      return k < 0 ? -1 : len + k;
   }
   for(int64_t q = plan.n_blk / plan.mid; q > 1; q /= plan.r_out) radices_out[len++] = plan.r_out;
   const int k = fufft_chain(plan.mid, 16, radices_out + len);
   return k < 0 ? -1 : len + k;
}

}  // extern "C"
