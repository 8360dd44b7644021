/*
 * fufft_b200.h -- C ABI of the B200-native fused FFT-convolution library.
 *
 * The reference (weiwang217/FuFFT) ships header-only CUDA templates that a
 * caller launches itself (fufft.cuh); this library replaces them with plain
 * C entry points: raw pointers and sizes, no C++ or torch types, one
 * cudaStream_t-compatible stream handle, a status code instead of exit().
 * Each entry point below names the reference interface it replaces.
 *
 * Common rules
 *   - Data pointers are DEVICE pointers owned by the caller, except where a
 *     function says "host".  Calls are asynchronous on `stream` (NULL = the
 *     legacy default stream) and keep no per-call state.
 *   - Complex data are interleaved fp32 pairs (re, im) = float2.  int16
 *     block-floating-point (BFP) data are packed (re, im) int16 pairs (short2,
 *     4 bytes per point) plus one fp32 scale per transform: value = q * scale.
 *   - A transform of n points is stored contiguously; `batch` transforms
 *     follow each other (transform t starts at element t*n).
 *   - Filter spectra already carry the 1/n normalisation (the reference's
 *     convention, bench_fufft.cu:156-165) and are stored in one of the
 *     fufft_layout orders below.  filter_stride is the element distance
 *     between the filters of consecutive transforms: n for one filter per
 *     transform, 0 for a single filter shared by the whole batch.
 *   - n must be a power of two within the range the layout supports
 *     (fufft_max_n()); batch >= 0; signal/result pointers 8-byte aligned,
 *     filter pointers 16-byte aligned.
 *   - The first call on a device builds that device's twiddle tables
 *     (a short kernel plus a synchronize); call fufft_init() first if the
 *     stream might be under graph capture.
 *   - Thread-safe across host threads, streams and devices.
 */
#ifndef FUFFT_B200_H
#define FUFFT_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#include <stddef.h>
#include <stdint.h>

typedef struct CUstream_st* fufft_stream_t; /* same type as cudaStream_t */

typedef enum fufft_status {
   FUFFT_OK = 0,
   FUFFT_ERR_INVALID_SIZE = 1,     /* n not a supported power of two */
   FUFFT_ERR_INVALID_BATCH = 2,    /* batch < 0 */
   FUFFT_ERR_MISALIGNED = 3,       /* a pointer or stride breaks the alignment rule */
   FUFFT_ERR_CUDA = 4,             /* a CUDA runtime call failed (fufft_last_cuda_error) */
   FUFFT_ERR_TIMEOUT = 5,          /* a bounded device wait gave up (fufft_device_status) */
   FUFFT_ERR_PEER_UNAVAILABLE = 6, /* multi-GPU: a peer device cannot be reached */
   FUFFT_ERR_INVALID_ARG = 7,      /* null pointer, bad enum value, bad stride */
   FUFFT_ERR_UNSUPPORTED = 8       /* valid request this build does not implement */
} fufft_status;

/* Mid-operation between the forward and the inverse transform; the
 * reference's policy structs MidNothing / MidMultiply / MidConjMultiply
 * (fufft.cuh:625-650). */
typedef enum fufft_midop {
   FUFFT_MID_NONE = 0,          /* round trip: out = n * a */
   FUFFT_MID_MULTIPLY = 1,      /* convolution: spectrum * filter */
   FUFFT_MID_CONJ_MULTIPLY = 2  /* correlation: spectrum * conj(filter) */
} fufft_midop;

/* Filter-spectrum orders.  "Chain order" is the order a DIF transform leaves
 * its spectrum in: bit-group reversal over the radix widths in pass order
 * (verify_kernel.cpp:145-156 mixedrev, :946-956 mixedrev16).
 *   R8 / R16        chain order of the radix-8 / radix-16 chain, linear:
 *                   filter[i] = spectrum[rev(i)] -- the layout taken by the
 *                   reference's fufft_pipeline_ip / fufft_pipeline_v16
 *   R8_BPERM /      the register-boundary layout of fufft_pipeline_fused /
 *   R16_BPERM       fufft_pipeline_v16f: bperm[L + k*T] = chain[V*L + k],
 *                   T = n/V, V = 8 / 16 (verify_kernel.cpp:1339-1344, :1382-1387)
 *   NATURAL         natural frequency order (input to fufft_filter_permute)
 * The BPERM layouts let the library prefetch the filter with one TMA bulk
 * copy and are the fastest. */
typedef enum fufft_layout {
   FUFFT_LAYOUT_R8 = 0,
   FUFFT_LAYOUT_R8_BPERM = 1,
   FUFFT_LAYOUT_R16 = 2,
   FUFFT_LAYOUT_R16_BPERM = 3,
   FUFFT_LAYOUT_NATURAL = 4
} fufft_layout;

/* ---- library ------------------------------------------------------------ */
const char* fufft_status_string(fufft_status s);
/* text of the last CUDA error seen by this host thread ("" if none) */
const char* fufft_last_cuda_error(void);
/* largest one-kernel n for a layout (R8*: 4096; R16*: 65536, above 8192 as a
 * thread-block cluster of n/4096 CTAs exchanging through distributed shared memory) */
int fufft_max_n(fufft_layout layout);
/* build the current device's twiddle tables now (otherwise done on first use) */
fufft_status fufft_init(void);
/* read and clear the device status word of the current device: bit 0 = a
 * bounded TMA wait timed out.  Synchronises `stream`. */
fufft_status fufft_device_status(uint32_t* status_out, fufft_stream_t stream);
/* number of fused-kernel launches this process has issued (all threads) */
uint64_t fufft_launch_count(void);
/* self-test of the bounded device waits: one thread waits limit_us
 * microseconds (1 .. 1e6) on an mbarrier that nothing completes, gives up and
 * sets bit 0 of the device status word, as any library kernel whose TMA copy
 * or peer data never arrived would; the context stays usable.  No reference
 * counterpart (the reference's kernels have no bounded waits). */
fufft_status fufft_selftest_wait_timeout(uint32_t limit_us, fufft_stream_t stream);

/* ---- index maps (host) -------------------------------------------------- */
/* radix chain of a one-kernel transform: [lead, R, ..., R]; returns its
 * length (<= 32) or -1.  Replaces factorise/factorise16 (verify_kernel.cpp:126-139). */
int fufft_chain(int n, int radix, int* radices_out);
/* chain-reversed index (verify_kernel.cpp:460-477 chain_rev) */
int64_t fufft_chain_rev(int64_t idx, const int* radices, int nrad);

/* ---- filter preparation -------------------------------------------------
 * Natural-order spectrum -> a kernel layout, per transform.  Replaces the
 * host loops of bench_fufft.cu:166-170 (mixedrev_host) and
 * verify_kernel.cpp:1339-1344 / :1382-1387 (bperm).
 * _host: host pointers; the other form: device pointers, async on stream.
 * in != out. */
fufft_status fufft_filter_permute_host(const float* spec_natural, float* out, int n, int batch,
                                       fufft_layout layout);
fufft_status fufft_filter_permute(const float* spec_natural, float* out, int n, int batch,
                                  fufft_layout layout, fufft_stream_t stream);

/* Filter taps (natural order, complex, one row of n per filter) -> the
 * filter spectrum with 1/n folded in, in `layout` (R8 / R16 / *_BPERM),
 * one kernel on the device, n <= fufft_max_n for one CTA (4096 radix 8,
 * 8192 radix 16).  Replaces the host-side preparation around the
 * reference's kernels: spectrum of the taps, 1/n folded in
 * (bench_fufft.cu:156-165), mixedrev permutation (bench_fufft.cu:166-170). */
fufft_status fufft_filter_from_taps_f32(const float* taps, float* out, int n, int64_t batch, fufft_layout layout,
                                       fufft_stream_t stream);

/* 2-D: slot (r, c) of the chain order holds spectrum (rev_H(r), rev_W(c)),
 * each dimension reversed over its own chain ([lead, R, ...]; radix 8 on
 * power-of-8 sides reproduces the reference's rev8 map, verify_kernel.cpp:738-748);
 * the BPERM layouts then apply the register-boundary order to the flattened
 * index.  on_host != 0: host pointers, synchronous; else device, async. */
fufft_status fufft_filter_permute2d(const float* spec_natural, float* out, int h, int w, int batch,
                                    fufft_layout layout, int on_host, fufft_stream_t stream);

/* ---- fused fp32 convolution ---------------------------------------------
 * out = IDFT(DFT(a) . mid(filter)) for each transform, one kernel launch,
 * three HBM streams (signal, filter, result).  a == out is allowed.
 * Replaces fufft_pipeline_ip (fufft.cuh:1757-1772, layout R8),
 * fufft_pipeline_fused (:1774-1791, R8_BPERM), fufft_pipeline_v16 / _r16
 * (:1518-1534, :1736-1755, R16) and fufft_pipeline_v16f (:1499-1516,
 * R16_BPERM), with any mid-op on every layout.  b may be NULL for
 * FUFFT_MID_NONE. */
fufft_status fufft_conv_c2c_f32(const float* a, const float* b, float* out, int n, int64_t batch,
                                fufft_layout layout, fufft_midop mid, int64_t filter_stride,
                                fufft_stream_t stream);

/* ---- fused fp32 convolution of HOST data --------------------------------
 * The same convolution for a, b, out in host memory (pinned for overlap):
 * the batch goes through the device in ~32 MiB chunks, uploads, kernels and
 * downloads of consecutive chunks overlapping on private streams; ordered
 * after the work queued on `stream`, and `stream` waits for its end.
 * filter_stride must be n or 0.  `workspace` is device memory of at least
 * fufft_conv_host_workspace(n, batch, filter_stride) bytes, 256-byte
 * aligned, not used by anything else until the call's work has finished.
 * No reference counterpart: the reference's caller copies the batch in and
 * out around the launches (bench_fufft.cu:183-186, :227). */
size_t fufft_conv_host_workspace(int n, int64_t batch, int64_t filter_stride);
fufft_status fufft_conv_c2c_f32_host(const float* a, const float* b, float* out, int n, int64_t batch,
                                     fufft_layout layout, fufft_midop mid, int64_t filter_stride, void* workspace,
                                     size_t workspace_bytes, fufft_stream_t stream);

/* ---- fused 2-D convolution ----------------------------------------------
 * Row-major h x w images: 2-D DFT (columns then rows), mid-op against the
 * 2-D filter spectrum (fufft_filter_permute2d order), inverse, one kernel
 * launch per batch.  Replaces fufft_conv2d<H, W, CPB> (fufft.cuh:1209-1258,
 * H, W powers of 8, H*W <= 4096, layout R8).  Here h, w are powers of two
 * with w >= 8 (R8) / 16 (R16) and h*w <= 4096 (R8) / 8192 (R16) per CTA;
 * filter_stride 0 shares one filter across the batch. */
fufft_status fufft_conv2d_f32(const float* a, const float* b, float* out, int h, int w, int64_t batch,
                              fufft_layout layout, fufft_midop mid, int64_t filter_stride,
                              fufft_stream_t stream);

/* ---- split forward / apply (one signal, many filters) -------------------
 * fwd: natural-order signal -> spectrum.  Replaces fufft_pipeline_fwd
 * (fufft.cuh:1343-1373).  The spectrum's order follows the layout, like a
 * filter's: R8 / R16 give the chain (digit-reversed) order of the reference;
 * R8_BPERM / R16_BPERM the register-boundary order of the same values
 * (spec[L + k*T] = chain[V*L + k], T = n/V), whose loads and stores are
 * coalesced -- the faster pair.
 * apply: spectrum (x) filter -> inverse -> natural order, both operands in
 * the order of `layout`.  Replaces fufft_pipeline_apply (fufft.cuh:1375-1407,
 * multiply only there); spec_stride is the element distance between
 * consecutive transforms' spectra (n, or 0 to apply many filters to one
 * spectrum). */
fufft_status fufft_fwd_f32(const float* a, float* spec, int n, int64_t batch, fufft_layout layout,
                           fufft_stream_t stream);
fufft_status fufft_apply_f32(const float* spec, const float* b, float* out, int n, int64_t batch,
                             fufft_layout layout, fufft_midop mid, int64_t spec_stride,
                             int64_t filter_stride, fufft_stream_t stream);

/* ---- natural-order transform -------------------------------------------
 * out = DFT(in) (sign -1) or the unnormalised inverse (sign +1), natural
 * order on both sides, 8 <= n <= 8192, in == out allowed.  Replaces the
 * reference's forward-only fufft_c2c (fufft.cuh:878-904, radix-8 Stockham,
 * powers of 8): one kernel, the DIF chain in registers and one swizzled
 * shared-memory scatter into natural order. */
fufft_status fufft_c2c_f32(const float* in, float* out, int n, int64_t batch, int sign, fufft_stream_t stream);

/* ---- the one-signal-many-filters shape at scale (no reference counterpart:
 * the reference's apply pairs spectrum i with filter i, fufft.cuh:1393-1395)
 * fwd_r2: two real signals as one complex transform, xr + i*yr -> spectrum
 *   in the order of `layout`, as fufft_fwd_f32 (the two-for-one packing of
 *   fufft_conv_r2, fufft.cuh:1283-1290, stopped at the register boundary).
 * apply_grid: every spectrum s < n_spec against every filter f < n_filt in one
 *   launch; out[s][f][0..n) = IDFT(spec_s (x) b_f), complex.  Spectra and
 *   filters are n apart, both in the order of `layout`.  mid is MULTIPLY or
 *   CONJ_MULTIPLY.
 * apply_grid_r2: the same for packed real pairs and REAL filters: pair s holds
 *   real signals 2s and 2s+1, and out is real, out[2s + j][f][0..n) for
 *   j = 0 (xr) and 1 (yr): signal i's filtered copies are rows i*n_filt ..
 *   (i+1)*n_filt-1 of an [2*n_pairs*n_filt][n] real array.  CONJ_MULTIPLY
 *   gives the cyclic cross-correlation with the filter. */
fufft_status fufft_fwd_r2_f32(const float* xr, const float* yr, float* spec, int n, int64_t batch,
                              fufft_layout layout, fufft_stream_t stream);
fufft_status fufft_apply_grid_f32(const float* spec, int64_t n_spec, const float* b, int64_t n_filt, float* out,
                                  int n, fufft_layout layout, fufft_midop mid, fufft_stream_t stream);
fufft_status fufft_apply_grid_r2_f32(const float* spec, int64_t n_pairs, const float* b, int64_t n_filt,
                                     float* out, int n, fufft_layout layout, fufft_midop mid,
                                     fufft_stream_t stream);

/* ---- two-for-one real convolution ---------------------------------------
 * Two real signals ride one complex transform (xr + i*yr); the filter must be
 * the spectrum of a REAL filter.  ur = xr (*) h, vr = yr (*) h.
 * Replaces fufft_conv_r2 (fufft.cuh:1273-1330). */
fufft_status fufft_conv_r2_f32(const float* xr, const float* yr, const float* b, float* ur, float* vr,
                               int n, int64_t batch, fufft_layout layout, fufft_midop mid,
                               int64_t filter_stride, fufft_stream_t stream);

/* ---- int16 block floating point -----------------------------------------
 * pack: fp32 complex -> int16 pairs + one scale per transform:
 *   mx = max(|re|,|im|) (>= 1e-30), q = rint(clamp(x * 32767/mx, +-32767)),
 *   scale = mx / 32767 -- bit-exact with bfp_quant_host (bench_fufft.cu:107-117)
 *   and bfp_quantize (verify_kernel.cpp:1092-1105).
 * unpack: q * scale. */
fufft_status fufft_bfp_pack(const float* x, int16_t* q, float* scale, int n, int64_t batch,
                            fufft_stream_t stream);
fufft_status fufft_bfp_unpack(const int16_t* q, const float* scale, float* x, int n, int64_t batch,
                              fufft_stream_t stream);
/* fused BFP convolution: dequantise, fp32 transforms, filter mid-op,
 * per-transform abs-max, requantise.  Replaces fufft_pipeline_v16_bfp
 * (fufft.cuh:1614-1701; layout R16, filter quantised per transform).  The
 * filter scale array has one entry per filter (1 when filter_stride == 0). */
fufft_status fufft_conv_c2c_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq,
                                const float* b_scale, int16_t* oq, float* o_scale, int n, int64_t batch,
                                fufft_layout layout, fufft_midop mid, int64_t filter_stride,
                                fufft_stream_t stream);

/* ---- four-step large N -------------------------------------------------
 * N = r_out^LOUT * mid (r_out 8 or 16, mid a one-kernel size >= 256 of the
 * layout's radix): LOUT outer DIF passes over HBM, the fused convolution on
 * each mid-point chunk, LOUT outer DIT passes (4*LOUT + 3 HBM passes).  The
 * filter is in the chain order of the whole sequence [r_out]*LOUT ++ middle
 * chain (verify_kernel.cpp:460-477 chain_rev; bench_fufft.cu:414-428); with a
 * BPERM layout each mid-point chunk of it is additionally in the middle's
 * register-boundary order.  fp32 runs in place on buf.
 * Replaces run_large / fufft_outer_pass_r / MidLaunch (bench_fufft.cu:368-451,
 * fufft.cuh:1113-1165, :1717-1734).
 * fufft_large_plan picks (r_out, mid) for n: radix-16 outer levels first. */
fufft_status fufft_large_plan(int64_t n, fufft_layout layout, int* r_out, int* mid);
fufft_status fufft_conv_large_f32(float* buf, const float* b, int64_t n, int64_t batch, int r_out, int mid,
                                  fufft_layout layout, fufft_midop mid_op, fufft_stream_t stream);
/* int16-BFP four-step (new: the reference's four-step is fp32 only).  Input,
 * filter and output are int16 pairs with one scale per N-point transform
 * (filter: quantised as one N-point block in chain order).  The intermediate
 * passes run in fp32 in a caller-provided workspace of
 * fufft_conv_large_bfp_workspace(n, batch) bytes (16-byte aligned); the output
 * scale is max|.|/32767 over the whole transform, as in the one-kernel form. */
size_t fufft_conv_large_bfp_workspace(int64_t n, int64_t batch);
fufft_status fufft_conv_large_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq, const float* b_scale,
                                  int16_t* oq, float* o_scale, int64_t n, int64_t batch, int r_out, int mid,
                                  fufft_layout layout, fufft_midop mid_op, void* workspace, size_t workspace_bytes,
                                  fufft_stream_t stream);

/* ---- distributed single-signal convolution (new: the reference is single-GPU)
 * One n-point transform over `world` ranks (2, 4 or 8), viewed as
 * [world][n/world]: rank g holds columns col0 = g*cols .. col0+cols-1 of every
 * row, cols = n/world^2, row k at x_local + k*cols.  fufft_dist_pass runs this
 * rank's share of the first DIF (sign -1) or last DIT (sign +1) radix-world
 * pass at stride n/world, in place.  Between the two, one all-to-all gives rank
 * k block k, which is convolved as an n/world-point transform with block k of
 * the chain-ordered filter (chain [world] ++ the block's chain); a second
 * all-to-all returns it.  fufft_b200.distributed drives the sequence over
 * torch.distributed (NCCL). */
fufft_status fufft_dist_pass(float* x_local, int world, int64_t cols, int64_t col0, int64_t n, int sign,
                             fufft_stream_t stream);

/* The same passes with the all-to-all fused in, over NVLink peer memory:
 * every rank holds an n/world-point block buffer mapped into all ranks
 * (fufft_peer_alloc / fufft_peer_open); peer_blocks is a HOST array of the
 * world block addresses as seen from this process (this rank's own at index
 * rank).  push: the first DIF pass of this rank's columns, row k's results
 * stored straight into rank k's block at offset rank*cols.  pull: the last
 * DIT pass, row k's inputs loaded straight from rank k's block.  Between push
 * and the block convolution, and between it and pull, every rank must have
 * finished (a barrier on the stream, e.g. a one-element all-reduce). */
fufft_status fufft_dist_pass_push(const float* x_local, const uint64_t* peer_blocks, int world, int rank,
                                  int64_t cols, int64_t n, fufft_stream_t stream);
fufft_status fufft_dist_pass_pull(float* x_local, const uint64_t* peer_blocks, int world, int rank, int64_t cols,
                                  int64_t n, fufft_stream_t stream);

/* Device buffers the other processes of the node can map (CUDA IPC).
 * alloc: `bytes` of device memory and its FUFFT_IPC_HANDLE_BYTES-byte handle;
 * open: map a handle from another process (FUFFT_ERR_PEER_UNAVAILABLE if the
 * GPUs cannot reach each other); close: unmap; free: release own buffer. */
#define FUFFT_IPC_HANDLE_BYTES 64
fufft_status fufft_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
fufft_status fufft_peer_open(const void* ipc_handle, void** dev_ptr);
fufft_status fufft_peer_close(void* dev_ptr);
fufft_status fufft_peer_free(void* dev_ptr);

/* ---- several GPUs from one host thread (new: the reference is single-GPU).
 * fufft_conv_multi_gpu runs one job over the GPUs of desc->shards.  It
 * enqueues on every shard's stream and returns without waiting, and it leaves
 * the caller's current device as it found it.  Modes:
 *   FUFFT_MG_BATCH: independent transforms.  Shard i convolves its own
 *     `batch` transforms exactly as fufft_conv_c2c_f32 would, with
 *     desc->layout / mid / filter_stride.  a, b, out are device memory of
 *     shard i's GPU.
 *   FUFFT_MG_BATCH_HOST: the same from pinned host memory.  Shard i runs
 *     fufft_conv_c2c_f32_host on its GPU with its own workspace
 *     (fufft_conv_host_workspace bytes on that GPU), so each GPU's PCIe link
 *     carries its own slice.
 *   FUFFT_MG_SINGLE_SIGNAL: one n-point convolution over 2, 4 or 8 shards
 *     (shard index = rank), the scheme of fufft_dist_pass_push / _pull.
 *     out: this rank's [world][n/world^2] slice of the signal, convolved in
 *     place (a must be NULL or equal to out).
 *     b: block `rank` of the filter, n/world points in the order of
 *     fufft_mg_chain, with 1/n folded in.
 *     workspace: n/world complex points on the shard's GPU; every rank stores
 *     into it and later loads from it.
 *     Distinct GPUs must reach each other by peer access, else
 *     FUFFT_ERR_PEER_UNAVAILABLE; shards may share a GPU.  Events between the
 *     shard streams order the phases, so no kernel of one rank waits on the
 *     device for another rank.
 * Arguments common to all shards are checked before the first launch.  The
 * BATCH modes check each shard's pointers when its turn comes; a CUDA error or
 * a rejected shard returns at once, and work already queued on earlier shards
 * stays queued. */
typedef enum fufft_mg_mode {
   FUFFT_MG_BATCH = 0,
   FUFFT_MG_BATCH_HOST = 1,
   FUFFT_MG_SINGLE_SIGNAL = 2
} fufft_mg_mode;
typedef struct fufft_mg_shard {
   int device;              /* CUDA device ordinal */
   fufft_stream_t stream;   /* a stream of that device (NULL: its legacy default stream) */
   const float* a;          /* signal (BATCH, BATCH_HOST) */
   const float* b;          /* filter(s) or the rank's filter block */
   float* out;              /* result, or the rank's slice (SINGLE_SIGNAL, in place) */
   int64_t batch;           /* transforms of this shard (BATCH, BATCH_HOST) */
   void* workspace;         /* BATCH_HOST: pipeline slots; SINGLE_SIGNAL: the rank's block */
   size_t workspace_bytes;
} fufft_mg_shard;
typedef struct fufft_mg_desc {
   fufft_mg_mode mode;
   int n_shards;            /* 1..FUFFT_MG_MAX_SHARDS; SINGLE_SIGNAL: 2, 4 or 8 */
   const fufft_mg_shard* shards;
   int64_t n;               /* points per transform (SINGLE_SIGNAL: of the one signal) */
   fufft_layout layout;     /* filter layout (BATCH, BATCH_HOST) */
   fufft_midop mid;
   int64_t filter_stride;   /* BATCH, BATCH_HOST: as in fufft_conv_c2c_f32 */
} fufft_mg_desc;
#define FUFFT_MG_MAX_SHARDS 64
fufft_status fufft_conv_multi_gpu(const fufft_mg_desc* desc);

/* Radix chain of the whole n-point transform of FUFFT_MG_SINGLE_SIGNAL over
 * `world` ranks: [world] followed by the block's chain.  Written to
 * radices_out (room for 32).  Returns its length, or -1 if the shape is not
 * supported.  Filter slot p holds spectrum bin
 * fufft_chain_rev(p, radices, length). */
int fufft_mg_chain(int64_t n, int world, int* radices_out);

/* The same BFP four-step for callers that cannot allocate device memory when
 * they call the library (a host whose device memory is entirely held by its
 * own pool allocator, or a latency-critical loop where an allocation's
 * possible device-wide synchronisation is not acceptable).  No counterpart in
 * the reference.  Instead of a caller workspace it uses a fixed scratch area
 * of FUFFT_NOALLOC_SCRATCH_BYTES that the library reserves on every GPU that
 * loads it (held until exit): 8 * n * batch must not exceed it, else
 * FUFFT_ERR_INVALID_SIZE -- for every request, including the one-outer-level
 * radix-16 plans that would not touch the area.  Other arguments are checked
 * first, in the order and with the status codes of fufft_conv_large_bfp.  All
 * calls on a device share that area, so calls that may overlap on the GPU
 * race -- keep them on one stream.  The first successful call on a device
 * looks up the area's address (a failed lookup is retried by the next call);
 * make it before any stream capture.  Allocates nothing. */
#define FUFFT_NOALLOC_SCRATCH_BYTES (16u << 20)
fufft_status fufft_conv_large_bfp_noalloc(const int16_t* aq, const float* a_scale, const int16_t* bq,
                                          const float* b_scale, int16_t* oq, float* o_scale, int64_t n,
                                          int64_t batch, int r_out, int mid, fufft_layout layout,
                                          fufft_midop mid_op, fufft_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FUFFT_B200_H */
