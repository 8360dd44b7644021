// fufft_api.cu -- C ABI entry points of the fused convolutions: argument
// validation, then one launch of the matching kernel family.
#include "fufft_internal.cuh"

using namespace fufft;
using namespace fufft::host;

namespace {

// common checks; fills args.tw / args.status; returns FUFFT_OK or an error.
// `*skip` is set when there is nothing to launch (batch == 0).
fufft_status prepare(int n, int64_t batch, fufft_layout layout, int* radix, ConvArgs* args, int* dev,
                     bool* skip)
{
   *skip = false;
   const int R = layout_radix(layout);
   if(!R) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(n) || n < R || n > max_n(R)) return FUFFT_ERR_INVALID_SIZE;
   if(batch < 0 || batch > (int64_t)1 << 40) return FUFFT_ERR_INVALID_BATCH;
   *radix = R;
   if(batch == 0) { *skip = true; return FUFFT_OK; }
   DeviceCtx c;
   fufft_status s = device_ctx(&c);
   if(s != FUFFT_OK) return s;
   args->tw = c.tw;
   args->status = c.status;
   args->batch = batch;
   *dev = c.device;
   return FUFFT_OK;
}

// filter pointer/stride rules shared by every mid-op entry point
fufft_status check_filter(const void* b, fufft_midop mid, int64_t filter_stride, int elem)
{
   if(mid < FUFFT_MID_NONE || mid > FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   if(mid == FUFFT_MID_NONE) return FUFFT_OK;
   if(!b) return FUFFT_ERR_INVALID_ARG;
   if(filter_stride < 0) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(b, 16) || (filter_stride * elem) % 16) return FUFFT_ERR_MISALIGNED;
   return FUFFT_OK;
}

}  // namespace

extern "C" {

fufft_status fufft_conv_c2c_f32(const float* a, const float* b, float* out, int n, int64_t batch,
                                fufft_layout layout, fufft_midop mid, int64_t filter_stride,
                                fufft_stream_t stream)
{
   // radix-16 transforms beyond one CTA: the cluster-fused kernel (chain [C, 16, 16, 16])
   if(layout_radix(layout) == 16 && pow2(n) && n > MAX_N_R16 && n <= MAX_N_CLUSTER) {
      if(batch < 0 || batch > (int64_t)1 << 40) return FUFFT_ERR_INVALID_BATCH;
      if(batch == 0) return FUFFT_OK;
      if(!a || !out) return FUFFT_ERR_INVALID_ARG;
      if(!aligned(a, 8) || !aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
      fufft_status s = check_filter(b, mid, filter_stride, 8);
      if(s != FUFFT_OK) return s;
      DeviceCtx c;
      if((s = device_ctx(&c)) != FUFFT_OK) return s;
      ConvArgs args{};
      args.tw = c.tw;
      args.status = c.status;
      args.batch = batch;
      args.a = a;
      args.b = b;
      args.out = out;
      args.filter_stride = filter_stride;
      return cluster_conv1d(n, mid, layout_bperm(layout), args, reinterpret_cast<cudaStream_t>(stream), c.device);
   }
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!a || !out) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(a, 8) || !aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   if((s = check_filter(b, mid, filter_stride, 8)) != FUFFT_OK) return s;
   args.a = a;
   args.b = b;
   args.out = out;
   args.filter_stride = filter_stride;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_conv_f32_r8 : family_conv_f32_r16)(n, mid, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_fwd_f32(const float* a, float* spec, int n, int64_t batch, fufft_layout layout,
                           fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!a || !spec) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(a, 8) || !aligned(spec, 16)) return FUFFT_ERR_MISALIGNED;
   args.a = a;
   args.out = spec;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_fwd_r8 : family_fwd_r16)(n, FUFFT_MID_NONE, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_apply_f32(const float* spec, const float* b, float* out, int n, int64_t batch,
                             fufft_layout layout, fufft_midop mid, int64_t spec_stride,
                             int64_t filter_stride, fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!spec || !out) return FUFFT_ERR_INVALID_ARG;
   if(spec_stride < 0) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(spec, 16) || (spec_stride * 8) % 16 || !aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   if((s = check_filter(b, mid, filter_stride, 8)) != FUFFT_OK) return s;
   args.a = spec;
   args.b = b;
   args.out = out;
   args.spec_stride = spec_stride;
   args.filter_stride = filter_stride;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_apply_r8 : family_apply_r16)(n, mid, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_filter_from_taps_f32(const float* taps, float* out, int n, int64_t batch, fufft_layout layout,
                                       fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!taps || !out) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(taps, 8) || !aligned(out, 16)) return FUFFT_ERR_MISALIGNED;
   args.a = taps;
   args.out = out;
   args.spec_scale = 1.0f / (float)n;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_fwd_r8 : family_fwd_r16)(n, FUFFT_MID_NONE, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_c2c_f32(const float* in, float* out, int n, int64_t batch, int sign, fufft_stream_t stream)
{
   if(sign != -1 && sign != 1) return FUFFT_ERR_INVALID_ARG;
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   // radix-16 chain from 16 points on, radix 8 for n = 8
   const fufft_layout layout = n >= 16 ? FUFFT_LAYOUT_R16 : FUFFT_LAYOUT_R8;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!in || !out) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(in, 8) || !aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   args.a = in;
   args.out = out;
   args.conj_io = sign > 0;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_c2c_r8 : family_c2c_r16)(n, FUFFT_MID_NONE, false, args, st, dev);
}

fufft_status fufft_fwd_r2_f32(const float* xr, const float* yr, float* spec, int n, int64_t batch,
                              fufft_layout layout, fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!xr || !yr || !spec) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(xr, 4) || !aligned(yr, 4) || !aligned(spec, 16)) return FUFFT_ERR_MISALIGNED;
   args.a = xr;
   args.a2 = yr;
   args.out = spec;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_fwd_r2_r8 : family_fwd_r2_r16)(n, FUFFT_MID_NONE, layout_bperm(layout), args, st, dev);
}

// every spectrum x every filter in one launch: transform t = s * n_filt + f
static fufft_status apply_grid(const float* spec, int64_t n_spec, const float* b, int64_t n_filt, float* out,
                               int n, fufft_layout layout, fufft_midop mid, bool real_pair, fufft_stream_t stream)
{
   if(n_spec < 0 || n_filt < 0) return FUFFT_ERR_INVALID_BATCH;
   if(n_filt > 0 && n_spec > ((int64_t)1 << 40) / n_filt) return FUFFT_ERR_INVALID_BATCH;
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, n_spec * n_filt, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!spec || !out) return FUFFT_ERR_INVALID_ARG;
   if(mid != FUFFT_MID_MULTIPLY && mid != FUFFT_MID_CONJ_MULTIPLY) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(spec, 16) || !aligned(out, real_pair ? 4 : 8)) return FUFFT_ERR_MISALIGNED;
   if((s = check_filter(b, mid, n, 8)) != FUFFT_OK) return s;
   args.a = spec;
   args.b = b;
   args.out = out;
   args.filter_stride = n;
   args.grid_filters = n_filt;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   if(!real_pair) return (R == 8 ? family_apply_r8 : family_apply_r16)(n, mid, layout_bperm(layout), args, st, dev);
   args.out2 = out + (size_t)n_filt * n;
   return (R == 8 ? family_apply_r2_r8 : family_apply_r2_r16)(n, mid, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_apply_grid_f32(const float* spec, int64_t n_spec, const float* b, int64_t n_filt, float* out,
                                  int n, fufft_layout layout, fufft_midop mid, fufft_stream_t stream)
{
   return apply_grid(spec, n_spec, b, n_filt, out, n, layout, mid, false, stream);
}

fufft_status fufft_apply_grid_r2_f32(const float* spec, int64_t n_pairs, const float* b, int64_t n_filt,
                                     float* out, int n, fufft_layout layout, fufft_midop mid,
                                     fufft_stream_t stream)
{
   return apply_grid(spec, n_pairs, b, n_filt, out, n, layout, mid, true, stream);
}

fufft_status fufft_conv_r2_f32(const float* xr, const float* yr, const float* b, float* ur, float* vr,
                               int n, int64_t batch, fufft_layout layout, fufft_midop mid,
                               int64_t filter_stride, fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!xr || !yr || !ur || !vr) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(xr, 4) || !aligned(yr, 4) || !aligned(ur, 4) || !aligned(vr, 4)) return FUFFT_ERR_MISALIGNED;
   if((s = check_filter(b, mid, filter_stride, 8)) != FUFFT_OK) return s;
   args.a = xr;
   args.a2 = yr;
   args.b = b;
   args.out = ur;
   args.out2 = vr;
   args.filter_stride = filter_stride;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_r2_r8 : family_r2_r16)(n, mid, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_conv_c2c_bfp(const int16_t* aq, const float* a_scale, const int16_t* bq,
                                const float* b_scale, int16_t* oq, float* o_scale, int n, int64_t batch,
                                fufft_layout layout, fufft_midop mid, int64_t filter_stride,
                                fufft_stream_t stream)
{
   ConvArgs args{};
   int R = 0, dev = 0;
   bool skip;
   fufft_status s = prepare(n, batch, layout, &R, &args, &dev, &skip);
   if(s != FUFFT_OK || skip) return s;
   if(!aq || !a_scale || !oq || !o_scale) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(aq, 4) || !aligned(oq, 4) || !aligned(a_scale, 4) || !aligned(o_scale, 4))
      return FUFFT_ERR_MISALIGNED;
   if((s = check_filter(bq, mid, filter_stride, 4)) != FUFFT_OK) return s;
   if(mid != FUFFT_MID_NONE && !b_scale) return FUFFT_ERR_INVALID_ARG;
   args.a = aq;
   args.a_scale = a_scale;
   args.b = bq;
   args.b_scale = b_scale;
   args.out = oq;
   args.out_scale = o_scale;
   args.filter_stride = filter_stride;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   return (R == 8 ? family_conv_bfp_r8 : family_conv_bfp_r16)(n, mid, layout_bperm(layout), args, st, dev);
}

fufft_status fufft_conv2d_f32(const float* a, const float* b, float* out, int h, int w, int64_t batch,
                              fufft_layout layout, fufft_midop mid, int64_t filter_stride, fufft_stream_t stream)
{
   const int R = layout_radix(layout);
   if(!R) return FUFFT_ERR_INVALID_ARG;
   if(!pow2(h) || !pow2(w)) return FUFFT_ERR_INVALID_SIZE;
   const bool cluster = R == 16 && cluster_conv2d_shape(h, w);
   if(!cluster && !(R == 8 ? conv2d_supported_r8(h, w) : conv2d_supported_r16(h, w))) return FUFFT_ERR_INVALID_SIZE;
   if(batch < 0 || batch > (int64_t)1 << 40) return FUFFT_ERR_INVALID_BATCH;
   if(batch == 0) return FUFFT_OK;
   if(!a || !out) return FUFFT_ERR_INVALID_ARG;
   if(!aligned(a, 8) || !aligned(out, 8)) return FUFFT_ERR_MISALIGNED;
   fufft_status s = check_filter(b, mid, filter_stride, 8);
   if(s != FUFFT_OK) return s;
   DeviceCtx c;
   if((s = device_ctx(&c)) != FUFFT_OK) return s;
   ConvArgs args{};
   args.tw = c.tw;
   args.status = c.status;
   args.batch = batch;
   args.a = a;
   args.b = b;
   args.out = out;
   args.filter_stride = filter_stride;
   cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
   if(cluster) return cluster_conv2d(h, w, mid, layout_bperm(layout), args, st, c.device);
   return (R == 8 ? family_conv2d_r8 : family_conv2d_r16)(h, w, mid, layout_bperm(layout), args, st, c.device);
}

}  // extern "C"
