// subsampling.cpp -- the dw_striding subsampling (the encoder's pre_encode,
// src/asr/modules/encoders/conformer.rs:1058-1588) behind the C ABI.
//
// One forward with n strides (log2 of the factor) on NHWC bf16 activations:
//   conv.0 + ReLU and the first depthwise conv      one kernel (the conv.0
//                                                   activations stay on chip)
//   pointwise conv + ReLU                           tcgen05 GEMM, ReLU epilogue
//   [further strides] depthwise conv; pointwise conv + ReLU
//   out linear                                      tcgen05 GEMM
// The reference flattens [B, T', F', C] as [B, T', C, F'] (channel-major, as
// NeMo's [B, C, T, F] permute does) before `out`; here the activations stay
// [B, T', F', C] and the columns of `out`'s weight are permuted once at load
// to the same order, so no transpose runs.  A quantised `out` is dequantised
// on the host at load (a 5 MB weight: its bf16 copy is what the 8-bit GEMM
// path would make each call).  By default the whole input is processed at
// once (the largest buffer, the first pointwise conv's output, is
// 2 * T/4 * F/4 * C bytes per utterance); nrp_subsampling_set_chunk_frames
// selects the reference's time chunking (forward_frames_chunked,
// 1334-1377), which bounds that memory and gives the same frames: each
// output frame is computed from the same input frames by the same
// arithmetic.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "../../include/nemo_relpos.h"
#include "gemm.h"
#include "handles.h"
#include "internal.h"

namespace {

using nrp::failf;

#define TRY_CUDA(expr)                                                        \
  do {                                                                        \
    const cudaError_t e_ = (expr);                                            \
    if (e_ != cudaSuccess) {                                                  \
      (void)cudaGetLastError(); /* not left for later launch checks */        \
      return failf(NRP_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
    }                                                                         \
  } while (0)

constexpr int kMaxStrides = 3;

// Subsampling::new (conformer.rs:1118-1123)
int strides_of(int factor) { return factor == 2 ? 1 : factor == 4 ? 2 : factor == 8 ? 3 : 2; }

// One stride-2 kernel-3 conv (1306-1326): causal floor(n/2) + 1, otherwise
// floor((n - 1)/2) + 1 with floor division.
int conv_len(int n, bool causal) {
  const int p = causal ? n : n - 1;
  return (p >= 0 ? p / 2 : -((-p + 1) / 2)) + 1;
}

struct HostConv {
  bool loaded = false;
  std::vector<float> w, b;
};

}  // namespace

struct nrp_subsampling {
  nrp_context* ctx = nullptr;
  int F = 0, D = 0, factor = 8, C = 256, S = 3;
  bool causal = false;
  int Fp = 0;  // F' (compute_freq_output_size)
  int dtype = NRP_DTYPE_F32;
  HostConv conv[kMaxStrides];  // conv.0, then the depthwise convs
  HostConv pw[kMaxStrides - 1];
  nrp::Linear out;
  bool dirty = true;
  nrp::DevBuf d_frag[kMaxStrides];  // conv.0, then depthwise, MMA B fragments
  nrp::DevBuf d_pw_w[kMaxStrides - 1], d_pw_b[kMaxStrides - 1];  // bf16 [C][C], [C]
  nrp::DevBuf d_out_w, d_out_b;  // bf16 [D][F' * C] (columns f' * C + c), [D]
  bool has_out_b = false;
  nrp::DevBuf act[2];  // ping-pong NHWC activations
  int chunk_frames = 0;   // mel frames per time chunk (0: the whole input at once)
  nrp::DevBuf chunk_out;  // one chunk's output frames, before the crop
};

namespace {

cudaError_t upload_bf16v(nrp::DevBuf& dst, const std::vector<float>& v) {
  std::vector<uint16_t> h(v.size());
  for (size_t i = 0; i < v.size(); ++i) h[i] = nrp::bf16_bits(v[i]);
  cudaError_t e = dst.ensure(h.size() * 2);
  if (e == cudaSuccess) e = cudaMemcpy(dst.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
  return e;
}

cudaError_t upload_u32(nrp::DevBuf& dst, const std::vector<uint32_t>& v) {
  cudaError_t e = dst.ensure(v.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(dst.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
  return e;
}

// Device parameters in bf16 (Subsampling::set_dtype, conformer.rs:1098-1108:
// every parameter rounded to the dtype).
int sync_sub(nrp_subsampling* s) {
  if (!s->dirty) return NRP_OK;
  const int C = s->C, K = s->C * s->Fp;
  for (int i = 0; i < s->S; ++i)
    if (!s->conv[i].loaded || (i > 0 && !s->pw[i - 1].loaded))
      return failf(NRP_ERR_INVALID, "subsampling conv weights not loaded (stage %d)", i);
  if (!s->out.loaded) return failf(NRP_ERR_INVALID, "subsampling out weights not loaded");
  for (int i = 0; i < s->S; ++i) {
    std::vector<uint32_t> frag;
    if (i == 0)
      nrp::subsample_conv0_frags(s->conv[i].w.data(), s->conv[i].b.data(), C, frag);
    else
      nrp::subsample_dw_frags(s->conv[i].w.data(), s->conv[i].b.data(), C, frag);
    TRY_CUDA(upload_u32(s->d_frag[i], frag));
  }
  for (int i = 0; i + 1 < s->S; ++i) {
    TRY_CUDA(upload_bf16v(s->d_pw_w[i], s->pw[i].w));
    TRY_CUDA(upload_bf16v(s->d_pw_b[i], s->pw[i].b));
  }
  std::vector<float> w;
  if (s->out.quant)
    nrp::dequant_linear_host(s->out, s->D, K, w);
  else
    w = s->out.w;
  // column c * F' + f (the reference's flattening) -> f * C + c (NHWC)
  std::vector<float> wp(w.size());
  for (int n = 0; n < s->D; ++n)
    for (int c = 0; c < C; ++c)
      for (int f = 0; f < s->Fp; ++f)
        wp[static_cast<size_t>(n) * K + static_cast<size_t>(f) * C + c] =
            w[static_cast<size_t>(n) * K + static_cast<size_t>(c) * s->Fp + f];
  TRY_CUDA(upload_bf16v(s->d_out_w, wp));
  s->has_out_b = !s->out.bias.empty();
  if (s->has_out_b) TRY_CUDA(upload_bf16v(s->d_out_b, s->out.bias));
  s->dirty = false;
  return NRP_OK;
}

}  // namespace

namespace nrp {

namespace {
uint32_t pack_pair(float lo, float hi) {
  return static_cast<uint32_t>(bf16_bits(lo)) | (static_cast<uint32_t>(bf16_bits(hi)) << 16);
}
}  // namespace

void subsample_conv0_frags(const float* w, const float* b, int C, std::vector<uint32_t>& out) {
  out.assign(static_cast<size_t>(C / 32) * 32 * kSubFragWords, 0u);
  for (int cg = 0; cg < C / 32; ++cg)
    for (int lane = 0; lane < 32; ++lane) {
      const int g = lane >> 2, t = lane & 3;
      uint32_t* o = out.data() + (static_cast<size_t>(cg) * 32 + lane) * kSubFragWords;
      for (int nt = 0; nt < 4; ++nt) {
        const float* wc = w + (cg * 32 + 8 * nt + g) * 9;
        const int cb = cg * 32 + 8 * nt + 2 * t;
        o[3 * nt] = pack_pair(wc[2 * t], wc[2 * t + 1]);
        o[3 * nt + 1] = t == 0 ? pack_pair(wc[8], 0.f) : 0u;
        o[3 * nt + 2] = pack_pair(b[cb], b[cb + 1]);
      }
    }
}

void subsample_dw_frags(const float* w, const float* b, int C, std::vector<uint32_t>& out) {
  out.assign(static_cast<size_t>(C / 8) * 32 * kSubFragWords, 0u);
  for (int q = 0; q < C / 8; ++q)
    for (int lane = 0; lane < 32; ++lane) {
      const int g = lane >> 2, t = lane & 3;
      uint32_t* o = out.data() + (static_cast<size_t>(q) * 32 + lane) * kSubFragWords;
      const float* wc = w + (q * 8 + g) * 9;
      for (int j = 0; j < 5; ++j) {
        const float lo = wc[2 * j], hi = j < 4 ? wc[2 * j + 1] : 0.f;
        o[2 * j] = pack_pair(g == 2 * t ? lo : 0.f, g == 2 * t + 1 ? lo : 0.f);
        o[2 * j + 1] = pack_pair(g == 2 * t ? hi : 0.f, g == 2 * t + 1 ? hi : 0.f);
      }
      o[10] = pack_pair(b[q * 8 + 2 * t], b[q * 8 + 2 * t + 1]);
    }
}

int subsampling_output_frames(const nrp_subsampling* s, int frames) {
  for (int i = 0; i < s->S; ++i) frames = conv_len(frames, s->causal);
  return std::max(frames, 0);
}

int subsampling_feat_in(const nrp_subsampling* s) { return s->F; }

namespace {

// The conv stack and `out` over mel frames [0, T) of mel (lengths counted
// from frame len_off of the full input).
int run_frames(nrp_subsampling* s, cudaStream_t st, const float* mel, int64_t bs, int64_t ts,
               int64_t fs, int B, int T, const int32_t* lengths, int len_off, void* out) {
  int rc = NRP_OK;
  const int C = s->C, pad = s->causal ? 2 : 1;
  int Ti[kMaxStrides + 1], Fi[kMaxStrides + 1];
  Ti[0] = T;
  Fi[0] = s->F;
  for (int i = 0; i < s->S; ++i) {
    Ti[i + 1] = conv_len(Ti[i], s->causal);
    Fi[i + 1] = conv_len(Fi[i], s->causal);
  }
  const int fused = s->S >= 2 ? 2 : 1;  // stages the first kernel covers
  if (Fi[1] > 80)
    return failf(NRP_ERR_UNSUPPORTED, "feat_in %d: the conv.0 kernel takes at most 80 conv.0 "
                 "columns (feat_in <= 158)", s->F);
  size_t act_elems = static_cast<size_t>(B) * Ti[fused] * Fi[fused] * C;
  TRY_CUDA(s->act[0].ensure(act_elems * 2));
  TRY_CUDA(s->act[1].ensure(act_elems * 2));
  // the last activation is the out GEMM's input: F' * C columns per frame
  __nv_bfloat16* buf[2] = {s->act[0].as<__nv_bfloat16>(), s->act[1].as<__nv_bfloat16>()};
  {
    SubConvArgs a;
    a.mel = mel;
    a.mel_bs = bs;
    a.mel_ts = ts;
    a.mel_fs = fs;
    a.len = lengths;
    a.len_off = len_off;
    a.T = T;
    a.F = s->F;
    a.T1 = Ti[1];
    a.F1 = Fi[1];
    a.T2 = fused == 2 ? Ti[2] : 0;
    a.F2 = fused == 2 ? Fi[2] : 0;
    a.C = C;
    a.pad = pad;
    a.f0 = s->d_frag[0].as<uint32_t>();
    if (fused == 2) a.f1 = s->d_frag[1].as<uint32_t>();
    a.out = buf[0];
    ProfScope ps(s->ctx, NRP_KERNEL_SUBSAMPLE, st);
    TRY_CUDA(launch_subsample_conv0(a, B, fused == 2, st));
  }
  int cur = 0;
  for (int i = 1; i < s->S; ++i) {
    if (i >= 2) {  // a further depthwise conv
      ProfScope ps(s->ctx, NRP_KERNEL_SUBSAMPLE, st);
      TRY_CUDA(launch_subsample_dw(buf[cur], B, Ti[i], Fi[i], C, pad,
                                   s->d_frag[i].as<uint32_t>(), buf[cur ^ 1], Ti[i + 1],
                                   Fi[i + 1], s->ctx->num_sms, st));
      cur ^= 1;
    }
    // pointwise conv + ReLU over [B * T_i+1 * F_i+1, C]
    Epilogue ep;
    ep.mode = kEpiRelu;
    const int M = B * Ti[i + 1] * Fi[i + 1];
    rc = linear(s->ctx, st, NRP_DTYPE_BF16, buf[cur], M, C, s->d_pw_w[i - 1].p, false, nullptr,
                nullptr, C, s->d_pw_b[i - 1].p, buf[cur ^ 1], C, RowTiling(), ep);
    if (rc) return rc;
    cur ^= 1;
  }
  const int Tp = Ti[s->S], K = C * Fi[s->S];
  return linear(s->ctx, st, NRP_DTYPE_BF16, buf[cur], B * Tp, K, s->d_out_w.p, false, nullptr,
                nullptr, s->D, s->has_out_b ? s->d_out_b.p : nullptr, out, s->D, RowTiling(),
                Epilogue());
}

}  // namespace

int subsampling_run(nrp_subsampling* s, cudaStream_t st, const float* mel, int64_t bs, int64_t ts,
                    int64_t fs, int B, int T, const int32_t* lengths, void* out) {
  if (s->dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_UNSUPPORTED, "the subsampling runs in bf16 (nrp_subsampling_set_dtype)");
  if (B <= 0 || T <= 0) return failf(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  if (!s->ctx) return failf(NRP_ERR_INVALID, "the subsampling was created without a context");
  if (select_device(s->ctx)) return NRP_ERR_CUDA;
  int rc = sync_sub(s);
  if (rc) return rc;
  // forward_frames_chunked (conformer.rs:1344-1377): chunks of a multiple of
  // the factor, each run with `context` real neighbouring frames on either
  // side (twice the receptive field of the stacked stride-2 convs, rounded
  // up to the factor), its first left/factor output frames cropped; the
  // last chunk keeps every frame after the crop.
  const int factor = 1 << s->S;
  const int chunk = s->chunk_frames > 0 ? std::max(s->chunk_frames, factor) / factor * factor : 0;
  if (chunk == 0 || T <= chunk)
    return run_frames(s, st, mel, bs, ts, fs, B, T, lengths, 0, out);
  const int receptive = 1 + (3 - 1) * (factor - 1);
  const int context = (2 * receptive + factor - 1) / factor * factor;
  const int Tp_all = subsampling_output_frames(s, T);
  const size_t row = static_cast<size_t>(s->D) * 2;  // bytes per output frame
  const int piece_max = chunk + 2 * context;
  TRY_CUDA(s->chunk_out.ensure(static_cast<size_t>(B) * subsampling_output_frames(s, piece_max) *
                               row));
  int done = 0;  // output frames written per utterance
  for (int start = 0; start < T;) {
    const int end = std::min(start + chunk, T);
    const int left = std::min(context, start), right = std::min(context, T - end);
    const int p0 = start - left, n = end + right - p0;
    const int Tp = subsampling_output_frames(s, n);
    rc = run_frames(s, st, mel + p0 * ts, bs, ts, fs, B, n, lengths, p0, s->chunk_out.p);
    if (rc) return rc;
    const int first = left / factor;
    const int keep = end == T ? Tp - first : (end - start) / factor;
    if (keep < 0 || done + keep > Tp_all)
      return failf(NRP_ERR_UNSUPPORTED, "chunk plan: %d + %d frames of %d", done, keep, Tp_all);
    if (keep > 0) {
      ProfScope ps(s->ctx, NRP_KERNEL_ELEMENTWISE, st);
      TRY_CUDA(cudaMemcpy2DAsync(static_cast<uint8_t*>(out) + done * row, Tp_all * row,
                                 s->chunk_out.as<uint8_t>() + first * row, Tp * row, keep * row,
                                 B, cudaMemcpyDeviceToDevice, st));
    }
    done += keep;
    start = end;
  }
  if (done != Tp_all)
    return failf(NRP_ERR_UNSUPPORTED, "chunk plan wrote %d of %d frames", done, Tp_all);
  return NRP_OK;
}

}  // namespace nrp

extern "C" {

int nrp_subsampling_create(nrp_context* ctx, int feat_in, int d_model, int subsampling_factor,
                           int conv_channels, int causal, nrp_subsampling** out) {
  if (!out) return failf(NRP_ERR_INVALID, "null argument");
  *out = nullptr;
  if (feat_in <= 0 || d_model <= 0 || conv_channels <= 0)
    return failf(NRP_ERR_INVALID, "invalid subsampling configuration");
  if (conv_channels % 64 != 0 || conv_channels > 2048 || (conv_channels & (conv_channels - 1)))
    return failf(NRP_ERR_UNSUPPORTED, "conv_channels %d: a power of two in [64, 2048]",
                 conv_channels);
  if (d_model % 32 != 0) return failf(NRP_ERR_UNSUPPORTED, "d_model %d not a multiple of 32", d_model);
  auto* s = new nrp_subsampling;
  s->ctx = ctx;
  s->F = feat_in;
  s->D = d_model;
  s->factor = subsampling_factor;
  s->C = conv_channels;
  s->S = strides_of(subsampling_factor);
  s->causal = causal != 0;
  int f = feat_in;
  for (int i = 0; i < s->S; ++i) f = conv_len(f, s->causal);
  s->Fp = f;
  *out = s;
  return NRP_OK;
}

int nrp_subsampling_destroy(nrp_subsampling* s) {
  delete s;
  return NRP_OK;
}

int nrp_subsampling_set_dtype(nrp_subsampling* s, int dtype) {
  if (!s) return failf(NRP_ERR_INVALID, "null subsampling");
  if (dtype != NRP_DTYPE_BF16 && dtype != NRP_DTYPE_F32)
    return failf(NRP_ERR_INVALID, "dtype %d", dtype);
  s->dtype = dtype;
  s->dirty = true;
  return NRP_OK;
}

int nrp_subsampling_feat_out(const nrp_subsampling* s, int* feat_out) {
  if (!s || !feat_out) return failf(NRP_ERR_INVALID, "null argument");
  *feat_out = s->Fp;
  return NRP_OK;
}

int nrp_subsampling_output_length(const nrp_subsampling* s, int frames, int* out_frames) {
  if (!s || !out_frames) return failf(NRP_ERR_INVALID, "null argument");
  *out_frames = nrp::subsampling_output_frames(s, frames);
  return NRP_OK;
}

int nrp_subsampling_load_conv(nrp_subsampling* s, int index, const float* weight,
                              const float* bias) {
  if (!s || !weight) return failf(NRP_ERR_INVALID, "null argument");
  const int C = s->C;
  HostConv* dst = nullptr;
  size_t n = 0;
  if (index == 0) {
    dst = &s->conv[0];
    n = static_cast<size_t>(C) * 9;
  } else if (index >= 2 && (index - 2) % 3 == 0 && (index - 2) / 3 + 1 < s->S) {
    dst = &s->conv[(index - 2) / 3 + 1];
    n = static_cast<size_t>(C) * 9;
  } else if (index >= 3 && (index - 3) % 3 == 0 && (index - 3) / 3 + 1 < s->S) {
    dst = &s->pw[(index - 3) / 3];
    n = static_cast<size_t>(C) * C;
  } else {
    return failf(NRP_ERR_INVALID, "pre_encode.conv.%d is not a conv of this subsampling", index);
  }
  dst->loaded = true;
  dst->w.assign(weight, weight + n);
  if (bias)
    dst->b.assign(bias, bias + C);
  else
    dst->b.assign(C, 0.f);
  s->dirty = true;
  return NRP_OK;
}

int nrp_subsampling_load_out(nrp_subsampling* s, const float* weight, const float* bias) {
  if (!s || !weight) return failf(NRP_ERR_INVALID, "null argument");
  nrp::Linear& L = s->out;
  L = nrp::Linear();
  L.loaded = true;
  L.w.assign(weight, weight + static_cast<size_t>(s->D) * s->C * s->Fp);
  if (bias) L.bias.assign(bias, bias + s->D);
  s->dirty = true;
  return NRP_OK;
}

int nrp_subsampling_load_out_quantized(nrp_subsampling* s, int bits, int group_size,
                                       const uint32_t* wq, const float* scales,
                                       const float* biases, const float* bias) {
  if (!s || !wq || !scales || !biases) return failf(NRP_ERR_INVALID, "null argument");
  if (bits != 8 || group_size != 64)
    return failf(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
  const int K = s->C * s->Fp;
  if (K % 64) return failf(NRP_ERR_UNSUPPORTED, "in features %d not a multiple of 64", K);
  nrp::Linear& L = s->out;
  L = nrp::Linear();
  L.loaded = true;
  L.quant = true;
  L.bits = bits;
  L.group = group_size;
  L.wq.assign(wq, wq + static_cast<size_t>(s->D) * K / 4);
  // the module dtype's scales and biases (LinearLayer::cast)
  L.qs.resize(static_cast<size_t>(s->D) * (K / 64));
  L.qb.resize(L.qs.size());
  for (size_t i = 0; i < L.qs.size(); ++i) {
    L.qs[i] = nrp::bf16_round(scales[i]);
    L.qb[i] = nrp::bf16_round(biases[i]);
  }
  if (bias) L.bias.assign(bias, bias + s->D);
  s->dirty = true;
  return NRP_OK;
}

int nrp_subsampling_set_chunk_frames(nrp_subsampling* s, int frames) {
  if (!s) return failf(NRP_ERR_INVALID, "null subsampling");
  if (frames < 0) return failf(NRP_ERR_INVALID, "chunk frames %d < 0", frames);
  s->chunk_frames = frames;
  return NRP_OK;
}

int nrp_subsampling_forward(nrp_subsampling* s, void* stream, const float* features, int layout,
                            int batch, int frames, const int32_t* lengths, void* out) {
  if (!s || !features || !out) return failf(NRP_ERR_INVALID, "null argument");
  if (layout != NRP_FEATURES_BFT && layout != NRP_FEATURES_BTF)
    return failf(NRP_ERR_INVALID, "features layout %d", layout);
  const int64_t F = s->F, T = frames;
  const int64_t bs = F * T;
  const int64_t ts = layout == NRP_FEATURES_BFT ? 1 : F;
  const int64_t fs = layout == NRP_FEATURES_BFT ? T : 1;
  return nrp::subsampling_run(s, static_cast<cudaStream_t>(stream), features, bs, ts, fs, batch,
                              frames, lengths, out);
}

}  // extern "C"
