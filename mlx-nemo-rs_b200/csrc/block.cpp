// block.cpp -- the Conformer block and encoder around the rel-pos attention
// (src/asr/modules/encoders/conformer.rs:694-722, 1617-2437).
//
// One block forward, x updated in place in bf16 (M = batch * seq_len rows):
//   LayerNorm                       -> h
//   FF1 linear1, epilogue SiLU      -> hid
//   FF1 linear2, epilogue x += 0.5 * (.)
//   LayerNorm -> h; the attention with linear_out's epilogue x += (.)
//   LayerNorm -> h; pointwise_conv1, epilogue GLU + padded frames zeroed -> glu
//   depthwise conv + BatchNorm affine + SiLU -> dw
//   pointwise_conv2, epilogue x += (.)
//   LayerNorm -> h; FF2 as FF1; final LayerNorm in place
// With lengths, every per-frame GEMM tiles rows per utterance and skips the
// row tiles past each length (padded rows are unspecified, conformer.rs:
// 1590-1593), as the attention's own projections do.  pointwise_conv1's rows
// are uploaded permuted ([128 value rows | their 128 gate rows] per 256-row
// tile) so the GLU happens inside one output tile.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

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

constexpr int kNumLinears = 6;
constexpr int kNumNorms = 5;

struct DevLinear {
  nrp::DevBuf w, s, z, b;  // bf16 weight (or u8 codes), bf16 scales, zero points, bias
  bool quant = false, has_b = false;
};

cudaError_t upload_bf16(nrp::DevBuf& dst, const float* src, size_t n) {
  std::vector<uint16_t> h(n);
  for (size_t i = 0; i < n; ++i) h[i] = nrp::bf16_bits(src[i]);
  cudaError_t e = dst.ensure(n * 2);
  if (e == cudaSuccess) e = cudaMemcpy(dst.p, h.data(), n * 2, cudaMemcpyHostToDevice);
  return e;
}

cudaError_t upload_f32(nrp::DevBuf& dst, const std::vector<float>& v) {
  cudaError_t e = dst.ensure(v.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(dst.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
  return e;
}

// Row order of pointwise_conv1 on the device: tile k (256 rows) holds value
// rows 128k.. and gate rows D + 128k.. (GLU splits the 2D outputs in halves).
int glu_source_row(int n, int D) {
  const int k = n / 256, j = n % 256;
  return j < 128 ? 128 * k + j : D + 128 * k + (j - 128);
}

}  // namespace

struct nrp_block {
  nrp_context* ctx = nullptr;
  std::weak_ptr<bool> ctx_alive;  // (see nrp_context::alive)
  int D = 0, H = 0, ff = 0, K = 0;
  bool causal = false;
  int conv_norm = 0;  // 0 batch norm, 1 layer norm
  int use_bias = 1;
  int dtype = NRP_DTYPE_F32;
  nrp_attn* attn = nullptr;
  nrp::Linear lin[kNumLinears];
  std::vector<float> ng[kNumNorms], nb[kNumNorms];
  std::vector<float> dw_w, dw_b;            // [D][K], [D]
  std::vector<float> cn_g, cn_b, cn_m, cn_v;  // conv norm
  bool dirty = true;
  DevLinear dl[kNumLinears];
  nrp::DevBuf d_ng[kNumNorms], d_nb[kNumNorms];
  nrp::DevBuf d_dw_w;  // taps-major [K][D]
  nrp::DevBuf d_dw_b, d_cn_scale, d_cn_shift, d_cn_g, d_cn_b;
  nrp::DevBuf h, hid, glu, dw;  // workspace
  nrp::DevBuf vbuf;             // [B] copies of a streaming step's valid length
};

struct nrp_encoder {
  nrp_context* ctx = nullptr;
  int D = 0, H = 0, max_len = 5000;
  float xscale = 1.f;
  int dtype = NRP_DTYPE_F32;
  std::vector<nrp_block*> blocks;
  nrp::DevBuf x, pos;
  int pos_T = -1, pos_dtype = -1;
  // bf16 copies of the quantised weights of two layers: layer i + 1's are
  // dequantised on `dq` into slot (i + 1) % 2 while layer i runs
  cudaStream_t dq = nullptr;
  cudaEvent_t dq_start = nullptr, dq_ready[2] = {}, dq_done[2] = {};
  nrp::DevBuf dq_slot[2];
  // pre_encode (nrp_encoder_add_subsampling) and the device copy of one
  // forward's mel lengths and subsampled lengths [2][B]
  nrp_subsampling* sub = nullptr;
  nrp::DevBuf lens;
  std::vector<int32_t> lens_host;
  // forward_streaming: the subsampled chunk before the pre-encode frames
  // are dropped, and the positional table of cache + chunk frames
  nrp::DevBuf sx, spos;
  int spos_T = -1;
};

// EncoderCache on the device (streaming/core.rs:117-185): per layer the
// attention's ring (last_channel) and the conv cache [B][K-1][D] bf16
// (last_time, time-major), and the fill level the streams share
// (forward_streaming reads the first stream's, conformer.rs:853-857, 892).
struct nrp_encoder_cache {
  nrp_encoder* enc = nullptr;
  int B = 0, C = 0, K = 0, D = 0;
  int filled = 0;
  std::vector<nrp_cache*> attn;
  nrp::DevBuf conv;  // [layer][B][K-1][D]
};

namespace {

// Output and input sizes of each block linear.
void linear_shape(const nrp_block* k, int which, int& N, int& Kin) {
  switch (which) {
    case NRP_BLOCK_FF1_LINEAR1:
    case NRP_BLOCK_FF2_LINEAR1: N = k->ff; Kin = k->D; return;
    case NRP_BLOCK_FF1_LINEAR2:
    case NRP_BLOCK_FF2_LINEAR2: N = k->D; Kin = k->ff; return;
    case NRP_BLOCK_CONV_PW1: N = 2 * k->D; Kin = k->D; return;
    default: N = k->D; Kin = k->D; return;
  }
}

// Device copies of the block's parameters in bf16 (LinearLayer::cast and
// cast_module of ConformerBlock::set_dtype, conformer.rs:1639-1659: every
// parameter rounded to bf16; the BatchNorm is then folded to
// scale = gamma / sqrt(var + eps), shift = beta - mean * scale).
int sync_block(nrp_block* k) {
  if (!k->dirty) return NRP_OK;
  const int D = k->D;
  for (int i = 0; i < kNumLinears; ++i) {
    const nrp::Linear& L = k->lin[i];
    if (!L.loaded) return failf(NRP_ERR_INVALID, "block linear %d has no weights loaded", i);
    int N, Kin;
    linear_shape(k, i, N, Kin);
    const bool glu = i == NRP_BLOCK_CONV_PW1;
    auto src_row = [&](int n) { return glu ? glu_source_row(n, D) : n; };
    DevLinear& d = k->dl[i];
    nrp::deq_forget(k->ctx, d.w.p);  // the codes are replaced
    d.quant = L.quant;
    if (L.quant) {
      if (L.bits != 8 || L.group != 64)
        return failf(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
      const int kg = Kin / 64;
      std::vector<uint8_t> codes(static_cast<size_t>(N) * Kin);
      std::vector<float> sc(static_cast<size_t>(N) * kg), zp(static_cast<size_t>(N) * kg);
      const uint8_t* wb = reinterpret_cast<const uint8_t*>(L.wq.data());
      for (int n = 0; n < N; ++n) {
        const int r = src_row(n);
        memcpy(codes.data() + static_cast<size_t>(n) * Kin, wb + static_cast<size_t>(r) * Kin, Kin);
        memcpy(sc.data() + static_cast<size_t>(n) * kg, L.qs.data() + static_cast<size_t>(r) * kg,
               sizeof(float) * kg);
        memcpy(zp.data() + static_cast<size_t>(n) * kg, L.qb.data() + static_cast<size_t>(r) * kg,
               sizeof(float) * kg);
      }
      TRY_CUDA(d.w.ensure(codes.size()));
      TRY_CUDA(cudaMemcpy(d.w.p, codes.data(), codes.size(), cudaMemcpyHostToDevice));
      TRY_CUDA(upload_bf16(d.s, sc.data(), sc.size()));
      TRY_CUDA(upload_bf16(d.z, zp.data(), zp.size()));
    } else {
      std::vector<float> w(static_cast<size_t>(N) * Kin);
      for (int n = 0; n < N; ++n)
        memcpy(w.data() + static_cast<size_t>(n) * Kin, L.w.data() + static_cast<size_t>(src_row(n)) * Kin,
               sizeof(float) * Kin);
      TRY_CUDA(upload_bf16(d.w, w.data(), w.size()));
    }
    d.has_b = !L.bias.empty();
    if (d.has_b) {
      std::vector<float> b(N);
      for (int n = 0; n < N; ++n) b[n] = L.bias[src_row(n)];
      TRY_CUDA(upload_bf16(d.b, b.data(), b.size()));
    }
  }
  auto rounded = [](const std::vector<float>& v) {
    std::vector<float> r(v.size());
    for (size_t i = 0; i < v.size(); ++i) r[i] = nrp::bf16_round(v[i]);
    return r;
  };
  for (int i = 0; i < kNumNorms; ++i) {
    TRY_CUDA(upload_f32(k->d_ng[i], rounded(k->ng[i])));
    TRY_CUDA(upload_f32(k->d_nb[i], rounded(k->nb[i])));
  }
  // depthwise weight: MLX [D, K, 1] == [D][K]
  {  // taps-major [K][D] on the device
    std::vector<float> wt(static_cast<size_t>(k->K) * D);
    for (int c = 0; c < D; ++c)
      for (int j = 0; j < k->K; ++j)
        wt[static_cast<size_t>(j) * D + c] = nrp::bf16_round(k->dw_w[static_cast<size_t>(c) * k->K + j]);
    TRY_CUDA(upload_f32(k->d_dw_w, wt));
  }
  if (!k->dw_b.empty()) TRY_CUDA(upload_f32(k->d_dw_b, rounded(k->dw_b)));
  if (k->conv_norm == 0) {
    std::vector<float> scale(D), shift(D);
    const float eps = nrp::bf16_round(1e-5f);
    for (int c = 0; c < D; ++c) {
      const float g = nrp::bf16_round(k->cn_g[c]), b = nrp::bf16_round(k->cn_b[c]);
      const float m = nrp::bf16_round(k->cn_m[c]), v = nrp::bf16_round(k->cn_v[c]);
      scale[c] = g / sqrtf(v + eps);
      shift[c] = b - m * scale[c];
    }
    TRY_CUDA(upload_f32(k->d_cn_scale, scale));
    TRY_CUDA(upload_f32(k->d_cn_shift, shift));
  } else {
    TRY_CUDA(upload_f32(k->d_cn_g, rounded(k->cn_g)));
    TRY_CUDA(upload_f32(k->d_cn_b, rounded(k->cn_b)));
  }
  k->dirty = false;
  return NRP_OK;
}

// A quantised weight of a layer: codes, scales, zero points, [N, K].
struct QuantWeight {
  const void* wq;
  const void* qs;
  const void* qb;
  int N, K;
};

// Rows (batch x frames) from which the encoder dequantises a layer's weights
// ahead of it: the linears dequantise whole weights from 256 rows on.
constexpr int64_t kPrefetchMinRows = 256;

// The quantised weights of a synced block, its attention's included.
void quant_weights(const nrp_block* k, std::vector<QuantWeight>& out) {
  for (int i = 0; i < kNumLinears; ++i) {
    const DevLinear& d = k->dl[i];
    if (!d.quant) continue;
    int N, Kin;
    linear_shape(k, i, N, Kin);
    out.push_back({d.w.p, d.s.p, d.z.p, N, Kin});
  }
  const nrp_attn* a = k->attn;
  if (a->qkv_quant) out.push_back({a->w_qkv.p, a->s_qkv.p, a->z_qkv.p, 3 * a->D, a->D});
  if (a->pos_quant) out.push_back({a->w_pos.p, a->s_pos.p, a->z_pos.p, a->D, a->D});
  if (a->out_quant) out.push_back({a->w_out.p, a->s_out.p, a->z_out.p, a->D, a->D});
}

int block_linear(nrp_block* k, cudaStream_t st, int which, const void* x, int M, void* y,
                 int ldy, const nrp::RowTiling& rt, const nrp::Epilogue& ep) {
  int N, Kin;
  linear_shape(k, which, N, Kin);
  const DevLinear& d = k->dl[which];
  return nrp::linear(k->ctx, st, NRP_DTYPE_BF16, x, M, Kin, d.w.p, d.quant, d.s.p, d.z.p, N,
                     d.has_b ? d.b.p : nullptr, y, ldy, rt, ep, true);
}

int layer_norm(nrp_block* k, cudaStream_t st, int which, const void* x, void* y, int64_t rows) {
  nrp::ProfScope ps(k->ctx, NRP_KERNEL_LAYERNORM, st);
  TRY_CUDA(nrp::launch_layernorm(static_cast<const __nv_bfloat16*>(x), k->d_ng[which].as<float>(),
                                 k->d_nb[which].as<float>(), static_cast<__nv_bfloat16*>(y), rows,
                                 k->D, 1e-5f, false, st));
  return NRP_OK;
}

}  // namespace

extern "C" {

int nrp_block_create(nrp_context* ctx, int d_model, int n_heads, int ff_dim, int conv_kernel,
                     int causal_conv, int conv_norm, int use_bias, nrp_block** out) {
  if (!ctx || !out) return failf(NRP_ERR_INVALID, "null argument");
  *out = nullptr;
  if (d_model <= 0 || n_heads <= 0 || d_model % n_heads || ff_dim <= 0 || conv_kernel <= 0 ||
      (conv_norm != 0 && conv_norm != 1))
    return failf(NRP_ERR_INVALID, "invalid block configuration");
  // a symmetric ("same") padding keeps T frames only for an odd kernel
  if (!causal_conv && conv_kernel % 2 == 0)
    return failf(NRP_ERR_UNSUPPORTED, "non-causal conv needs an odd kernel (%d)", conv_kernel);
  auto* k = new nrp_block;
  k->ctx = ctx;
  k->ctx_alive = ctx->alive;
  k->D = d_model;
  k->H = n_heads;
  k->ff = ff_dim;
  k->K = conv_kernel;
  k->causal = causal_conv != 0;
  k->conv_norm = conv_norm;
  k->use_bias = use_bias;
  int rc = nrp_attn_create(ctx, d_model, n_heads, use_bias, &k->attn);
  if (rc) {
    delete k;
    return rc;
  }
  // nn::LayerNorm::new / BatchNorm::new defaults: weight 1, bias 0, running
  // mean 0, running var 1; the linears start as zeros with biases
  // (FeedForward::new 2046-2063, ConvolutionModule::new 2137-2196).
  for (int i = 0; i < kNumNorms; ++i) {
    k->ng[i].assign(d_model, 1.f);
    k->nb[i].assign(d_model, 0.f);
  }
  k->cn_g.assign(d_model, 1.f);
  k->cn_b.assign(d_model, 0.f);
  k->cn_m.assign(d_model, 0.f);
  k->cn_v.assign(d_model, 1.f);
  k->dw_w.assign(static_cast<size_t>(d_model) * conv_kernel, 0.f);
  if (use_bias) k->dw_b.assign(d_model, 0.f);
  for (int i = 0; i < kNumLinears; ++i) {
    int N, Kin;
    linear_shape(k, i, N, Kin);
    nrp::Linear& L = k->lin[i];
    L.loaded = true;
    L.w.assign(static_cast<size_t>(N) * Kin, 0.f);
    const bool conv = i == NRP_BLOCK_CONV_PW1 || i == NRP_BLOCK_CONV_PW2;
    if (use_bias || conv) L.bias.assign(N, 0.f);
  }
  *out = k;
  return NRP_OK;
}

int nrp_block_destroy(nrp_block* k) {
  if (!k) return NRP_OK;
  if (!k->ctx_alive.expired())
    for (const DevLinear& d : k->dl) nrp::deq_forget(k->ctx, d.w.p);
  nrp_attn_destroy(k->attn);
  delete k;
  return NRP_OK;
}

int nrp_block_set_dtype(nrp_block* k, int dtype) {
  if (!k) return failf(NRP_ERR_INVALID, "null block");
  if (dtype != NRP_DTYPE_F32 && dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_INVALID, "dtype %d", dtype);
  k->dtype = dtype;
  k->dirty = true;
  return nrp_attn_set_dtype(k->attn, dtype);
}

int nrp_block_attn(nrp_block* k, nrp_attn** attn) {
  if (!k || !attn) return failf(NRP_ERR_INVALID, "null argument");
  *attn = k->attn;
  return NRP_OK;
}

int nrp_block_load_linear(nrp_block* k, int which, const float* w, const float* bias) {
  if (!k || !w) return failf(NRP_ERR_INVALID, "null argument");
  if (which < 0 || which >= kNumLinears) return failf(NRP_ERR_INVALID, "linear %d", which);
  int N, Kin;
  linear_shape(k, which, N, Kin);
  nrp::Linear& L = k->lin[which];
  L = nrp::Linear();
  L.loaded = true;
  L.w.assign(w, w + static_cast<size_t>(N) * Kin);
  if (bias) L.bias.assign(bias, bias + N);
  k->dirty = true;
  return NRP_OK;
}

int nrp_block_load_linear_quantized(nrp_block* k, int which, int bits, int group_size,
                                    const uint32_t* wq, const float* scales,
                                    const float* biases, const float* bias) {
  if (!k || !wq || !scales || !biases) return failf(NRP_ERR_INVALID, "null argument");
  if (which < 0 || which >= kNumLinears) return failf(NRP_ERR_INVALID, "linear %d", which);
  if (bits != 8 || group_size != 64)
    return failf(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
  int N, Kin;
  linear_shape(k, which, N, Kin);
  if (Kin % 64) return failf(NRP_ERR_UNSUPPORTED, "in features %d not a multiple of 64", Kin);
  nrp::Linear& L = k->lin[which];
  L = nrp::Linear();
  L.loaded = true;
  L.quant = true;
  L.bits = bits;
  L.group = group_size;
  L.wq.assign(wq, wq + static_cast<size_t>(N) * Kin / 4);
  L.qs.assign(scales, scales + static_cast<size_t>(N) * (Kin / 64));
  L.qb.assign(biases, biases + static_cast<size_t>(N) * (Kin / 64));
  if (bias) L.bias.assign(bias, bias + N);
  k->dirty = true;
  return NRP_OK;
}

int nrp_block_load_norm(nrp_block* k, int which, const float* gamma, const float* beta) {
  if (!k || !gamma || !beta) return failf(NRP_ERR_INVALID, "null argument");
  if (which < 0 || which >= kNumNorms) return failf(NRP_ERR_INVALID, "norm %d", which);
  k->ng[which].assign(gamma, gamma + k->D);
  k->nb[which].assign(beta, beta + k->D);
  k->dirty = true;
  return NRP_OK;
}

int nrp_block_load_depthwise(nrp_block* k, const float* w, const float* bias) {
  if (!k || !w) return failf(NRP_ERR_INVALID, "null argument");
  k->dw_w.assign(w, w + static_cast<size_t>(k->D) * k->K);
  if (bias) k->dw_b.assign(bias, bias + k->D);
  else k->dw_b.clear();
  k->dirty = true;
  return NRP_OK;
}

int nrp_block_load_conv_norm(nrp_block* k, const float* gamma, const float* beta,
                             const float* mean, const float* var) {
  if (!k || !gamma || !beta) return failf(NRP_ERR_INVALID, "null argument");
  k->cn_g.assign(gamma, gamma + k->D);
  k->cn_b.assign(beta, beta + k->D);
  if (k->conv_norm == 0) {
    if (!mean || !var) return failf(NRP_ERR_INVALID, "batch norm needs running statistics");
    k->cn_m.assign(mean, mean + k->D);
    k->cn_v.assign(var, var + k->D);
  }
  k->dirty = true;
  return NRP_OK;
}

int nrp_block_forward(nrp_block* k, void* stream, const void* x, int B, int T,
                      const void* pos_emb, const int32_t* lengths,
                      const nrp_att_context* context, void* out) {
  if (!k || !x || !pos_emb || !out) return failf(NRP_ERR_INVALID, "null argument");
  if (B <= 0 || T <= 0) return failf(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  if (k->dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_UNSUPPORTED, "the conformer block runs in bf16 (nrp_block_set_dtype)");
  const int D = k->D;
  if (D != 256 && D != 512 && D != 1024 && D != 2048)
    return failf(NRP_ERR_UNSUPPORTED, "d_model %d (the block needs 256, 512, 1024 or 2048)", D);
  if (k->ff % 64) return failf(NRP_ERR_UNSUPPORTED, "ff_dim %d not a multiple of 64", k->ff);
  // padded frames are zeroed by the GEMMs' per-utterance row tiling
  if (lengths && B > 256)
    return failf(NRP_ERR_UNSUPPORTED, "the block with lengths supports batch <= 256");
  if (nrp::select_device(k->ctx)) return NRP_ERR_CUDA;
  int rc = sync_block(k);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t M = static_cast<int64_t>(B) * T;
  if (M > INT32_MAX / 4) return failf(NRP_ERR_UNSUPPORTED, "batch x seq_len too large");
  const int Mi = static_cast<int>(M);
  TRY_CUDA(k->h.ensure(M * D * 2));
  TRY_CUDA(k->hid.ensure(M * k->ff * 2));
  TRY_CUDA(k->glu.ensure(M * D * 2));
  TRY_CUDA(k->dw.ensure(M * D * 2));
  if (out != x) {
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(cudaMemcpyAsync(out, x, M * D * 2, cudaMemcpyDeviceToDevice, st));
  }
  nrp::RowTiling rows;
  if (lengths && B <= 256) rows = {lengths, T, B};
  auto residual = [&](float alpha) {
    nrp::Epilogue e;
    e.mode = nrp::kEpiResidual;
    e.res = static_cast<const __nv_bfloat16*>(out);
    e.ldr = D;
    e.alpha = alpha;
    return e;
  };
  nrp::Epilogue silu;
  silu.mode = nrp::kEpiSilu;
  auto feed_forward = [&](int norm, int l1, int l2) -> int {
    int r = layer_norm(k, st, norm, out, k->h.p, M);
    if (!r) r = block_linear(k, st, l1, k->h.p, Mi, k->hid.p, k->ff, rows, silu);
    if (!r) r = block_linear(k, st, l2, k->hid.p, Mi, out, D, rows, residual(0.5f));
    return r;
  };
  // 1703-1733: x += 0.5 * FF1(LN x)
  rc = feed_forward(NRP_BLOCK_NORM_FF1, NRP_BLOCK_FF1_LINEAR1, NRP_BLOCK_FF1_LINEAR2);
  if (rc) return rc;
  // 1750-1785: x += MHA(LN x)
  rc = layer_norm(k, st, NRP_BLOCK_NORM_ATT, out, k->h.p, M);
  if (rc) return rc;
  rc = nrp::attn_forward(k->attn, st, k->h.p, B, T, pos_emb, lengths, context, out, residual(1.f));
  if (rc) return rc;
  // 1797-1824, 2249-2330: x += Conv(LN x)
  rc = layer_norm(k, st, NRP_BLOCK_NORM_CONV, out, k->h.p, M);
  if (rc) return rc;
  nrp::Epilogue glu;
  glu.mode = nrp::kEpiGlu;
  glu.len = rows.len;
  rc = block_linear(k, st, NRP_BLOCK_CONV_PW1, k->h.p, Mi, k->glu.p, D, rows, glu);
  if (rc) return rc;
  {
    const bool bn = k->conv_norm == 0;
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_DWCONV, st);
    TRY_CUDA(nrp::launch_dwconv(k->glu.as<__nv_bfloat16>(), k->d_dw_w.as<float>(),
                                k->dw_b.empty() ? nullptr : k->d_dw_b.as<float>(),
                                bn ? k->d_cn_scale.as<float>() : nullptr,
                                bn ? k->d_cn_shift.as<float>() : nullptr,
                                k->dw.as<__nv_bfloat16>(), B, T, D, k->K, k->causal, bn, st));
  }
  if (k->conv_norm == 1) {  // LayerNorm conv norm, then SiLU
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_LAYERNORM, st);
    TRY_CUDA(nrp::launch_layernorm(k->dw.as<__nv_bfloat16>(), k->d_cn_g.as<float>(),
                                   k->d_cn_b.as<float>(), k->dw.as<__nv_bfloat16>(), M, D, 1e-5f,
                                   true, st));
  }
  rc = block_linear(k, st, NRP_BLOCK_CONV_PW2, k->dw.p, Mi, out, D, rows, residual(1.f));
  if (rc) return rc;
  // 1826-1858: x += 0.5 * FF2(LN x)
  rc = feed_forward(NRP_BLOCK_NORM_FF2, NRP_BLOCK_FF2_LINEAR1, NRP_BLOCK_FF2_LINEAR2);
  if (rc) return rc;
  // 1861: final LayerNorm
  return layer_norm(k, st, NRP_BLOCK_NORM_OUT, out, out, M);
}

int nrp_block_forward_with_cache(nrp_block* k, void* stream, const void* x, int B, int T,
                                 const void* pos_emb, nrp_cache* attn_cache, void* conv_cache,
                                 int filled, int valid, const nrp_att_context* context,
                                 void* out) {
  if (!k || !x || !pos_emb || !attn_cache || !out) return failf(NRP_ERR_INVALID, "null argument");
  if (k->K > 1 && !conv_cache) return failf(NRP_ERR_INVALID, "null conv cache");
  if (B <= 0 || T <= 0) return failf(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  if (k->dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_UNSUPPORTED, "the conformer block runs in bf16 (nrp_block_set_dtype)");
  const int D = k->D, K = k->K;
  if (D != 256 && D != 512 && D != 1024 && D != 2048)
    return failf(NRP_ERR_UNSUPPORTED, "d_model %d (the block needs 256, 512, 1024 or 2048)", D);
  if (k->ff % 64) return failf(NRP_ERR_UNSUPPORTED, "ff_dim %d not a multiple of 64", k->ff);
  if (B > 256) return failf(NRP_ERR_UNSUPPORTED, "the streaming block supports batch <= 256");
  if (nrp::select_device(k->ctx)) return NRP_ERR_CUDA;
  int rc = sync_block(k);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t M = static_cast<int64_t>(B) * T;
  const int Tc = K - 1 + T;  // the conv cache, then the chunk
  const int64_t Mc = static_cast<int64_t>(B) * Tc;
  if (Mc > INT32_MAX / 4) return failf(NRP_ERR_UNSUPPORTED, "batch x seq_len too large");
  const int Mi = static_cast<int>(M);
  valid = std::min(std::max(valid, 0), T);
  TRY_CUDA(k->h.ensure(M * D * 2));
  TRY_CUDA(k->hid.ensure(M * k->ff * 2));
  TRY_CUDA(k->glu.ensure(Mc * D * 2));
  TRY_CUDA(k->dw.ensure(Mc * D * 2));
  TRY_CUDA(k->vbuf.ensure(static_cast<size_t>(B) * 4));
  if (out != x) {
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(cudaMemcpyAsync(out, x, M * D * 2, cudaMemcpyDeviceToDevice, st));
  }
  auto residual = [&](float alpha) {
    nrp::Epilogue e;
    e.mode = nrp::kEpiResidual;
    e.res = static_cast<const __nv_bfloat16*>(out);
    e.ldr = D;
    e.alpha = alpha;
    return e;
  };
  nrp::Epilogue silu;
  silu.mode = nrp::kEpiSilu;
  const nrp::RowTiling flat;
  auto feed_forward = [&](int norm, int l1, int l2) -> int {
    int r = layer_norm(k, st, norm, out, k->h.p, M);
    if (!r) r = block_linear(k, st, l1, k->h.p, Mi, k->hid.p, k->ff, flat, silu);
    if (!r) r = block_linear(k, st, l2, k->hid.p, Mi, out, D, flat, residual(0.5f));
    return r;
  };
  // 1916-1923: x += 0.5 * FF1(LN x)
  rc = feed_forward(NRP_BLOCK_NORM_FF1, NRP_BLOCK_FF1_LINEAR1, NRP_BLOCK_FF1_LINEAR2);
  if (rc) return rc;
  // 1925-1935: x += MHA(LN x) against the attention cache
  rc = layer_norm(k, st, NRP_BLOCK_NORM_ATT, out, k->h.p, M);
  if (rc) return rc;
  rc = nrp::attn_forward_with_cache(k->attn, st, k->h.p, B, T, pos_emb, attn_cache, filled, valid,
                                    context, out, residual(1.f));
  if (rc) return rc;
  // 1943-1948, 2332-2400: x += Conv(LN x) with the conv cache.  The GLU
  // output of the chunk goes after each utterance's K-1 cached frames
  // (frames >= valid zeroed: the pad mask, 929-941); the depthwise conv runs
  // over [cache | chunk] and its last T outputs feed pointwise_conv2; the
  // new cache is the last K-1 frames of [cache | chunk].
  rc = layer_norm(k, st, NRP_BLOCK_NORM_CONV, out, k->h.p, M);
  if (rc) return rc;
  auto* glu = k->glu.as<__nv_bfloat16>();
  {
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(nrp::launch_fill_i32(k->vbuf.as<int32_t>(), valid, B, st));
  }
  nrp::RowTiling grows;
  grows.len = k->vbuf.as<int32_t>();
  grows.T = T;
  grows.B = B;
  grows.y_bstride = static_cast<int64_t>(Tc) * D;
  nrp::Epilogue gl;
  gl.mode = nrp::kEpiGlu;
  gl.len = grows.len;
  rc = block_linear(k, st, NRP_BLOCK_CONV_PW1, k->h.p, Mi, glu + static_cast<size_t>(K - 1) * D, D,
                    grows, gl);
  if (rc) return rc;
  if (K > 1) {
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_ELEMENTWISE, st);
    const size_t row = static_cast<size_t>(D) * 2;
    TRY_CUDA(cudaMemcpy2DAsync(glu, Tc * row, conv_cache, (K - 1) * row, (K - 1) * row, B,
                               cudaMemcpyDeviceToDevice, st));
    TRY_CUDA(cudaMemcpy2DAsync(conv_cache, (K - 1) * row, glu + static_cast<size_t>(T) * D, Tc * row,
                               (K - 1) * row, B, cudaMemcpyDeviceToDevice, st));
  }
  {
    const bool bn = k->conv_norm == 0;
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_DWCONV, st);
    // causal over the Tc rows: output row K-1+t reads rows t .. t+K-1 only
    TRY_CUDA(nrp::launch_dwconv(glu, k->d_dw_w.as<float>(),
                                k->dw_b.empty() ? nullptr : k->d_dw_b.as<float>(),
                                bn ? k->d_cn_scale.as<float>() : nullptr,
                                bn ? k->d_cn_shift.as<float>() : nullptr,
                                k->dw.as<__nv_bfloat16>(), B, Tc, D, K, true, bn, st));
  }
  if (k->conv_norm == 1) {
    nrp::ProfScope ps(k->ctx, NRP_KERNEL_LAYERNORM, st);
    TRY_CUDA(nrp::launch_layernorm(k->dw.as<__nv_bfloat16>(), k->d_cn_g.as<float>(),
                                   k->d_cn_b.as<float>(), k->dw.as<__nv_bfloat16>(), Mc, D, 1e-5f,
                                   true, st));
  }
  nrp::RowTiling drows;
  drows.T = T;
  drows.B = B;
  drows.x_bstride = static_cast<int64_t>(Tc) * D;
  rc = block_linear(k, st, NRP_BLOCK_CONV_PW2,
                    k->dw.as<__nv_bfloat16>() + static_cast<size_t>(K - 1) * D, Mi, out, D, drows,
                    residual(1.f));
  if (rc) return rc;
  // 1952-1958: x += 0.5 * FF2(LN x)
  rc = feed_forward(NRP_BLOCK_NORM_FF2, NRP_BLOCK_FF2_LINEAR1, NRP_BLOCK_FF2_LINEAR2);
  if (rc) return rc;
  // 1961: final LayerNorm
  return layer_norm(k, st, NRP_BLOCK_NORM_OUT, out, out, M);
}

// ---------------------------------------------------------------- encoder
int nrp_encoder_create(nrp_context* ctx, int n_layers, int d_model, int n_heads, int ff_dim,
                       int conv_kernel, int causal_conv, int conv_norm, int use_bias,
                       int xscaling, int max_len, nrp_encoder** out) {
  if (!ctx || !out) return failf(NRP_ERR_INVALID, "null argument");
  *out = nullptr;
  if (n_layers <= 0 || max_len <= 0) return failf(NRP_ERR_INVALID, "invalid encoder configuration");
  auto* e = new nrp_encoder;
  e->ctx = ctx;
  e->D = d_model;
  e->H = n_heads;
  e->max_len = max_len;
  e->xscale = nrp_pe_xscale(d_model, xscaling);
  for (int i = 0; i < n_layers; ++i) {
    nrp_block* b = nullptr;
    const int rc = nrp_block_create(ctx, d_model, n_heads, ff_dim, conv_kernel, causal_conv,
                                    conv_norm, use_bias, &b);
    if (rc) {
      nrp_encoder_destroy(e);
      return rc;
    }
    e->blocks.push_back(b);
  }
  *out = e;
  return NRP_OK;
}

int nrp_encoder_destroy(nrp_encoder* e) {
  if (!e) return NRP_OK;
  if (e->dq) {
    cudaStreamSynchronize(e->dq);
    cudaStreamDestroy(e->dq);
  }
  for (cudaEvent_t ev : {e->dq_start, e->dq_ready[0], e->dq_ready[1], e->dq_done[0], e->dq_done[1]})
    if (ev) cudaEventDestroy(ev);
  for (nrp_block* b : e->blocks) nrp_block_destroy(b);
  nrp_subsampling_destroy(e->sub);
  delete e;
  (void)cudaGetLastError();
  return NRP_OK;
}

int nrp_encoder_cache_create(nrp_encoder* e, int batch, int cache_len, nrp_encoder_cache** out) {
  if (!e || !out) return failf(NRP_ERR_INVALID, "null argument");
  *out = nullptr;
  if (batch <= 0 || cache_len <= 0) return failf(NRP_ERR_INVALID, "invalid cache arguments");
  if (e->dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_UNSUPPORTED, "set the encoder's dtype (bf16) before making its cache");
  if (nrp::select_device(e->ctx)) return NRP_ERR_CUDA;
  auto* c = new nrp_encoder_cache;
  c->enc = e;
  c->B = batch;
  c->C = cache_len;
  c->K = e->blocks.empty() ? 1 : e->blocks[0]->K;
  c->D = e->D;
  for (nrp_block* b : e->blocks) {
    nrp_cache* ac = nullptr;
    const int rc = nrp_cache_create(b->attn, batch, cache_len, &ac);
    if (rc) {
      nrp_encoder_cache_destroy(c);
      return rc;
    }
    c->attn.push_back(ac);
  }
  const size_t bytes = e->blocks.size() * static_cast<size_t>(batch) * (c->K - 1) * c->D * 2;
  if (c->conv.ensure(bytes) != cudaSuccess || cudaMemset(c->conv.p, 0, bytes ? bytes : 16)) {
    (void)cudaGetLastError();
    nrp_encoder_cache_destroy(c);
    return failf(NRP_ERR_NOMEM, "encoder cache allocation failed");
  }
  *out = c;
  return NRP_OK;
}

int nrp_encoder_cache_destroy(nrp_encoder_cache* c) {
  if (!c) return NRP_OK;
  for (nrp_cache* a : c->attn) nrp_cache_destroy(a);
  delete c;
  (void)cudaGetLastError();
  return NRP_OK;
}

int nrp_encoder_cache_reset(nrp_encoder_cache* c, void* stream) {
  if (!c) return failf(NRP_ERR_INVALID, "null cache");
  for (nrp_cache* a : c->attn) {
    const int rc = nrp_cache_reset(a, stream);
    if (rc) return rc;
  }
  if (c->conv.bytes)
    TRY_CUDA(cudaMemsetAsync(c->conv.p, 0, c->conv.bytes, static_cast<cudaStream_t>(stream)));
  c->filled = 0;
  return NRP_OK;
}

int nrp_encoder_cache_get_filled(const nrp_encoder_cache* c, int* filled) {
  if (!c || !filled) return failf(NRP_ERR_INVALID, "null argument");
  *filled = c->filled;
  return NRP_OK;
}

int nrp_encoder_cache_set_filled(nrp_encoder_cache* c, int filled) {
  if (!c) return failf(NRP_ERR_INVALID, "null cache");
  c->filled = std::min(std::max(filled, 0), c->C);
  return NRP_OK;
}

int nrp_encoder_cache_layer(nrp_encoder_cache* c, int layer, nrp_cache** attn_cache,
                            void** conv_cache) {
  if (!c) return failf(NRP_ERR_INVALID, "null cache");
  if (layer < 0 || layer >= static_cast<int>(c->attn.size()))
    return failf(NRP_ERR_INVALID, "layer %d of %d", layer, static_cast<int>(c->attn.size()));
  if (attn_cache) *attn_cache = c->attn[layer];
  if (conv_cache)
    *conv_cache = c->conv.as<__nv_bfloat16>() +
                  static_cast<size_t>(layer) * c->B * (c->K - 1) * c->D;
  return NRP_OK;
}

int nrp_encoder_cache_copy_conv(nrp_encoder_cache* c, int layer, void* data, int to_cache,
                                void* stream) {
  if (!c || !data) return failf(NRP_ERR_INVALID, "null argument");
  void* conv = nullptr;
  const int rc = nrp_encoder_cache_layer(c, layer, nullptr, &conv);
  if (rc) return rc;
  const size_t bytes = static_cast<size_t>(c->B) * (c->K - 1) * c->D * 2;
  if (bytes)
    TRY_CUDA(cudaMemcpyAsync(to_cache ? conv : data, to_cache ? data : conv, bytes,
                             cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
  return NRP_OK;
}

int nrp_encoder_block(nrp_encoder* e, int layer, nrp_block** block) {
  if (!e || !block) return failf(NRP_ERR_INVALID, "null argument");
  if (layer < 0 || layer >= static_cast<int>(e->blocks.size()))
    return failf(NRP_ERR_INVALID, "layer %d of %d", layer, static_cast<int>(e->blocks.size()));
  *block = e->blocks[layer];
  return NRP_OK;
}

int nrp_encoder_set_dtype(nrp_encoder* e, int dtype) {
  if (!e) return failf(NRP_ERR_INVALID, "null encoder");
  for (nrp_block* b : e->blocks) {
    const int rc = nrp_block_set_dtype(b, dtype);
    if (rc) return rc;
  }
  if (e->sub) {
    const int rc = nrp_subsampling_set_dtype(e->sub, dtype);
    if (rc) return rc;
  }
  e->dtype = dtype;
  return NRP_OK;
}

int nrp_encoder_add_subsampling(nrp_encoder* e, int feat_in, int subsampling_factor,
                                int conv_channels, int causal_downsampling,
                                nrp_subsampling** sub) {
  if (!e) return failf(NRP_ERR_INVALID, "null encoder");
  if (e->sub) return failf(NRP_ERR_INVALID, "the encoder already has a subsampling");
  nrp_subsampling* s = nullptr;
  int rc = nrp_subsampling_create(e->ctx, feat_in, e->D, subsampling_factor, conv_channels,
                                  causal_downsampling, &s);
  if (!rc) rc = nrp_subsampling_set_dtype(s, e->dtype);
  if (rc) {
    nrp_subsampling_destroy(s);
    return rc;
  }
  e->sub = s;
  if (sub) *sub = s;
  return NRP_OK;
}

}  // extern "C"

namespace {

// x * xscale, the blocks and the transpose to [B, D, T] over the embeddings
// in e->x (conformer.rs:530-557 and 694-722).
int encoder_layers(nrp_encoder* e, void* stream, int B, int T, const int32_t* lengths,
                   const nrp_att_context* context, void* out) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = e->D;
  const int64_t n = static_cast<int64_t>(B) * T * D;
  // 707-708: the positional table for this length (built once per length;
  // nrp_pe_encoding stages it through the host)
  if (e->pos_T != T) {
    TRY_CUDA(e->pos.ensure(static_cast<size_t>(2 * T - 1) * D * 2));
    const int rc = nrp_pe_encoding(e->ctx, D, e->max_len, T, NRP_DTYPE_BF16, e->pos.p, stream);
    if (rc) return rc;
    e->pos_T = T;
  }
  // 701-704: x * xscale
  if (e->xscale != 1.f) {
    nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(nrp::launch_scale(e->x.as<__nv_bfloat16>(), n, nrp::bf16_round(e->xscale), st));
  }
  // Quantised layers: the next layer's weights are dequantised on e->dq
  // while the current layer runs (every forward still dequantises every
  // weight; only the order of the work changes).  Not worth a stream below
  // the rows from which the linears dequantise whole weights anyway.
  const int L = static_cast<int>(e->blocks.size());
  std::vector<std::vector<QuantWeight>> qw(L);
  size_t slot_bytes = 0;
  // (with the context's kept bf16 copies, the linears dequantise nothing after
  // the first forward: nothing to prefetch)
  if (n / D >= kPrefetchMinRows && !e->ctx->deq_cache_on) {
    for (int i = 0; i < L; ++i) {
      int rc = sync_block(e->blocks[i]);
      if (!rc) rc = nrp::attn_sync(e->blocks[i]->attn);
      if (rc) return rc;
      size_t bytes = 0;
      quant_weights(e->blocks[i], qw[i]);
      for (const QuantWeight& q : qw[i]) bytes += static_cast<size_t>(q.N) * q.K * 2;
      slot_bytes = std::max(slot_bytes, bytes);
    }
  }
  const bool pre = slot_bytes > 0;
  if (pre) {
    if (!e->dq) {
      TRY_CUDA(cudaStreamCreateWithFlags(&e->dq, cudaStreamNonBlocking));
      for (cudaEvent_t* ev : {&e->dq_start, &e->dq_ready[0], &e->dq_ready[1], &e->dq_done[0],
                              &e->dq_done[1]})
        TRY_CUDA(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
    }
    TRY_CUDA(e->dq_slot[0].ensure(slot_bytes));
    TRY_CUDA(e->dq_slot[1].ensure(slot_bytes));
    // slots are free once the work queued so far on st (an earlier forward) is done
    TRY_CUDA(cudaEventRecord(e->dq_start, st));
    TRY_CUDA(cudaStreamWaitEvent(e->dq, e->dq_start, 0));
  }
  // jobs of layer i into its slot; the (codes -> copy) table the linears look up
  auto slot_jobs = [&](int i, std::vector<nrp::DeqJob>& jobs,
                       std::vector<std::pair<const void*, const void*>>& table) {
    auto* dst = e->dq_slot[i & 1].as<__nv_bfloat16>();
    for (const QuantWeight& q : qw[i]) {
      jobs.push_back({static_cast<const uint8_t*>(q.wq), static_cast<const __nv_bfloat16*>(q.qs),
                      static_cast<const __nv_bfloat16*>(q.qb), dst, q.N, q.K});
      table.emplace_back(q.wq, dst);
      dst += static_cast<size_t>(q.N) * q.K;
    }
  };
  auto issue = [&](int i) -> int {
    std::vector<nrp::DeqJob> jobs;
    std::vector<std::pair<const void*, const void*>> table;
    slot_jobs(i, jobs, table);
    if (i >= 2) TRY_CUDA(cudaStreamWaitEvent(e->dq, e->dq_done[i & 1], 0));  // layer i-2 done
    {
      nrp::ProfScope ps(e->ctx, NRP_KERNEL_DEQUANT, e->dq);
      TRY_CUDA(nrp::launch_dequant_q8_batch(jobs.data(), static_cast<int>(jobs.size()),
                                            e->ctx->num_sms, e->dq));
    }
    TRY_CUDA(cudaEventRecord(e->dq_ready[i & 1], e->dq));
    return NRP_OK;
  };
  if (pre) {
    const int rc = issue(0);
    if (rc) return rc;
  }
  for (int i = 0; i < L; ++i) {
    if (pre) {
      if (i + 1 < L) {
        const int rc = issue(i + 1);
        if (rc) return rc;
      }
      TRY_CUDA(cudaStreamWaitEvent(st, e->dq_ready[i & 1], 0));
      std::vector<nrp::DeqJob> jobs;
      slot_jobs(i, jobs, e->ctx->predeq);
    }
    const int rc = nrp_block_forward(e->blocks[i], stream, e->x.p, B, T, e->pos.p, lengths,
                                     context, e->x.p);
    e->ctx->predeq.clear();
    if (pre) TRY_CUDA(cudaEventRecord(e->dq_done[i & 1], st));
    if (rc) return rc;
  }
  // 717: transpose to [B, D, T]
  nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, st);
  TRY_CUDA(nrp::launch_transpose_btd(e->x.as<__nv_bfloat16>(), static_cast<__nv_bfloat16*>(out), B,
                                     T, D, st));
  return NRP_OK;
}

int encoder_checks(nrp_encoder* e, int B, int T) {
  if (B <= 0 || T <= 0) return failf(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  if (e->dtype != NRP_DTYPE_BF16)
    return failf(NRP_ERR_UNSUPPORTED, "the encoder runs in bf16 (nrp_encoder_set_dtype)");
  if (nrp::select_device(e->ctx)) return NRP_ERR_CUDA;
  return NRP_OK;
}

}  // namespace

extern "C" {

int nrp_encoder_forward_from_embeddings(nrp_encoder* e, void* stream, const void* x, int B, int T,
                                        const int32_t* lengths, const nrp_att_context* context,
                                        void* out) {
  if (!e || !x || !out) return failf(NRP_ERR_INVALID, "null argument");
  int rc = encoder_checks(e, B, T);
  if (rc) return rc;
  const int64_t n = static_cast<int64_t>(B) * T * e->D;
  TRY_CUDA(e->x.ensure(n * 2));
  {
    nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, static_cast<cudaStream_t>(stream));
    TRY_CUDA(cudaMemcpyAsync(e->x.p, x, n * 2, cudaMemcpyDeviceToDevice,
                             static_cast<cudaStream_t>(stream)));
  }
  return encoder_layers(e, stream, B, T, lengths, context, out);
}

int nrp_encoder_forward_streaming(nrp_encoder* e, void* stream, const float* features, int B,
                                  int frames, const int32_t* lengths, nrp_encoder_cache* cache,
                                  int drop_extra_pre_encoded, const nrp_att_context* context,
                                  void* out, int32_t* out_lengths, int* out_frames) {
  if (!e || !features || !cache || !out) return failf(NRP_ERR_INVALID, "null argument");
  if (!e->sub) return failf(NRP_ERR_INVALID, "the encoder has no subsampling");
  if (cache->enc != e) return failf(NRP_ERR_INVALID, "cache belongs to another encoder");
  if (B != cache->B) return failf(NRP_ERR_INVALID, "batch %d does not match the cache", B);
  if (B <= 0 || frames <= 0 || drop_extra_pre_encoded < 0)
    return failf(NRP_ERR_INVALID, "empty input [%d, %d] or negative drop", B, frames);
  const int Ts = nrp::subsampling_output_frames(e->sub, frames);
  const int T = Ts - drop_extra_pre_encoded;  // 864-868
  int rc = encoder_checks(e, B, T);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = e->D, C = cache->C;
  const size_t row = static_cast<size_t>(D) * 2;
  // 860-862: the conv stack over the chunk (no mel mask on this path)
  void* sub_out = e->x.p;
  TRY_CUDA(e->x.ensure(static_cast<size_t>(B) * T * row));
  if (drop_extra_pre_encoded > 0) {
    TRY_CUDA(e->sx.ensure(static_cast<size_t>(B) * Ts * row));
    sub_out = e->sx.p;
  } else {
    sub_out = e->x.p;
  }
  const int64_t F = nrp::subsampling_feat_in(e->sub);
  rc = nrp::subsampling_run(e->sub, st, features, F * frames, 1, frames, B, frames, nullptr,
                            sub_out);
  if (rc) return rc;
  if (drop_extra_pre_encoded > 0) {
    nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(cudaMemcpy2DAsync(e->x.p, T * row,
                               static_cast<uint8_t*>(e->sx.p) + drop_extra_pre_encoded * row,
                               Ts * row, T * row, B, cudaMemcpyDeviceToDevice, st));
  }
  // 869-876: subsampled lengths less the dropped frames
  std::vector<int32_t> olen(B);
  for (int b = 0; b < B; ++b) {
    const int len = lengths ? std::max(lengths[b], 0) : frames;
    olen[b] = std::max(nrp::subsampling_output_frames(e->sub, len) - drop_extra_pre_encoded, 0);
  }
  // 878-882: x * xscale
  const int64_t n = static_cast<int64_t>(B) * T * D;
  if (e->xscale != 1.f) {
    nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(nrp::launch_scale(e->x.as<__nv_bfloat16>(), n, nrp::bf16_round(e->xscale), st));
  }
  // 884-892: the first stream's valid length and fill level; the positional
  // table of cache + chunk frames
  const int valid = std::min(olen[0], T);
  const int filled = std::min(std::max(cache->filled, 0), C);
  if (e->spos_T != C + T) {
    TRY_CUDA(e->spos.ensure(static_cast<size_t>(2 * (C + T) - 1) * row));
    rc = nrp_pe_encoding(e->ctx, D, e->max_len, C + T, NRP_DTYPE_BF16, e->spos.p, stream);
    if (rc) return rc;
    e->spos_T = C + T;
  }
  // 943-1000: every block with its caches
  for (size_t i = 0; i < e->blocks.size(); ++i) {
    void* conv = nullptr;
    rc = nrp_encoder_cache_layer(cache, static_cast<int>(i), nullptr, &conv);
    if (!rc)
      rc = nrp_block_forward_with_cache(e->blocks[i], stream, e->x.p, B, T, e->spos.p,
                                        cache->attn[i], conv, filled, valid, context, e->x.p);
    if (rc) return rc;
  }
  // 1003-1004: [B, D, T]
  {
    nrp::ProfScope ps(e->ctx, NRP_KERNEL_ELEMENTWISE, st);
    TRY_CUDA(nrp::launch_transpose_btd(e->x.as<__nv_bfloat16>(), static_cast<__nv_bfloat16*>(out),
                                       B, T, D, st));
  }
  // 1020-1030: fill level += frames kept (T - cache_drop_size)
  const int drop = e->blocks.empty() ? 0 : nrp::attn_cache_drop(e->blocks[0]->attn);
  cache->filled = std::min(filled + std::max(T - drop, 0), C);
  if (out_lengths)
    for (int b = 0; b < B; ++b) out_lengths[b] = olen[b];
  if (out_frames) *out_frames = T;
  return NRP_OK;
}

int nrp_encoder_forward(nrp_encoder* e, void* stream, const float* features, int B, int frames,
                        const int32_t* lengths, const nrp_att_context* context, void* out,
                        int32_t* out_lengths) {
  if (!e || !features || !out) return failf(NRP_ERR_INVALID, "null argument");
  if (!e->sub) return failf(NRP_ERR_INVALID, "the encoder has no subsampling");
  if (B <= 0 || frames <= 0) return failf(NRP_ERR_INVALID, "empty input [%d, %d]", B, frames);
  const int T = nrp::subsampling_output_frames(e->sub, frames);
  int rc = encoder_checks(e, B, T);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 484-518: mel frames past each length read as zero; 1387-1411: the
  // subsampled lengths, which mask the blocks (PaddingMask::new, 1603-1614:
  // none when no frame is padding)
  e->lens_host.resize(2 * static_cast<size_t>(B));
  bool padded = false;
  for (int b = 0; b < B; ++b) {
    const int len = lengths ? lengths[b] : frames;
    e->lens_host[b] = len;
    e->lens_host[B + b] = nrp::subsampling_output_frames(e->sub, std::max(len, 0));
    padded = padded || e->lens_host[B + b] < T;
  }
  TRY_CUDA(e->lens.ensure(2 * static_cast<size_t>(B) * 4));
  TRY_CUDA(cudaMemcpyAsync(e->lens.p, e->lens_host.data(), 2 * static_cast<size_t>(B) * 4,
                           cudaMemcpyHostToDevice, st));
  const int32_t* d_len = e->lens.as<int32_t>();
  TRY_CUDA(e->x.ensure(static_cast<size_t>(B) * T * e->D * 2));
  const int64_t F = nrp::subsampling_feat_in(e->sub);
  rc = nrp::subsampling_run(e->sub, st, features, F * frames, 1, frames, B, frames,
                            lengths ? d_len : nullptr, e->x.p);
  if (rc) return rc;
  rc = encoder_layers(e, stream, B, T, padded ? d_len + B : nullptr, context, out);
  if (rc) return rc;
  if (out_lengths)
    for (int b = 0; b < B; ++b) out_lengths[b] = e->lens_host[B + b];
  return NRP_OK;
}

}  // extern "C"
