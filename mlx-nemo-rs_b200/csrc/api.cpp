// api.cpp -- the C ABI of libnemo_relpos.so (declared in include/nemo_relpos.h).
//
// Host-side logic of the drop-in: parameter loading and dtype casts
// (RelPositionMultiHeadAttention::{load_weights,set_dtype},
// src/asr/modules/encoders/attention.rs:409-423, 863-893; LinearLayer::cast,
// src/core/quantization.rs:92-114), the positional table
// (attention.rs:59-177), masks (attention.rs:210-294,
// src/asr/modules/encoders/conformer.rs:97-323), the streaming cache
// bookkeeping (attention.rs:606-816, conformer.rs:883-1037) and
// compute_streaming_config (src/asr/streaming/core.rs:247-362).  All
// arithmetic on tensors runs in the CUDA kernels; nothing here computes on
// the host what the device path computes.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/nemo_relpos.h"
#include "gemm.h"
#include "handles.h"
#include "internal.h"

using nrp::DevBuf;
using nrp::Linear;
using nrp::ProfRec;
using nrp::ProfScope;
using nrp::take_event;


namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int ok() { return NRP_OK; }

}  // namespace

namespace nrp {
int report_error(int code, const char* msg) {
  g_err = msg;
  return code;
}
int failf(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
}  // namespace nrp

namespace {

// A failed call's error is also taken out of the runtime's last-error slot,
// where the launch checks (cudaGetLastError) of later calls would find it.
#define CUDA_TRY(expr)                                                                    \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      (void)cudaGetLastError();                                                          \
      return fail(NRP_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));        \
    }                                                                                    \
  } while (0)

using nrp::bf16_bits;
using nrp::bf16_round;

}  // namespace

namespace {

// Folds finished records into the per-kind totals.
int prof_collect(nrp_context* c) {
  for (auto& r : c->recs) {
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return fail(NRP_ERR_CUDA, "cudaEventSynchronize: %s", cudaGetErrorString(e));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.start, r.stop);
    c->prof_ms[r.kind] += ms;
    c->prof_n[r.kind] += 1;
    c->prof_log.emplace_back(r.kind, ms);
    c->pool.push_back(r.start);
    c->pool.push_back(r.stop);
  }
  c->recs.clear();
  return NRP_OK;
}

size_t esize(int dtype) { return dtype == NRP_DTYPE_BF16 ? 2 : 4; }

// Upload a float vector in the module dtype.
cudaError_t upload(DevBuf& dst, const float* src, size_t n, int dtype) {
  cudaError_t e = dst.ensure(n * esize(dtype));
  if (e != cudaSuccess) return e;
  if (dtype == NRP_DTYPE_BF16) {
    std::vector<uint16_t> h(n);
    for (size_t i = 0; i < n; ++i) h[i] = bf16_bits(src[i]);
    return cudaMemcpy(dst.p, h.data(), n * 2, cudaMemcpyHostToDevice);
  }
  return cudaMemcpy(dst.p, src, n * 4, cudaMemcpyHostToDevice);
}

// MLX affine dequantisation on the host (f32 modules run quantised layers
// through the f32 GEMM): w = scale * q + bias (quantization.rs:4-8).
void dequant_host(const Linear& L, int N, int K, std::vector<float>& w) {
  w.resize(static_cast<size_t>(N) * K);
  const int per = 32 / L.bits, kg = K / L.group;
  const uint32_t mask = (1u << L.bits) - 1u;
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      const uint32_t q = (L.wq[static_cast<size_t>(n) * (K / per) + k / per] >> (L.bits * (k % per))) & mask;
      w[static_cast<size_t>(n) * K + k] =
          L.qs[static_cast<size_t>(n) * kg + k / L.group] * static_cast<float>(q) +
          L.qb[static_cast<size_t>(n) * kg + k / L.group];
    }
}

}  // namespace

void nrp::dequant_linear_host(const Linear& L, int N, int K, std::vector<float>& w) {
  dequant_host(L, N, K, w);
}

namespace {

// Device copies of the parameters in the module dtype.  Q, K and V are
// concatenated into one [3D, D] projection so the three run as one GEMM.
int sync_params(nrp_attn* a) {
  if (!a->dirty) return ok();
  const int D = a->D;
  const size_t DD = static_cast<size_t>(D) * D;
  const bool bf = a->dtype == NRP_DTYPE_BF16;
  for (int i = 0; i < 5; ++i)
    if (!a->lin[i].loaded) return fail(NRP_ERR_INVALID, "linear %d has no weights loaded", i);
  const Linear* qkv[3] = {&a->lin[0], &a->lin[1], &a->lin[2]};
  const bool q0 = qkv[0]->quant;
  if (qkv[1]->quant != q0 || qkv[2]->quant != q0)
    return fail(NRP_ERR_UNSUPPORTED, "linear_q/k/v must all be quantized or all standard");
  // quantised layers run quantised only in bf16 modules
  a->qkv_quant = bf && q0;
  a->out_quant = bf && a->lin[3].quant;
  a->pos_quant = bf && a->lin[4].quant;

  auto stage_std = [&](const Linear& L, std::vector<float>& w) {
    if (L.quant) dequant_host(L, D, D, w);
    else w = L.w;
  };
  auto upload_quant = [&](const Linear* const* Ls, int n, DevBuf& wq, DevBuf& sc, DevBuf& zp)
      -> cudaError_t {
    const int kg = D / 64;
    std::vector<uint8_t> codes(static_cast<size_t>(n) * DD);
    std::vector<float> s(static_cast<size_t>(n) * D * kg), z(static_cast<size_t>(n) * D * kg);
    for (int i = 0; i < n; ++i) {
      memcpy(codes.data() + i * DD, Ls[i]->wq.data(), DD);
      memcpy(s.data() + static_cast<size_t>(i) * D * kg, Ls[i]->qs.data(), sizeof(float) * D * kg);
      memcpy(z.data() + static_cast<size_t>(i) * D * kg, Ls[i]->qb.data(), sizeof(float) * D * kg);
    }
    cudaError_t e = wq.ensure(codes.size());
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(wq.p, codes.data(), codes.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return e;
    e = upload(sc, s.data(), s.size(), NRP_DTYPE_BF16);
    if (e != cudaSuccess) return e;
    return upload(zp, z.data(), z.size(), NRP_DTYPE_BF16);
  };

  // codes about to be replaced: their kept bf16 copies go too
  for (const DevBuf* q : {&a->w_qkv, &a->w_out, &a->w_pos}) nrp::deq_forget(a->ctx, q->p);
  // --- fused Q|K|V
  if (a->qkv_quant) {
    for (int i = 0; i < 3; ++i)
      if (qkv[i]->bits != 8 || qkv[i]->group != 64)
        return fail(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
    CUDA_TRY(upload_quant(qkv, 3, a->w_qkv, a->s_qkv, a->z_qkv));
  } else {
    std::vector<float> w(3 * DD), tmp;
    for (int i = 0; i < 3; ++i) {
      stage_std(*qkv[i], tmp);
      memcpy(w.data() + i * DD, tmp.data(), sizeof(float) * DD);
    }
    CUDA_TRY(upload(a->w_qkv, w.data(), w.size(), a->dtype));
  }
  a->has_b_qkv = !qkv[0]->bias.empty() || !qkv[1]->bias.empty() || !qkv[2]->bias.empty();
  if (a->has_b_qkv) {
    std::vector<float> b(3 * static_cast<size_t>(D), 0.f);
    for (int i = 0; i < 3; ++i)
      if (!qkv[i]->bias.empty()) memcpy(b.data() + i * D, qkv[i]->bias.data(), sizeof(float) * D);
    CUDA_TRY(upload(a->b_qkv, b.data(), b.size(), a->dtype));
  }
  // --- out
  const Linear* lo = &a->lin[3];
  if (a->out_quant) {
    if (lo->bits != 8 || lo->group != 64)
      return fail(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
    CUDA_TRY(upload_quant(&lo, 1, a->w_out, a->s_out, a->z_out));
  } else {
    std::vector<float> w;
    stage_std(*lo, w);
    CUDA_TRY(upload(a->w_out, w.data(), w.size(), a->dtype));
  }
  a->has_b_out = !lo->bias.empty();
  if (a->has_b_out) CUDA_TRY(upload(a->b_out, lo->bias.data(), D, a->dtype));
  // --- pos (no bias)
  const Linear* lp = &a->lin[4];
  if (a->pos_quant) {
    if (lp->bits != 8 || lp->group != 64)
      return fail(NRP_ERR_UNSUPPORTED, "quantized layers need bits 8, group 64");
    CUDA_TRY(upload_quant(&lp, 1, a->w_pos, a->s_pos, a->z_pos));
  } else {
    std::vector<float> w;
    stage_std(*lp, w);
    CUDA_TRY(upload(a->w_pos, w.data(), w.size(), a->dtype));
  }
  // --- position biases: kept in f32 on the device, rounded like the cast
  std::vector<float> u = a->u, v = a->v;
  if (u.empty()) u.assign(D, 0.f);
  if (v.empty()) v.assign(D, 0.f);
  if (bf)
    for (int i = 0; i < D; ++i) {
      u[i] = bf16_round(u[i]);
      v[i] = bf16_round(v[i]);
    }
  CUDA_TRY(upload(a->u_dev, u.data(), D, NRP_DTYPE_F32));
  CUDA_TRY(upload(a->v_dev, v.data(), D, NRP_DTYPE_F32));
  a->uv_packed.assign(static_cast<size_t>(a->H) * 128, 0u);
  for (int h = 0; h < a->H; ++h)
    for (int k = 0; k < 64; ++k) {
      const int c = h * a->dh + 2 * k;
      if (c + 1 >= D) break;
      a->uv_packed[h * 128 + k] =
          bf16_bits(u[c]) | (static_cast<uint32_t>(bf16_bits(u[c + 1])) << 16);
      a->uv_packed[h * 128 + 64 + k] =
          bf16_bits(v[c]) | (static_cast<uint32_t>(bf16_bits(v[c + 1])) << 16);
    }
  a->dirty = false;
  a->spos_len = -1;
  return ok();
}

// Rows from which a quantised linear runs as the bf16 tcgen05 GEMM over its
// weight's bf16 copy (kept, or dequantised once per call: N*K read, 2*N*K
// written).  Up to kQSmallMaxM rows the small-M kernel reads the codes
// directly.  Measured (N = 4096, K = 1024, M = 128): the tcgen05 GEMM that
// dequantises in its B producer took 53 us, because only N/256 CTAs work and
// each dequantises its whole slab, and dequantise-once + the bf16 GEMM 19 us
// (two launches, few tiles at 128 rows); so the former serves only what the
// small-M kernel cannot (GLU, batched-stride epilogues) below this row count.
constexpr int kDequantOnceMinRows = nrp::kQSmallMaxM + 1;

// y[M,N] (row stride ldy) = x[M,K] . W^T (+ bias) in the module dtype; W is
// either a dense [N,K] matrix or 8-bit codes with bf16 scales/zero points.
// keep: the weight belongs to a module (its codes' address stays theirs
// until the module re-uploads or frees them), so a quantised weight's bf16
// copy may be kept (nrp_context::deq_cache); caller-owned buffers
// (nrp_qlinear) are never kept.
int run_linear(nrp_context* ctx, cudaStream_t st, int dtype, const void* x, int M, int K,
               const void* w, bool quant, const void* qs, const void* qb, int N,
               const void* bias, void* y, int ldy, const nrp::RowTiling& rt = nrp::RowTiling(),
               const nrp::Epilogue& ep = nrp::Epilogue(), bool keep = false,
               bool w_owned = true) {
  if (M <= 0) return ok();
  if (dtype == NRP_DTYPE_F32) {
    if (ep.mode != nrp::kEpiBias)
      return fail(NRP_ERR_UNSUPPORTED, "fused epilogues run in bf16 modules only");
    ProfScope ps(ctx, NRP_KERNEL_GEMM_F32, st);
    CUDA_TRY(nrp::launch_gemm_f32(static_cast<const float*>(x), M, K, static_cast<const float*>(w),
                                  N, static_cast<const float*>(bias), static_cast<float*>(y), ldy,
                                  ctx->num_sms, ctx->d_err, st));
    return ok();
  }
  if (K % 64 != 0 || N % 32 != 0 || ldy % 8 != 0)
    return fail(NRP_ERR_UNSUPPORTED, "bf16 linear needs K %% 64 == 0 and N %% 32 == 0 (K=%d N=%d)", K, N);
  // Up to 256 rows: the small-M kernel reads the 8-bit codes (1 byte per
  // weight) even where a bf16 copy exists.  It writes flat rows: not for an
  // output or input with its own batch stride, nor the GLU epilogue.
  if (quant && rt.y_bstride == 0 && rt.x_bstride == 0 &&
      (ep.mode != nrp::kEpiResidual || ep.res_bs == 0 ||
       (rt.T > 0 && ep.res_bs == static_cast<int64_t>(rt.T) * ep.ldr)) &&
      nrp::qgemm_small_supported(M, K, x, w, ep)) {
    ProfScope ps(ctx, NRP_KERNEL_QGEMV, st);
    CUDA_TRY(nrp::launch_qgemm_small(static_cast<const __nv_bfloat16*>(x), M, K,
                                     static_cast<const uint8_t*>(w),
                                     static_cast<const __nv_bfloat16*>(qs),
                                     static_cast<const __nv_bfloat16*>(qb),
                                     static_cast<const __nv_bfloat16*>(bias),
                                     static_cast<__nv_bfloat16*>(y), ldy, N, ctx->num_sms,
                                     ctx->d_err, st, ep));
    return ok();
  }
  if (quant)
    for (const auto& pr : ctx->predeq)
      if (pr.first == w) {
        w = pr.second;
        quant = false;
        break;
      }
  // Quantised weights with many rows: the weight's bf16 copy, made on its
  // first such use and kept (the in-register producer would redo the
  // dequantisation for every 128-row tile)
  if (quant && M >= kDequantOnceMinRows && keep && ctx->deq_cache_on) {
    auto it = ctx->deq_cache.find(w);
    if (it == ctx->deq_cache.end()) {
      auto copy = std::make_unique<nrp::DevBuf>();
      CUDA_TRY(copy->ensure(static_cast<size_t>(N) * K * 2));
      {
        ProfScope ps(ctx, NRP_KERNEL_DEQUANT, st);
        CUDA_TRY(nrp::launch_dequant_q8(static_cast<const uint8_t*>(w),
                                        static_cast<const __nv_bfloat16*>(qs),
                                        static_cast<const __nv_bfloat16*>(qb),
                                        copy->as<__nv_bfloat16>(), N, K, ctx->num_sms, st));
      }
      // once: later calls may come on any stream
      CUDA_TRY(cudaStreamSynchronize(st));
      it = ctx->deq_cache.emplace(w, std::move(copy)).first;
    }
    w = it->second->p;
    quant = false;
  }
  // Without the kept copies: dequantise the weight once per call into the
  // context's scratch.
  bool w_from_scratch = false;
  if (quant && M >= kDequantOnceMinRows) {
    w_from_scratch = true;
    // one scratch per stream the library uses, so overlapping calls on the
    // caller's stream and the side stream never share it
    nrp::DevBuf& scratch = st == ctx->side ? ctx->wscratch_side : ctx->wscratch;
    CUDA_TRY(scratch.ensure(static_cast<size_t>(N) * K * 2));
    {
      ProfScope ps(ctx, NRP_KERNEL_DEQUANT, st);
      CUDA_TRY(nrp::launch_dequant_q8(static_cast<const uint8_t*>(w),
                                      static_cast<const __nv_bfloat16*>(qs),
                                      static_cast<const __nv_bfloat16*>(qb),
                                      scratch.as<__nv_bfloat16>(), N, K, ctx->num_sms, st));
    }
    w = scratch.p;
    quant = false;
  }
  CUtensorMap mx;
  const bool xmap_ok =
      rt.T > 0 ? nrp::make_tmap_3d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, rt.T, rt.B,
                                   static_cast<uint64_t>(K) * 2,
                                   static_cast<uint64_t>(rt.x_bstride ? rt.x_bstride
                                                                      : static_cast<int64_t>(K) * rt.T) * 2,
                                   64, 128, 1, true)
               : nrp::make_tmap_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M,
                                   static_cast<uint64_t>(K) * 2, 64, 128, true);
  if (!xmap_ok) return fail(NRP_ERR_CUDA, "TMA descriptor for x rejected");
  if (quant) {
    ProfScope ps(ctx, NRP_KERNEL_GEMM_Q8, st);
    CUDA_TRY(nrp::launch_gemm_q8(mx, static_cast<const uint8_t*>(w),
                                 static_cast<const __nv_bfloat16*>(qs),
                                 static_cast<const __nv_bfloat16*>(qb),
                                 static_cast<const __nv_bfloat16*>(bias),
                                 static_cast<__nv_bfloat16*>(y), ldy, M, N, K, ctx->num_sms,
                                 ctx->d_err, st, rt, ep));
  } else {
    ProfScope ps(ctx, NRP_KERNEL_GEMM_BF16, st);
    // Module weights were uploaded or dequantised ahead (kept copies after a
    // sync, prefetched copies behind an event); weights dequantised into the
    // scratch just now, and caller-owned ones, may come from the previous
    // kernel
    CUDA_TRY(nrp::launch_gemm_bf16(mx, w, static_cast<const __nv_bfloat16*>(bias),
                                   static_cast<__nv_bfloat16*>(y), ldy, M, N, K, ctx->num_sms,
                                   ctx->d_err, st, rt, ep, w_owned && !w_from_scratch));
  }
  return ok();
}

int check_device(nrp_context* ctx) {
  int cur = -1;
  CUDA_TRY(cudaGetDevice(&cur));
  if (cur != ctx->device) CUDA_TRY(cudaSetDevice(ctx->device));
  return ok();
}

}  // namespace

extern "C" {

int nrp_abi_version(void) { return NRP_ABI_VERSION; }

const char* nrp_last_error(void) { return g_err.c_str(); }

// ------------------------------------------------------------ host logic
int nrp_pe_encoding_host(int d_model, int max_len, int seq_len, float* out) {
  if (!out || d_model <= 0 || d_model % 2 || max_len <= 0)
    return fail(NRP_ERR_INVALID, "invalid positional encoding arguments");
  if (seq_len <= 0) return fail(NRP_ERR_INVALID, "positional encoding requested for an empty sequence");
  // A table of length L holds positions (L-1)..-(L-1); get_encoding slices
  // positions (seq_len-1)..-(seq_len-1) from it, or rebuilds at seq_len.
  const int half = d_model / 2;
  std::vector<float> div(half);
  const float lnf = logf(10000.0f) / static_cast<float>(d_model);
  for (int k = 0; k < half; ++k) div[k] = expf(-static_cast<float>(2 * k) * lnf);
  for (int r = 0; r < 2 * seq_len - 1; ++r) {
    const float pos = static_cast<float>(seq_len - 1 - r);
    float* row = out + static_cast<size_t>(r) * d_model;
    for (int k = 0; k < half; ++k) {
      const float ang = pos * div[k];
      row[2 * k] = sinf(ang);
      row[2 * k + 1] = cosf(ang);
    }
  }
  return ok();
}

float nrp_pe_xscale(int d_model, int xscaling) {
  return xscaling ? sqrtf(static_cast<float>(d_model)) : 1.0f;
}

int nrp_att_context_new(int left, int right, const char* style, nrp_att_context* out) {
  if (left < 0 && right < 0) return 0;
  if (out) {
    out->left = left;
    out->right = right;
    out->chunked = (style && strcmp(style, "chunked_limited") == 0) ? 1 : 0;
  }
  return 1;
}

static inline int ctx_visible(const nrp_att_context* c, int i, int j) {
  if (c->chunked && c->right >= 0) {
    const int chunk = c->right + 1;
    const int lc = c->left >= 0 ? c->left / chunk : 10000;
    const int diff = i / chunk - j / chunk;
    return diff >= 0 && diff <= lc;
  }
  const int off = j - i;
  int vis = c->left < 0 ? 1 : off >= -std::max(c->left, 0);
  if (!c->chunked && c->right >= 0) vis = vis && off <= c->right;
  return vis;
}

int nrp_block_mask_host(const nrp_att_context* context, int start, int end, int seq_len,
                        uint8_t* vis) {
  if (!context || !vis || end < start || seq_len < 0) return fail(NRP_ERR_INVALID, "invalid mask arguments");
  for (int i = start; i < end; ++i)
    for (int j = 0; j < seq_len; ++j)
      vis[static_cast<size_t>(i - start) * seq_len + j] = static_cast<uint8_t>(ctx_visible(context, i, j));
  return ok();
}

int nrp_key_padding_mask_host(const int32_t* lengths, int batch, int seq_len, float* mask) {
  if (!lengths || batch < 0) return fail(NRP_ERR_INVALID, "invalid key padding arguments");
  bool any = false;
  for (int b = 0; b < batch; ++b) any = any || lengths[b] < seq_len;
  if (!any) return 0;
  if (mask)
    for (int b = 0; b < batch; ++b) {
      const int len = std::max(lengths[b], 1);
      for (int j = 0; j < seq_len; ++j)
        mask[static_cast<size_t>(b) * seq_len + j] = j < len ? 0.0f : -INFINITY;
    }
  return 1;
}

int nrp_streaming_mask_host(const nrp_att_context* context, int max_audio_length, int cache_len,
                            int filled_cache_len, int tensor_seq_len, int valid_seq_len,
                            uint8_t* vis) {
  if (!vis || tensor_seq_len < 0 || max_audio_length < cache_len + tensor_seq_len)
    return fail(NRP_ERR_INVALID, "invalid streaming mask arguments");
  const int offset = cache_len - filled_cache_len;
  for (int ii = 0; ii < tensor_seq_len; ++ii) {
    const int i = cache_len + ii;
    for (int j = 0; j < max_audio_length; ++j) {
      int m = 1;
      if (context) {
        if (context->chunked && context->right == -1) {
          if (context->left >= 0) m = (j - i) >= -context->left;
        } else {
          m = ctx_visible(context, i, j);
        }
      }
      if (offset > 0) m = m && j >= offset;
      if (valid_seq_len < tensor_seq_len) m = m && ii < valid_seq_len;
      vis[static_cast<size_t>(ii) * max_audio_length + j] = static_cast<uint8_t>(m);
    }
  }
  return ok();
}

int nrp_streaming_config_compute(int left, int right, int chunked, int n_layers,
                                 int subsampling_factor, int conv_kernel_size, int causal_conv,
                                 int mode_idx, int max_context, nrp_streaming_config* out) {
  if (!out || subsampling_factor <= 0 || conv_kernel_size <= 0 || n_layers < 0)
    return fail(NRP_ERR_INVALID, "invalid streaming config arguments");
  const int ctx0 = causal_conv ? conv_kernel_size - 1 : (conv_kernel_size - 1) / 2;
  const int ctx1 = causal_conv ? 0 : (conv_kernel_size - 1) / 2;
  int la, drop;
  if (chunked) {
    la = std::max(right, 0);
    drop = 0;
  } else {
    la = right >= 0 ? right * n_layers + ctx1 * n_layers : 0;
    drop = la;
  }
  const int sf = subsampling_factor;
  out->cache_drop_size = drop;
  out->last_channel_cache_size = left >= 0 ? left : max_context;
  out->last_time_cache_size = ctx0;
  out->chunk_size[0] = 1 + sf * la;
  out->chunk_size[1] = sf + sf * la;
  const int shift_steps = std::max(la - drop, 0);
  out->shift_size[0] = 1 + sf * shift_steps;
  out->shift_size[1] = sf + sf * shift_steps;
  out->valid_out_len = (out->shift_size[1] - sf) / sf + 1;
  out->pre_encode_cache_size[0] = 0;
  out->pre_encode_cache_size[1] = sf + 1;
  out->drop_extra_pre_encoded = 1 + (out->pre_encode_cache_size[1] - 1) / sf;
  out->lookahead_frames = la;
  out->mode_idx = mode_idx;
  out->left_context = left;
  out->right_context = right;
  return ok();
}

// --------------------------------------------------------------- context
int nrp_context_create(int device, nrp_context** out) {
  if (!out) return fail(NRP_ERR_INVALID, "null output handle");
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(NRP_ERR_INVALID, "device %d out of range (%d devices)", device, n);
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(NRP_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  // the no-allocation forward's static array: its module is loaded (and the
  // array's device memory committed) here, not by a noalloc call
  if (int rc = nrp::noalloc_scratch_prepare(device)) return rc;
  auto* c = new nrp_context;
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaMalloc(&c->d_err, sizeof(int) * kCtxInts);
  if (e != cudaSuccess) {
    delete c;
    return fail(NRP_ERR_NOMEM, "cudaMalloc: %s", cudaGetErrorString(e));
  }
  cudaMemset(c->d_err, 0, sizeof(int) * kCtxInts);
  e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    nrp_context_destroy(c);
    return fail(NRP_ERR_CUDA, "side stream: %s", cudaGetErrorString(e));
  }
  *out = c;
  return ok();
}

int nrp_context_destroy(nrp_context* ctx) {
  if (!ctx) return ok();
  cudaSetDevice(ctx->device);  // (errors of this teardown are dropped below)
  prof_collect(ctx);
  for (cudaEvent_t e : ctx->pool) cudaEventDestroy(e);
  if (ctx->side) {
    cudaStreamSynchronize(ctx->side);
    cudaStreamDestroy(ctx->side);
  }
  if (ctx->fork) cudaEventDestroy(ctx->fork);
  if (ctx->join) cudaEventDestroy(ctx->join);
  cudaFree(ctx->d_err);
  delete ctx;
  (void)cudaGetLastError();
  return ok();
}

int nrp_context_set_weight_cache(nrp_context* ctx, int enable) {
  if (!ctx) return fail(NRP_ERR_INVALID, "null context");
  ctx->deq_cache_on = enable != 0;
  if (!ctx->deq_cache_on) {
    if (check_device(ctx)) return NRP_ERR_CUDA;
    CUDA_TRY(cudaDeviceSynchronize());  // (copies still read by queued work)
    ctx->deq_cache.clear();
  }
  return ok();
}

int nrp_context_check(nrp_context* ctx, void* stream) {
  if (!ctx) return fail(NRP_ERR_INVALID, "null context");
  if (check_device(ctx)) return NRP_ERR_CUDA;
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int e = 0;
  CUDA_TRY(cudaMemcpy(&e, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    return fail(NRP_ERR_DEVICE, "a kernel gave up on a bounded wait (code %d)", e);
  }
  return ok();
}

int nrp_context_selftest_wait_expiry(nrp_context* ctx, void* stream, int budget_us) {
  if (!ctx) return fail(NRP_ERR_INVALID, "null context");
  if (budget_us < 1 || budget_us > 1000000)
    return fail(NRP_ERR_INVALID, "budget %d us outside [1, 1000000]", budget_us);
  if (check_device(ctx)) return NRP_ERR_CUDA;
  CUDA_TRY(nrp::launch_wait_expiry(ctx->d_err, static_cast<uint64_t>(budget_us) * 1000,
                                   static_cast<cudaStream_t>(stream)));
  return ok();
}

int nrp_pe_encoding(nrp_context* ctx, int d_model, int max_len, int seq_len, int dtype,
                    void* dev_out, void* stream) {
  if (!ctx || !dev_out) return fail(NRP_ERR_INVALID, "null argument");
  std::vector<float> h(static_cast<size_t>(2 * std::max(seq_len, 1) - 1) * std::max(d_model, 1));
  int rc = nrp_pe_encoding_host(d_model, max_len, seq_len, h.data());
  if (rc) return rc;
  if (check_device(ctx)) return NRP_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NRP_DTYPE_BF16) {
    std::vector<uint16_t> b(h.size());
    for (size_t i = 0; i < h.size(); ++i) b[i] = bf16_bits(h[i]);
    CUDA_TRY(cudaMemcpyAsync(dev_out, b.data(), b.size() * 2, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaStreamSynchronize(st));  // host staging buffer goes out of scope
  } else {
    CUDA_TRY(cudaMemcpyAsync(dev_out, h.data(), h.size() * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaStreamSynchronize(st));
  }
  return ok();
}

// ------------------------------------------------------------- attention
int nrp_attn_create(nrp_context* ctx, int d_model, int n_heads, int use_bias, nrp_attn** out) {
  if (!ctx || !out) return fail(NRP_ERR_INVALID, "null argument");
  if (d_model <= 0 || n_heads <= 0 || d_model % n_heads)
    return fail(NRP_ERR_INVALID, "d_model %d not divisible by n_heads %d", d_model, n_heads);
  if (d_model / n_heads > 128)
    return fail(NRP_ERR_UNSUPPORTED, "head_dim %d > 128", d_model / n_heads);
  auto* a = new nrp_attn;
  a->ctx = ctx;
  a->device = ctx->device;
  a->ctx_alive = ctx->alive;
  a->D = d_model;
  a->H = n_heads;
  a->dh = d_model / n_heads;
  a->use_bias = use_bias;
  // zero parameters, like RelPositionMultiHeadAttention::new
  for (int i = 0; i < 5; ++i) {
    a->lin[i].loaded = true;
    a->lin[i].w.assign(static_cast<size_t>(d_model) * d_model, 0.f);
    if (use_bias && i != NRP_LINEAR_POS) a->lin[i].bias.assign(d_model, 0.f);
  }
  a->u.assign(d_model, 0.f);
  a->v.assign(d_model, 0.f);
  *out = a;
  return ok();
}

int nrp_attn_destroy(nrp_attn* attn) {
  if (attn) {
    // (its context may be gone already: only the device number is used)
    cudaSetDevice(attn->device);
    if (!attn->ctx_alive.expired())
      for (const DevBuf* q : {&attn->w_qkv, &attn->w_out, &attn->w_pos})
        nrp::deq_forget(attn->ctx, q->p);
    delete attn;
    (void)cudaGetLastError();
  }
  return ok();
}

int nrp_attn_set_dtype(nrp_attn* attn, int dtype) {
  if (!attn) return fail(NRP_ERR_INVALID, "null module");
  if (dtype != NRP_DTYPE_F32 && dtype != NRP_DTYPE_BF16)
    return fail(NRP_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (dtype == NRP_DTYPE_BF16 && attn->dh != 128)
    return fail(NRP_ERR_UNSUPPORTED, "bf16 kernels need head_dim 128 (got %d)", attn->dh);
  attn->dtype = dtype;
  attn->dirty = true;
  attn->spos_len = -1;
  return ok();
}

int nrp_attn_set_cache_drop_size(nrp_attn* attn, int cache_drop_size) {
  if (!attn || cache_drop_size < 0) return fail(NRP_ERR_INVALID, "invalid cache_drop_size");
  attn->cache_drop = cache_drop_size;
  return ok();
}

int nrp_attn_load_linear(nrp_attn* attn, int which, const float* weight, const float* bias) {
  if (!attn || !weight || which < 0 || which > 4) return fail(NRP_ERR_INVALID, "invalid linear arguments");
  Linear& L = attn->lin[which];
  const size_t n = static_cast<size_t>(attn->D) * attn->D;
  L = Linear();
  L.loaded = true;
  L.w.assign(weight, weight + n);
  if (bias) L.bias.assign(bias, bias + attn->D);
  attn->dirty = true;
  return ok();
}

int nrp_attn_load_linear_quantized(nrp_attn* attn, int which, int bits, int group_size,
                                   const uint32_t* wq, const float* scales, const float* biases,
                                   const float* bias) {
  if (!attn || !wq || !scales || !biases || which < 0 || which > 4)
    return fail(NRP_ERR_INVALID, "invalid quantized linear arguments");
  if (bits != 8 || group_size != 64)
    return fail(NRP_ERR_UNSUPPORTED, "quantized linear: bits %d group %d (supported: 8, 64)", bits, group_size);
  const int D = attn->D;
  if (D % 64) return fail(NRP_ERR_UNSUPPORTED, "d_model %d not a multiple of the group size", D);
  Linear& L = attn->lin[which];
  L = Linear();
  L.loaded = true;
  L.quant = true;
  L.bits = bits;
  L.group = group_size;
  L.wq.assign(wq, wq + static_cast<size_t>(D) * D / 4);
  L.qs.assign(scales, scales + static_cast<size_t>(D) * (D / 64));
  L.qb.assign(biases, biases + static_cast<size_t>(D) * (D / 64));
  if (bias) L.bias.assign(bias, bias + D);
  attn->dirty = true;
  return ok();
}

int nrp_attn_load_pos_bias(nrp_attn* attn, const float* u, const float* v) {
  if (!attn || !u || !v) return fail(NRP_ERR_INVALID, "null pos bias");
  attn->u.assign(u, u + attn->D);
  attn->v.assign(v, v + attn->D);
  attn->dirty = true;
  return ok();
}

int nrp_attn_forward(nrp_attn* a, void* stream, const void* x, int B, int T, const void* pos_emb,
                     const int32_t* lengths, const nrp_att_context* context, void* out) {
  return nrp::attn_forward(a, static_cast<cudaStream_t>(stream), x, B, T, pos_emb, lengths,
                           context, out, nrp::Epilogue());
}

}  // extern "C"

namespace nrp {

int attn_forward(nrp_attn* a, cudaStream_t st, const void* x, int B, int T, const void* pos_emb,
                 const int32_t* lengths, const nrp_att_context* context, void* out,
                 const Epilogue& out_ep) {
  if (!a || !x || !pos_emb || !out) return fail(NRP_ERR_INVALID, "null argument");
  if (B <= 0 || T <= 0) return fail(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  nrp_context* ctx = a->ctx;
  if (check_device(ctx)) return NRP_ERR_CUDA;
  int rc = sync_params(a);
  if (rc) return rc;
  const int D = a->D, P = 2 * T - 1;
  const size_t es = esize(a->dtype);
  const size_t BT = static_cast<size_t>(B) * T;
  CUDA_TRY(a->qkv.ensure(BT * 3 * D * es));
  CUDA_TRY(a->cbuf.ensure(BT * D * es));
  CUDA_TRY(a->pbuf.ensure(static_cast<size_t>(P) * D * es));
  nrp::AttnContextDev cd{0, -1, -1, 0};
  if (context) cd = {1, context->left, context->right, context->chunked};
  // With a key padding mask the row tiles of the per-frame GEMMs follow the
  // utterances and skip frames past each length (their rows are zeros:
  // padded rows are unspecified in the reference, conformer.rs:1590-1593).
  nrp::RowTiling rows;
  if (lengths && B <= 256) rows = {lengths, T, B};
  if (a->dtype == NRP_DTYPE_BF16) {
    // 478-480: q, k, v in one GEMM; 493: linear_pos
    // linear_pos only over the P rows the context's relative positions
    // reach (all 2T-1 without a window; 257 for a (128, 128) window), on the
    // side stream: it fills the SMs the q|k|v GEMM leaves idle in its last
    // wave, and joins before the attention
    nrp::AttnGeom g = nrp::full_geom(T, D);
    int dmin, dmax;
    nrp::visible_offsets(cd, T, dmin, dmax);
    g.p_base = T - 1 + dmin;
    g.p_rows = dmax - dmin + 1;
    CUDA_TRY(cudaEventRecord(ctx->fork, st));
    CUDA_TRY(cudaStreamWaitEvent(ctx->side, ctx->fork, 0));
    rc = run_linear(ctx, ctx->side, a->dtype,
                    static_cast<const uint8_t*>(pos_emb) + static_cast<size_t>(g.p_base) * D * es,
                    g.p_rows, D, a->w_pos.p, a->pos_quant, a->s_pos.p, a->z_pos.p, D, nullptr,
                    a->pbuf.p, D, nrp::RowTiling(), nrp::Epilogue(), true);
    if (rc) return rc;
    CUDA_TRY(cudaEventRecord(ctx->join, ctx->side));
    rc = run_linear(ctx, st, a->dtype, x, static_cast<int>(BT), D, a->w_qkv.p, a->qkv_quant,
                    a->s_qkv.p, a->z_qkv.p, 3 * D, a->has_b_qkv ? a->b_qkv.p : nullptr, a->qkv.p,
                    3 * D, rows, nrp::Epilogue(), true);
    if (rc) return rc;
    CUDA_TRY(cudaStreamWaitEvent(st, ctx->join, 0));
    ProfScope ps(ctx, NRP_KERNEL_ATTN_SM100, st);
    CUDA_TRY(nrp::launch_relpos_attn_bf16(a->qkv.p, a->pbuf.p, a->uv_packed.data(), lengths,
                                          cd, g, a->cbuf.p, B, a->H, ctx->d_err,
                                          nrp::sched_slot(ctx), ctx->num_sms, st));
  } else {
    rc = run_linear(ctx, st, a->dtype, x, static_cast<int>(BT), D, a->w_qkv.p, a->qkv_quant,
                    a->s_qkv.p, a->z_qkv.p, 3 * D, a->has_b_qkv ? a->b_qkv.p : nullptr, a->qkv.p,
                    3 * D, nrp::RowTiling(), nrp::Epilogue(), true);
    if (rc) return rc;
    rc = run_linear(ctx, st, a->dtype, pos_emb, P, D, a->w_pos.p, a->pos_quant, a->s_pos.p,
                    a->z_pos.p, D, nullptr, a->pbuf.p, D, nrp::RowTiling(), nrp::Epilogue(), true);
    if (rc) return rc;
    const float* q = a->qkv.as<float>();
    nrp::StreamMaskDev none{};
    ProfScope ps(ctx, NRP_KERNEL_ATTN_SIMT, st);
    CUDA_TRY(nrp::launch_relpos_attn_f32(q, 3 * D, q + D, 3 * D, q + 2 * D, 3 * D,
                                         a->pbuf.as<float>(), a->u_dev.as<float>(),
                                         a->v_dev.as<float>(), lengths, cd, none,
                                         a->cbuf.as<float>(), B, T, T, D, a->H, st));
  }
  // 565: linear_out (the caller's epilogue: a block adds its residual here)
  return run_linear(ctx, st, a->dtype, a->cbuf.p, static_cast<int>(BT), D, a->w_out.p,
                    a->out_quant, a->s_out.p, a->z_out.p, D, a->has_b_out ? a->b_out.p : nullptr,
                    out, D, rows, out_ep, true);
}

int attn_sync(nrp_attn* a) { return sync_params(a); }

int attn_cache_drop(const nrp_attn* a) { return a->cache_drop; }

void deq_forget(nrp_context* ctx, const void* codes) {
  if (ctx && codes) ctx->deq_cache.erase(codes);
}

int linear(nrp_context* ctx, cudaStream_t st, int dtype, const void* x, int M, int K,
           const void* w, bool quant, const void* qs, const void* qb, int N, const void* bias,
           void* y, int ldy, const RowTiling& rt, const Epilogue& ep, bool keep) {
  return run_linear(ctx, st, dtype, x, M, K, w, quant, qs, qb, N, bias, y, ldy, rt, ep, keep);
}

int select_device(nrp_context* ctx) { return check_device(ctx); }

}  // namespace nrp

extern "C" {

// ------------------------------------------------------ sequence split
int nrp_partition_utterances(const int32_t* lengths, int n, int nranks, int d_model,
                             int32_t* rank_of, double* rank_cost) {
  if (!lengths || !rank_of || n < 0 || nranks <= 0 || d_model <= 0)
    return fail(NRP_ERR_INVALID, "invalid partition arguments");
  // cost of an utterance of L frames: attention 6 d L^2 and projections
  // 8 d^2 L (q, k, v, out), in units of 6 d
  const double g = 4.0 * d_model / 3.0;
  std::vector<double> cost(n);
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) {
    const double L = std::max(lengths[i], 0);
    cost[i] = L * L + g * L;
    order[i] = i;
  }
  // longest processing time first: each utterance to the least loaded rank
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return cost[a] > cost[b]; });
  std::vector<double> load(nranks, 0.0);
  for (int i : order) {
    int r = 0;
    for (int k = 1; k < nranks; ++k)
      if (load[k] < load[r]) r = k;
    rank_of[i] = r;
    load[r] += cost[i];
  }
  if (rank_cost)
    for (int k = 0; k < nranks; ++k) rank_cost[k] = load[k];
  return ok();
}

int nrp_copy_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                    int64_t row_bytes, void* stream, int64_t* bytes) {
  if (!dst || !src || !lengths || B < 0 || T < 0 || row_bytes <= 0)
    return fail(NRP_ERR_INVALID, "invalid copy_frames arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t bstride = static_cast<int64_t>(T) * row_bytes;
  int64_t total = 0;
  for (int b = 0; b < B; ++b) {
    const int L = std::min(std::max(lengths[b], 0), T);
    if (!L) continue;
    const int64_t off = b * bstride;
    const cudaError_t e =
        cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, static_cast<const uint8_t*>(src) + off,
                        static_cast<size_t>(L) * row_bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NRP_ERR_CUDA, cudaGetErrorString(e));
    }
    total += L * row_bytes;
  }
  if (bytes) *bytes = total;
  return ok();
}

namespace {
// Shared by nrp_unpack_frames / nrp_pack_frames: validates the arguments and
// returns the packed byte count of the batch.
int frames_args(const void* a, const void* b, const int32_t* lengths, int B, int T,
                int64_t row_bytes, int64_t* packed_bytes) {
  if (!a || !b || !lengths || B < 0 || T < 0 || row_bytes <= 0)
    return fail(NRP_ERR_INVALID, "invalid frames arguments");
  int64_t rows = 0;
  for (int i = 0; i < B; ++i) {
    if (lengths[i] < 0 || lengths[i] > T)
      return fail(NRP_ERR_INVALID, "lengths[%d] = %d outside [0, %d]", i, lengths[i], T);
    rows += lengths[i];
  }
  *packed_bytes = rows * row_bytes;
  return ok();
}

// The scatter (to_padded) or gather of the whole batch between the padded
// tensor and packed device rows, kMaxFrameUtts utterances per launch.
int frames_launch(void* padded, void* packed, const int32_t* lengths, int B, int T,
                  int64_t row_bytes, bool to_padded, int32_t* dev_lengths, cudaStream_t st) {
  nrp::FramesPlan plan;
  plan.row_bytes = row_bytes;
  plan.bstride = static_cast<int64_t>(T) * row_bytes;
  int64_t off = 0;
  for (int b0 = 0; b0 < B; b0 += nrp::kMaxFrameUtts) {
    const int n = std::min(nrp::kMaxFrameUtts, B - b0);
    plan.b0 = b0;
    for (int u = 0; u < n; ++u) {
      plan.off[u] = off;
      plan.len[u] = lengths[b0 + u];
      off += lengths[b0 + u];
    }
    if (cudaError_t e = nrp::launch_frames(padded, packed, plan, n, to_padded, dev_lengths, st))
      return fail(NRP_ERR_CUDA, "frames kernel: %s", cudaGetErrorString(e));
  }
  return ok();
}
}  // namespace

int nrp_unpack_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                      int64_t row_bytes, void* staging, int32_t* dev_lengths, void* stream,
                      int64_t* bytes) {
  int64_t nb = 0;
  if (int rc = frames_args(dst, src, lengths, B, T, row_bytes, &nb)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* packed = src;
  if (staging && nb > 0) {  // the one copy over the link
    const cudaError_t e = cudaMemcpyAsync(staging, src, static_cast<size_t>(nb),
                                          cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NRP_ERR_CUDA, cudaGetErrorString(e));
    }
    packed = staging;
  }
  if (int rc = frames_launch(dst, const_cast<void*>(packed), lengths, B, T, row_bytes, true,
                             dev_lengths, st))
    return rc;
  if (bytes) *bytes = nb;
  return ok();
}

int nrp_pack_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                    int64_t row_bytes, void* staging, void* stream, int64_t* bytes) {
  int64_t nb = 0;
  if (int rc = frames_args(dst, src, lengths, B, T, row_bytes, &nb)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* packed = staging ? staging : dst;
  if (int rc = frames_launch(const_cast<void*>(src), packed, lengths, B, T, row_bytes, false,
                             nullptr, st))
    return rc;
  if (staging && nb > 0) {
    const cudaError_t e = cudaMemcpyAsync(dst, staging, static_cast<size_t>(nb),
                                          cudaMemcpyDefault, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(NRP_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  if (bytes) *bytes = nb;
  return ok();
}

int nrp_seq_shard(int seq_len, int nranks, int rank, int* start, int* len) {
  if (!start || !len) return fail(NRP_ERR_INVALID, "null output");
  if (seq_len <= 0 || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(NRP_ERR_INVALID, "seq_len %d, rank %d of %d", seq_len, rank, nranks);
  const int seg = (seq_len + nranks - 1) / nranks;
  const long long s = std::min<long long>(seq_len, static_cast<long long>(rank) * seg);
  *start = static_cast<int>(s);
  *len = static_cast<int>(std::min<long long>(seq_len, s + seg) - s);
  return ok();
}

int nrp_seq_shard_plan(int T, int n, int r, const nrp_att_context* context, nrp_seq_plan* out) {
  if (!out) return fail(NRP_ERR_INVALID, "null output");
  int s = 0, len = 0, s_last = 0, len_last = 0;
  int rc = nrp_seq_shard(T, n, r, &s, &len);
  if (rc) return rc;
  nrp_seq_shard(T, n, n - 1, &s_last, &len_last);
  if (len_last <= 0)
    return fail(NRP_ERR_UNSUPPORTED, "%d frames leave some of %d ranks without frames", T, n);
  nrp::AttnContextDev cd{0, -1, -1, 0};
  if (context) cd = {1, context->left, context->right, context->chunked};
  int dmin, dmax;
  nrp::visible_offsets(cd, T, dmin, dmax);
  // the part of [s0 + dmin, e0 + dmax) within the sequence outside [s0, e0)
  auto left_halo = [&](int s0) { return s0 - std::max(0, std::min(s0, s0 + dmin)); };
  auto right_halo = [&](int e0) { return std::max(e0, std::min(T, e0 + dmax)) - e0; };
  const int e = s + len;
  nrp_seq_plan p{s, len, left_halo(s), right_halo(e), 0, 0};
  int tmp = 0, len_prev = 0, len_next = 0;
  if (r > 0) {
    nrp_seq_shard(T, n, r - 1, &tmp, &len_prev);
    p.send_prev = right_halo(s);  // rank r-1's right halo: my first frames
  }
  if (r + 1 < n) {
    nrp_seq_shard(T, n, r + 1, &tmp, &len_next);
    p.send_next = left_halo(e);  // rank r+1's left halo: my last frames
  }
  if (p.halo_left > len_prev || p.halo_right > len_next || p.send_prev > len ||
      p.send_next > len)
    return fail(NRP_ERR_UNSUPPORTED,
                "the attention window (key offsets %d..%d) reaches past the neighbouring "
                "segments of %d frames", dmin, dmax, len);
  *out = p;
  return ok();
}

int nrp_attn_forward_seq_sharded(nrp_attn* a, nrp_halo* h, void* stream, const void* x, int B,
                                 int T, const void* pos_emb, const int32_t* lengths,
                                 const nrp_att_context* context, void* out) {
  if (!a || !h || !x || !pos_emb || !out) return fail(NRP_ERR_INVALID, "null argument");
  if (B <= 0 || T <= 0) return fail(NRP_ERR_INVALID, "empty input [%d, %d]", B, T);
  if (h->dead) return fail(NRP_ERR_DEVICE, "the halo communicator was aborted");
  nrp_context* ctx = a->ctx;
  if (h->ctx->device != ctx->device)
    return fail(NRP_ERR_INVALID, "halo communicator on device %d, module on %d",
                h->ctx->device, ctx->device);
  if (check_device(ctx)) return NRP_ERR_CUDA;
  int rc = sync_params(a);
  if (rc) return rc;
  if (a->dtype != NRP_DTYPE_BF16)
    return fail(NRP_ERR_UNSUPPORTED, "the sequence-split forward runs in bf16");
  if (B > 256) return fail(NRP_ERR_UNSUPPORTED, "sequence split supports batch <= 256");
  nrp_seq_plan plan;
  rc = nrp_seq_shard_plan(T, h->nranks, h->rank, context, &plan);
  if (rc) return rc;
  const int D = a->D;
  const int s = plan.start, len = plan.len, e = s + len;
  const int hl = plan.halo_left, hr = plan.halo_right;
  const int send_prev = plan.send_prev, send_next = plan.send_next;
  nrp::AttnContextDev cd{0, -1, -1, 0};
  if (context) cd = {1, context->left, context->right, context->chunked};
  int dmin, dmax;
  nrp::visible_offsets(cd, T, dmin, dmax);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int tbuf = hl + len + hr;
  const size_t row = static_cast<size_t>(B) * 3 * D * 2;  // one time-major frame, all utterances
  CUDA_TRY(h->buf.ensure(static_cast<size_t>(tbuf) * row));
  CUDA_TRY(a->cbuf.ensure(static_cast<size_t>(B) * len * D * 2));
  nrp::AttnGeom g;
  g.Tg = T;
  g.tbuf = tbuf;
  g.base = s - hl;
  g.qkv_ts = static_cast<int64_t>(B) * 3 * D;
  g.qkv_bs = 3 * D;
  g.q_lo = s;
  g.q_hi = e;
  g.k_lo = s - hl;
  g.k_hi = e + hr;
  g.p_base = T - 1 + dmin;
  g.p_rows = dmax - dmin + 1;
  g.out_base = s;
  g.out_bs = static_cast<int64_t>(len) * D;
  CUDA_TRY(a->pbuf.ensure(static_cast<size_t>(g.p_rows) * D * 2));
  // linear_pos over the window's P rows (attention.rs:493)
  rc = run_linear(ctx, st, a->dtype,
                  static_cast<const uint8_t*>(pos_emb) + static_cast<size_t>(g.p_base) * D * 2,
                  g.p_rows, D, a->w_pos.p, a->pos_quant, a->s_pos.p, a->z_pos.p, D, nullptr,
                  a->pbuf.p, D, nrp::RowTiling(), nrp::Epilogue(), true);
  if (rc) return rc;
  // q|k|v of the local frames into the buffer's middle rows (478-480)
  nrp::RowTiling rt;
  rt.T = len;
  rt.B = B;
  rt.y_bstride = 3 * D;
  uint8_t* buf = static_cast<uint8_t*>(h->buf.p);
  rc = run_linear(ctx, st, a->dtype, x, B * len, D, a->w_qkv.p, a->qkv_quant, a->s_qkv.p,
                  a->z_qkv.p, 3 * D, a->has_b_qkv ? a->b_qkv.p : nullptr,
                  buf + static_cast<size_t>(hl) * row, B * 3 * D, rt, nrp::Epilogue(), true);
  if (rc) return rc;
  const bool exchange = hl + hr + send_prev + send_next > 0;
  if (exchange) {
    const size_t send_off[2] = {static_cast<size_t>(hl) * row,
                                static_cast<size_t>(hl + len - send_next) * row};
    const size_t send_bytes[2] = {static_cast<size_t>(send_prev) * row,
                                  static_cast<size_t>(send_next) * row};
    const size_t recv_off[2] = {0, static_cast<size_t>(hl + len) * row};
    const size_t recv_bytes[2] = {static_cast<size_t>(hl) * row, static_cast<size_t>(hr) * row};
    rc = nrp::halo_exchange(h, send_off, send_bytes, recv_off, recv_bytes, st);
    if (rc) return rc;
  }
  // Query tiles (128 frames from s) whose keys are all local run while the
  // halo is in flight; the others after it has arrived.
  const int ntiles = (len + 127) / 128;
  int first = 0, last = ntiles;  // local tiles [first, last)
  if (hl > 0) first = std::min(ntiles, (-dmin + 127) / 128);
  if (hr > 0) last = std::max(0, (len - dmax) / 128);
  // A launch that runs while the halo is in flight sees only the segment's
  // own frames: its tensor map starts at the segment and ends with it, so the
  // key tiles that overhang the segment load zeros instead of halo rows that
  // are being written (or were never written) -- masked keys still meet the
  // P.V product with probability 0, which must not see a NaN.
  auto attend = [&](int q_lo, int q_hi, bool local_only) -> int {
    if (q_hi <= q_lo) return ok();
    nrp::AttnGeom gi = g;
    gi.q_lo = q_lo;
    gi.q_hi = q_hi;
    const void* qkv = h->buf.p;
    if (local_only) {
      gi.base = s;
      gi.tbuf = len;
      gi.k_lo = s;
      gi.k_hi = e;
      qkv = buf + static_cast<size_t>(hl) * row;
    }
    ProfScope ps(ctx, NRP_KERNEL_ATTN_SM100, st);
    CUDA_TRY(nrp::launch_relpos_attn_bf16(qkv, a->pbuf.p, a->uv_packed.data(), lengths, cd,
                                          gi, a->cbuf.p, B, a->H, ctx->d_err,
                                          nrp::sched_slot(ctx), ctx->num_sms, st));
    return ok();
  };
  if (!exchange || first >= last) {
    if (exchange) CUDA_TRY(cudaStreamWaitEvent(st, h->done, 0));
    rc = attend(s, e, false);
    if (rc) return rc;
  } else {
    const int mid_lo = s + 128 * first, mid_hi = std::min(e, s + 128 * last);
    rc = attend(mid_lo, mid_hi, true);
    if (rc) return rc;
    CUDA_TRY(cudaStreamWaitEvent(st, h->done, 0));
    rc = attend(s, mid_lo, false);
    if (!rc) rc = attend(mid_hi, e, false);
    if (rc) return rc;
  }
  // linear_out (565)
  return run_linear(ctx, st, a->dtype, a->cbuf.p, B * len, D, a->w_out.p, a->out_quant,
                    a->s_out.p, a->z_out.p, D, a->has_b_out ? a->b_out.p : nullptr, out, D, nrp::RowTiling(), nrp::Epilogue(), true);
}

// -------------------------------------------------------------- caches
int nrp_cache_create(nrp_attn* attn, int batch, int cache_len, nrp_cache** out) {
  if (!attn || !out || batch <= 0 || cache_len <= 0) return fail(NRP_ERR_INVALID, "invalid cache arguments");
  if (check_device(attn->ctx)) return NRP_ERR_CUDA;
  auto* c = new nrp_cache;
  c->attn = attn;
  c->device = attn->ctx->device;
  c->B = batch;
  c->C = cache_len;
  c->D = attn->D;
  c->dtype = attn->dtype;
  const size_t n = static_cast<size_t>(batch) * cache_len * attn->D * esize(c->dtype);
  if (c->kc.ensure(n) || c->vc.ensure(n) || c->hc.ensure(n)) {
    delete c;
    return fail(NRP_ERR_NOMEM, "cache allocation failed");
  }
  cudaMemset(c->kc.p, 0, n);
  cudaMemset(c->vc.p, 0, n);
  cudaMemset(c->hc.p, 0, n);
  *out = c;
  return ok();
}

int nrp_cache_destroy(nrp_cache* cache) {
  if (cache) {
    // (its module may have been destroyed first: only the device number is used)
    cudaSetDevice(cache->device);
    delete cache;
    (void)cudaGetLastError();
  }
  return ok();
}

int nrp_cache_reset(nrp_cache* c, void* stream) {
  if (!c) return fail(NRP_ERR_INVALID, "null cache");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemsetAsync(c->kc.p, 0, c->kc.bytes, st));
  CUDA_TRY(cudaMemsetAsync(c->vc.p, 0, c->vc.bytes, st));
  CUDA_TRY(cudaMemsetAsync(c->hc.p, 0, c->hc.bytes, st));
  c->head = 0;
  return ok();
}

int nrp_cache_get_head(const nrp_cache* c, int* head) {
  if (!c || !head) return fail(NRP_ERR_INVALID, "null argument");
  *head = c->head;
  return ok();
}

int nrp_cache_set_head(nrp_cache* c, int head) {
  if (!c) return fail(NRP_ERR_INVALID, "null cache");
  if (head < 0 || head >= c->C) return fail(NRP_ERR_INVALID, "ring slot %d of %d", head, c->C);
  c->head = head;
  return ok();
}

int nrp_cache_export_h(nrp_cache* c, float* h, void* stream) {
  if (!c || !h) return fail(NRP_ERR_INVALID, "null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t es = esize(c->dtype);
  const size_t row = static_cast<size_t>(c->D) * es;
  const size_t pitch = row * c->C;
  void* dst = h;
  if (c->dtype != NRP_DTYPE_F32) {
    CUDA_TRY(c->tmp.ensure(pitch * c->B));
    dst = c->tmp.p;
  }
  // oldest frame first: slots head..C-1, then 0..head-1
  const int n1 = c->C - c->head;
  CUDA_TRY(cudaMemcpy2DAsync(dst, pitch, static_cast<uint8_t*>(c->hc.p) + c->head * row, pitch,
                             n1 * row, c->B, cudaMemcpyDeviceToDevice, st));
  if (c->head)
    CUDA_TRY(cudaMemcpy2DAsync(static_cast<uint8_t*>(dst) + n1 * row, pitch, c->hc.p, pitch,
                               c->head * row, c->B, cudaMemcpyDeviceToDevice, st));
  if (c->dtype != NRP_DTYPE_F32)
    CUDA_TRY(nrp::launch_bf16_to_f32(c->tmp.as<__nv_bfloat16>(), h,
                                     static_cast<int64_t>(c->B) * c->C * c->D, st));
  return ok();
}

int nrp_cache_import_h(nrp_cache* c, const float* h, void* stream) {
  if (!c || !h) return fail(NRP_ERR_INVALID, "null argument");
  nrp_attn* a = c->attn;
  if (a->dtype != c->dtype) return fail(NRP_ERR_INVALID, "module dtype changed since the cache was created");
  int rc = sync_params(a);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = c->D;
  const size_t n = static_cast<size_t>(c->B) * c->C * D;
  if (c->dtype == NRP_DTYPE_F32) {
    CUDA_TRY(cudaMemcpyAsync(c->hc.p, h, n * 4, cudaMemcpyDeviceToDevice, st));
  } else {
    CUDA_TRY(nrp::launch_f32_to_bf16(h, c->hc.as<__nv_bfloat16>(), static_cast<int64_t>(n), st));
  }
  c->head = 0;
  // K/V of the cached frames: the K and V blocks of the fused projection
  const size_t es = esize(c->dtype);
  const size_t DD = static_cast<size_t>(D) * D;
  const int M = c->B * c->C;
  for (int which = 1; which <= 2; ++which) {
    const void* w = static_cast<const uint8_t*>(a->w_qkv.p) + (a->qkv_quant ? which * DD : which * DD * es);
    const void* s = a->qkv_quant ? static_cast<const uint8_t*>(a->s_qkv.p) + which * static_cast<size_t>(D) * (D / 64) * 2 : nullptr;
    const void* z = a->qkv_quant ? static_cast<const uint8_t*>(a->z_qkv.p) + which * static_cast<size_t>(D) * (D / 64) * 2 : nullptr;
    const void* bias = a->has_b_qkv ? static_cast<const uint8_t*>(a->b_qkv.p) + which * D * es : nullptr;
    // (an address inside the fused codes: not kept, the module forgets only
    // the buffer's own address)
    rc = run_linear(a->ctx, st, c->dtype, c->hc.p, M, D, w, a->qkv_quant, s, z, D, bias,
                    which == 1 ? c->kc.p : c->vc.p, D);
    if (rc) return rc;
  }
  return ok();
}

int nrp_attn_forward_with_cache(nrp_attn* a, void* stream, const void* x, int B, int T,
                                const void* pos_emb, nrp_cache* c, int filled, int valid,
                                const nrp_att_context* context, void* out) {
  return nrp::attn_forward_with_cache(a, static_cast<cudaStream_t>(stream), x, B, T, pos_emb, c,
                                      filled, valid, context, out, nrp::Epilogue());
}

}  // extern "C"

int nrp::attn_forward_with_cache(nrp_attn* a, cudaStream_t st, const void* x, int B, int T,
                                 const void* pos_emb, nrp_cache* c, int filled, int valid,
                                 const nrp_att_context* context, void* out,
                                 const nrp::Epilogue& out_ep) {
  if (!a || !x || !pos_emb || !c || !out) return fail(NRP_ERR_INVALID, "null argument");
  if (c->attn != a) return fail(NRP_ERR_INVALID, "cache belongs to another module");
  if (B != c->B || T <= 0) return fail(NRP_ERR_INVALID, "batch %d / seq_len %d do not match the cache", B, T);
  if (a->dtype != c->dtype) return fail(NRP_ERR_INVALID, "module dtype changed since the cache was created");
  nrp_context* ctx = a->ctx;
  if (check_device(ctx)) return NRP_ERR_CUDA;
  int rc = sync_params(a);
  if (rc) return rc;
  const int D = a->D, C = c->C, Tk = C + T, P = 2 * Tk - 1;
  const size_t es = esize(a->dtype);
  const size_t BT = static_cast<size_t>(B) * T;
  CUDA_TRY(a->qkv.ensure(BT * 3 * D * es));
  CUDA_TRY(a->cbuf.ensure(BT * D * es));
  rc = run_linear(ctx, st, a->dtype, x, static_cast<int>(BT), D, a->w_qkv.p, a->qkv_quant,
                  a->s_qkv.p, a->z_qkv.p, 3 * D, a->has_b_qkv ? a->b_qkv.p : nullptr, a->qkv.p, 3 * D, nrp::RowTiling(), nrp::Epilogue(), true);
  if (rc) return rc;
  if (a->spos_len != P) {  // 749-761: projected positions reused per pos_len
    CUDA_TRY(a->spos.ensure(static_cast<size_t>(P) * D * es));
    rc = run_linear(ctx, st, a->dtype, pos_emb, P, D, a->w_pos.p, a->pos_quant, a->s_pos.p,
                    a->z_pos.p, D, nullptr, a->spos.p, D, nrp::RowTiling(), nrp::Epilogue(), true);
    if (rc) return rc;
    a->spos_len = P;
  }
  nrp::StreamMaskDev sm{};
  sm.has = 1;
  sm.cache_len = C;
  sm.filled = std::min(std::max(filled, 0), C);
  sm.valid = std::min(std::max(valid, 0), T);
  sm.ctx_has = context ? 1 : 0;
  sm.left = context ? context->left : -1;
  sm.right = context ? context->right : -1;
  sm.chunked = context ? context->chunked : 0;
  // slide the window: the first q_keep new frames replace the oldest
  // (661-684); more than C of them keep only the newest C (992-996)
  const int q_keep = std::max(T - a->cache_drop, 0);
  const int n_app = std::min(q_keep, C);
  const int src0 = q_keep - n_app;
  bool appended = false;
  {
    ProfScope ps_attn(ctx, NRP_KERNEL_ATTN_STREAM, st);
    if (a->dtype == NRP_DTYPE_BF16 && nrp::stream_attn_supported(C, T, D, a->H)) {
      // tensor-core kernel; it also slides the ring when the chunk fits one CTA
      const bool fuse = T <= 16;
      const auto* q = a->qkv.as<__nv_bfloat16>();
      CUDA_TRY(nrp::launch_relpos_attn_stream_mma(
          q, c->kc.as<__nv_bfloat16>(), c->vc.as<__nv_bfloat16>(), c->hc.as<__nv_bfloat16>(),
          static_cast<const __nv_bfloat16*>(x), C, c->head, fuse ? n_app : 0, src0,
          a->spos.as<__nv_bfloat16>(), a->u_dev.as<float>(), a->v_dev.as<float>(), sm,
          a->cbuf.as<__nv_bfloat16>(), B, T, D, a->H, ctx->d_err, st));
      appended = fuse;
    } else if (a->dtype == NRP_DTYPE_BF16) {
      const auto* q = a->qkv.as<__nv_bfloat16>();
      CUDA_TRY(nrp::launch_relpos_attn_stream_simt<__nv_bfloat16>(
          q, 3 * D, q + D, q + 2 * D, 3 * D, c->kc.as<__nv_bfloat16>(), c->vc.as<__nv_bfloat16>(),
          C, c->head, a->spos.as<__nv_bfloat16>(), a->u_dev.as<float>(), a->v_dev.as<float>(), sm,
          a->cbuf.as<__nv_bfloat16>(), B, T, D, a->H, st));
    } else {
      const auto* q = a->qkv.as<float>();
      CUDA_TRY(nrp::launch_relpos_attn_stream_simt<float>(
          q, 3 * D, q + D, q + 2 * D, 3 * D, c->kc.as<float>(), c->vc.as<float>(), C, c->head,
          a->spos.as<float>(), a->u_dev.as<float>(), a->v_dev.as<float>(), sm,
          a->cbuf.as<float>(), B, T, D, a->H, st));
    }
  }
  if (n_app > 0 && !appended) {
    ProfScope ps(ctx, NRP_KERNEL_RING_APPEND, st);
    const uint8_t* qkv = static_cast<const uint8_t*>(a->qkv.p);
    const int64_t sb = static_cast<int64_t>(T) * 3 * D, sr = 3 * D;
    CUDA_TRY(nrp::launch_ring_append(qkv + (src0 * 3 * D + D) * es, sb, sr, c->kc.p,
                                     static_cast<int64_t>(C) * D, C, c->head, n_app, B, D,
                                     static_cast<int>(es), st));
    CUDA_TRY(nrp::launch_ring_append(qkv + (src0 * 3 * D + 2 * D) * es, sb, sr, c->vc.p,
                                     static_cast<int64_t>(C) * D, C, c->head, n_app, B, D,
                                     static_cast<int>(es), st));
    CUDA_TRY(nrp::launch_ring_append(static_cast<const uint8_t*>(x) + src0 * D * es,
                                     static_cast<int64_t>(T) * D, D, c->hc.p,
                                     static_cast<int64_t>(C) * D, C, c->head, n_app, B, D,
                                     static_cast<int>(es), st));
  }
  if (n_app > 0) c->head = (c->head + n_app) % C;
  return run_linear(ctx, st, a->dtype, a->cbuf.p, static_cast<int>(BT), D, a->w_out.p,
                    a->out_quant, a->s_out.p, a->z_out.p, D, a->has_b_out ? a->b_out.p : nullptr,
                    out, D, nrp::RowTiling(), out_ep, true);
}

extern "C" {

// ------------------------------------------------------------ profiling
int nrp_profile_enable(nrp_context* ctx, int enable) {
  if (!ctx) return fail(NRP_ERR_INVALID, "null context");
  ctx->prof = enable != 0;
  return ok();
}

int nrp_profile_reset(nrp_context* ctx) {
  if (!ctx) return fail(NRP_ERR_INVALID, "null context");
  int rc = prof_collect(ctx);
  for (int k = 0; k < NRP_KERNEL_KINDS; ++k) {
    ctx->prof_ms[k] = 0.0;
    ctx->prof_n[k] = 0;
  }
  ctx->prof_log.clear();
  return rc;
}

int nrp_profile_launches(nrp_context* ctx, int* kinds, float* ms, int64_t capacity,
                         int64_t* count) {
  if (!ctx || !count || capacity < 0 || (capacity > 0 && (!kinds || !ms)))
    return fail(NRP_ERR_INVALID, "invalid profile log arguments");
  int rc = prof_collect(ctx);
  if (rc) return rc;
  const int64_t n = static_cast<int64_t>(ctx->prof_log.size());
  for (int64_t i = 0; i < n && i < capacity; ++i) {
    kinds[i] = ctx->prof_log[i].first;
    ms[i] = ctx->prof_log[i].second;
  }
  *count = n;
  return ok();
}

int nrp_profile_read(nrp_context* ctx, int kind, int64_t* launches, double* total_ms) {
  if (!ctx || kind < 0 || kind >= NRP_KERNEL_KINDS) return fail(NRP_ERR_INVALID, "bad kernel kind");
  int rc = prof_collect(ctx);
  if (rc) return rc;
  if (launches) *launches = ctx->prof_n[kind];
  if (total_ms) *total_ms = ctx->prof_ms[kind];
  return ok();
}

// ------------------------------------------------------- linear entries
int nrp_linear(nrp_context* ctx, void* stream, int dtype, const void* x, int M, int K,
               const void* w, int N, const void* bias, void* y) {
  if (!ctx || !x || !w || !y || M < 0 || K <= 0 || N <= 0) return fail(NRP_ERR_INVALID, "invalid linear arguments");
  if (dtype != NRP_DTYPE_F32 && dtype != NRP_DTYPE_BF16) return fail(NRP_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (check_device(ctx)) return NRP_ERR_CUDA;
  return run_linear(ctx, static_cast<cudaStream_t>(stream), dtype, x, M, K, w, false, nullptr,
                    nullptr, N, bias, y, N, nrp::RowTiling(), nrp::Epilogue(), false, false);
}

int nrp_qlinear(nrp_context* ctx, void* stream, const void* x, int M, int K, const uint32_t* wq,
                const void* scales, const void* biases, int N, int group_size, int bits,
                const void* bias, void* y) {
  if (!ctx || !x || !wq || !scales || !biases || !y || M < 0 || K <= 0 || N <= 0)
    return fail(NRP_ERR_INVALID, "invalid quantized linear arguments");
  if (bits != 8 || group_size != 64)
    return fail(NRP_ERR_UNSUPPORTED, "quantized linear: bits %d group %d (supported: 8, 64)", bits, group_size);
  if (check_device(ctx)) return NRP_ERR_CUDA;
  return run_linear(ctx, static_cast<cudaStream_t>(stream), NRP_DTYPE_BF16, x, M, K, wq, true,
                    scales, biases, N, bias, y, N, nrp::RowTiling(), nrp::Epilogue(), false, false);
}

}  // extern "C"
