// internal.h -- helpers shared by the C ABI's translation units (api.cpp,
// block.cpp): error messages, per-launch profiling, the linear dispatcher
// and the attention forward with a caller-chosen output epilogue.
#pragma once

#include <cuda_runtime.h>
#include <string.h>

#include <cstdint>
#include <vector>

#include "gemm.h"
#include "handles.h"

namespace nrp {

// f32 -> bf16 bits, round to nearest even (NaN kept quiet).
inline uint16_t bf16_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u)
    return static_cast<uint16_t>((u >> 16) | ((u & 0xffff) ? 0x40 : 0));
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

inline float bf16_round(float x) {
  uint32_t u = static_cast<uint32_t>(bf16_bits(x)) << 16;
  float y;
  memcpy(&y, &u, 4);
  return y;
}

// Sets this thread's nrp_last_error() message (printf format); returns code.
int failf(int code, const char* fmt, ...);

inline cudaEvent_t take_event(nrp_context* c) {
  if (!c->pool.empty()) {
    cudaEvent_t e = c->pool.back();
    c->pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Scope guard: records start/stop events around one launch when enabled.
struct ProfScope {
  nrp_context* c;
  int kind;
  cudaStream_t st;
  cudaEvent_t a = nullptr;
  ProfScope(nrp_context* c_, int kind_, cudaStream_t st_) : c(c_), kind(kind_), st(st_) {
    if (c && c->prof) {
      a = take_event(c);
      cudaEventRecord(a, st);
    }
  }
  ~ProfScope() {
    if (a) {
      cudaEvent_t b = take_event(c);
      cudaEventRecord(b, st);
      c->recs.push_back({kind, a, b});
    }
  }
  ProfScope(const ProfScope&) = delete;
  ProfScope& operator=(const ProfScope&) = delete;
};

// y[M,N] (row stride ldy) = x[M,K] . W^T (+ bias) with the epilogue `ep`,
// dispatched as nrp_linear / the module projections are (bf16 tcgen05 GEMM,
// 8-bit GEMM, small-M GEMV, f32 CUDA-core GEMM).
// keep: the weight is module-owned, so its bf16 copy may be kept
// (nrp_context::deq_cache).
int linear(nrp_context* ctx, cudaStream_t st, int dtype, const void* x, int M, int K,
           const void* w, bool quant, const void* qs, const void* qb, int N, const void* bias,
           void* y, int ldy, const RowTiling& rt, const Epilogue& ep, bool keep = false);

// Drops the persistent bf16 copy of the quantised weight whose codes are at
// `codes` (before the codes are re-uploaded or freed).
void deq_forget(nrp_context* ctx, const void* codes);

// Uploads the module's parameters in its dtype if they changed.
int attn_sync(nrp_attn* a);

// nrp_attn_forward with `out_ep` as the epilogue of linear_out.
int attn_forward(nrp_attn* a, cudaStream_t st, const void* x, int B, int T, const void* pos_emb,
                 const int32_t* lengths, const nrp_att_context* context, void* out,
                 const Epilogue& out_ep);

// nrp_attn_forward_with_cache with `out_ep` as the epilogue of linear_out.
int attn_forward_with_cache(nrp_attn* a, cudaStream_t st, const void* x, int B, int T,
                            const void* pos_emb, nrp_cache* c, int filled, int valid,
                            const nrp_att_context* context, void* out, const Epilogue& out_ep);

// The module's cache_drop_size (nrp_attn_set_cache_drop_size).
int attn_cache_drop(const nrp_attn* a);

// Makes the context's device current.
int select_device(nrp_context* ctx);

// MLX affine dequantisation of a quantised Linear on the host (f32 [N, K]).
void dequant_linear_host(const Linear& L, int N, int K, std::vector<float>& w);

// The subsampling (subsampling.cpp): mel element (b, t, f) at mel[b * bs +
// t * ts + f * fs]; lengths device int32 [B] or null (mel mask).
int subsampling_run(nrp_subsampling* s, cudaStream_t st, const float* mel, int64_t bs, int64_t ts,
                    int64_t fs, int B, int T, const int32_t* lengths, void* out);
int subsampling_output_frames(const nrp_subsampling* s, int frames);
int subsampling_feat_in(const nrp_subsampling* s);

}  // namespace nrp
