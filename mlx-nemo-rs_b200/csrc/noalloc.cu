// noalloc.cu -- nrp_attn_forward_noalloc: the rel-pos MHA forward without any
// device allocation.
//
// nrp_attn_forward keeps its intermediate tensors (the fused q|k|v
// projections, the projected positions and the attention context) in
// buffers it grows with cudaMalloc.  Some callers cannot let a library call
// cudaMalloc: an audio thread with a real-time deadline cannot wait on it
// (it synchronises the device), and a host process whose device memory is
// handed out by another runtime's allocator has none to give.  For them
// this entry point takes the same inputs and output as nrp_attn_forward and
// places its intermediates in g_static_scratch, a fixed array in the
// library's own device memory, so the call allocates nothing.
//
// The array is kStaticScratchBytes (32 MiB).  It sits in a module of its own
// (this file has no kernels), which the CUDA runtime loads on the first use
// of the array: nrp_context_create makes that use (it looks the array's
// device address up), so every GPU with a context holds the array from then
// until the process exits, and no noalloc call loads anything.  Every call
// shares the array: a call overwrites what the previous call left there (it
// clears nothing because every byte it reads is written earlier in the same
// call), and two calls whose work overlaps on the GPU (different streams, or
// different modules on one device) race on it.  Callers serialise such calls
// themselves.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "gemm.h"
#include "handles.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

int report(int code, const char* fmt, long long a = 0, long long b = 0) {
  char buf[256];
  snprintf(buf, sizeof buf, fmt, a, b);
  return nrp::report_error(code, buf);
}

// Device address of g_static_scratch on `device`, looked up by
// nrp::noalloc_scratch_prepare when the device's first context was created.
void* scratch_address(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  return g_scratch_addr[device];
}

// Makes `device` current for the call and gives the caller's current device
// back when the call returns.
struct DeviceScope {
  int prev = -1;
  cudaError_t enter(int device) {
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    if (prev == device) {
      prev = -1;
      return cudaSuccess;
    }
    return cudaSetDevice(device);
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

#define TRY_CUDA(expr)                                                         \
  do {                                                                         \
    const cudaError_t e_ = (expr);                                             \
    if (e_ != cudaSuccess) {                                                   \
      (void)cudaGetLastError();                                                \
      return nrp::report_error(NRP_ERR_CUDA, cudaGetErrorString(e_));          \
    }                                                                          \
  } while (0)

// y[M,N] (row stride ldy) = x[M,K] . W^T (+ bias), with nothing allocated.
// The kernels are those nrp_attn_forward runs.  A quantised weight with many
// rows uses the bf16 copy an earlier allocating forward kept (the context's
// weight cache), as nrp_attn_forward does; without one, the 8-bit tcgen05
// GEMM dequantises it in its producer (correct, but it redoes the
// dequantisation per 128-row tile: about a fifth of the bf16 GEMM's rate).
int linear(nrp_context* ctx, cudaStream_t st, int dtype, const void* x, int M, int K,
           const void* w, bool quant, const void* qs, const void* qb, int N, const void* bias,
           void* y, int ldy) {
  if (M <= 0) return NRP_OK;
  if (dtype == NRP_DTYPE_F32) {
    TRY_CUDA(nrp::launch_gemm_f32(static_cast<const float*>(x), M, K, static_cast<const float*>(w),
                                  N, static_cast<const float*>(bias), static_cast<float*>(y), ldy,
                                  ctx->num_sms, ctx->d_err, st));
    return NRP_OK;
  }
  if (quant && nrp::qgemm_small_supported(M, K, x, w, nrp::Epilogue())) {
    TRY_CUDA(nrp::launch_qgemm_small(static_cast<const __nv_bfloat16*>(x), M, K,
                                     static_cast<const uint8_t*>(w),
                                     static_cast<const __nv_bfloat16*>(qs),
                                     static_cast<const __nv_bfloat16*>(qb),
                                     static_cast<const __nv_bfloat16*>(bias),
                                     static_cast<__nv_bfloat16*>(y), ldy, N, ctx->num_sms,
                                     ctx->d_err, st));
    return NRP_OK;
  }
  if (quant && M > nrp::kQSmallMaxM) {
    const auto it = ctx->deq_cache.find(w);
    if (it != ctx->deq_cache.end()) {
      w = it->second->p;
      quant = false;
    }
  }
  CUtensorMap mx;
  if (!nrp::make_tmap_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M,
                         static_cast<uint64_t>(K) * 2, 64, 128, true))
    return report(NRP_ERR_CUDA, "TMA descriptor for x rejected");
  if (quant) {
    TRY_CUDA(nrp::launch_gemm_q8(mx, static_cast<const uint8_t*>(w),
                                 static_cast<const __nv_bfloat16*>(qs),
                                 static_cast<const __nv_bfloat16*>(qb),
                                 static_cast<const __nv_bfloat16*>(bias),
                                 static_cast<__nv_bfloat16*>(y), ldy, M, N, K, ctx->num_sms,
                                 ctx->d_err, st));
    return NRP_OK;
  }
  TRY_CUDA(nrp::launch_gemm_bf16(mx, w, static_cast<const __nv_bfloat16*>(bias),
                                 static_cast<__nv_bfloat16*>(y), ldy, M, N, K, ctx->num_sms,
                                 ctx->d_err, st));
  return NRP_OK;
}

}  // namespace

namespace nrp {

int noalloc_scratch_prepare(int device) {
  if (device < 0 || device >= kMaxDevices)
    return report(NRP_ERR_UNSUPPORTED, "device %lld beyond the static scratch table", device);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[device]) return NRP_OK;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess || !p) {
    (void)cudaGetLastError();
    return report_error(NRP_ERR_CUDA, e != cudaSuccess ? cudaGetErrorString(e)
                                                       : "no device address for the static scratch");
  }
  g_scratch_addr[device] = p;
  return NRP_OK;
}

}  // namespace nrp

extern "C" int nrp_attn_forward_noalloc(nrp_attn* a, void* stream, const void* x, int B, int T,
                                        const void* pos_emb, const int32_t* lengths,
                                        const nrp_att_context* context, void* out) {
  if (!a || !x || !pos_emb || !out) return report(NRP_ERR_INVALID, "null argument");
  if (B <= 0 || T <= 0) return report(NRP_ERR_INVALID, "empty input [%lld, %lld]", B, T);
  if (a->dirty)
    return report(NRP_ERR_INVALID,
                  "the module's parameters are not on the device yet: one nrp_attn_forward or "
                  "nrp_attn_forward_with_cache call (which allocates them) must come first");
  nrp_context* ctx = a->ctx;
  DeviceScope scope;
  TRY_CUDA(scope.enter(ctx->device));
  const int D = a->D, P = 2 * T - 1;
  const size_t es = a->dtype == NRP_DTYPE_BF16 ? 2 : 4;
  const size_t BT = static_cast<size_t>(B) * T;
  nrp::AttnContextDev cd{0, -1, -1, 0};
  if (context) cd = {1, context->left, context->right, context->chunked};
  // bf16 projects only the P rows the context's relative positions reach
  // (257 for a (128, 128) window), as nrp_attn_forward; f32 all 2T-1
  nrp::AttnGeom g = nrp::full_geom(T, D);
  if (a->dtype == NRP_DTYPE_BF16) {
    int dmin, dmax;
    nrp::visible_offsets(cd, T, dmin, dmax);
    g.p_base = T - 1 + dmin;
    g.p_rows = dmax - dmin + 1;
  }
  const size_t qkv_bytes = round256(BT * 3 * D * es);
  const size_t ctx_bytes = round256(BT * D * es);
  const size_t pos_bytes =
      round256(static_cast<size_t>(a->dtype == NRP_DTYPE_BF16 ? g.p_rows : P) * D * es);
  const size_t need = qkv_bytes + ctx_bytes + pos_bytes;
  if (need > kStaticScratchBytes)
    return report(NRP_ERR_INVALID,
                  "batch x seq_len needs %lld bytes of intermediates, more than the %lld-byte "
                  "static scratch of nrp_attn_forward_noalloc (use nrp_attn_forward)",
                  static_cast<long long>(need), static_cast<long long>(kStaticScratchBytes));
  void* base = scratch_address(ctx->device);
  if (!base)
    return report(NRP_ERR_INVALID,
                  "no static scratch address for device %lld (no context was created on it)",
                  ctx->device);
  uint8_t* qkv = static_cast<uint8_t*>(base);
  uint8_t* cbuf = qkv + qkv_bytes;
  uint8_t* pbuf = cbuf + ctx_bytes;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = linear(ctx, st, a->dtype, x, static_cast<int>(BT), D, a->w_qkv.p, a->qkv_quant,
                  a->s_qkv.p, a->z_qkv.p, 3 * D, a->has_b_qkv ? a->b_qkv.p : nullptr, qkv, 3 * D);
  if (rc) return rc;
  if (a->dtype == NRP_DTYPE_BF16) {
    rc = linear(ctx, st, a->dtype,
                static_cast<const uint8_t*>(pos_emb) + static_cast<size_t>(g.p_base) * D * es,
                g.p_rows, D, a->w_pos.p, a->pos_quant, a->s_pos.p, a->z_pos.p, D, nullptr, pbuf,
                D);
    if (rc) return rc;
    TRY_CUDA(nrp::launch_relpos_attn_bf16(qkv, pbuf, a->uv_packed.data(), lengths, cd, g, cbuf,
                                          B, a->H, ctx->d_err, nrp::sched_slot(ctx),
                                          ctx->num_sms, st));
  } else {
    rc = linear(ctx, st, a->dtype, pos_emb, P, D, a->w_pos.p, a->pos_quant, a->s_pos.p,
                a->z_pos.p, D, nullptr, pbuf, D);
    if (rc) return rc;
    const float* q = reinterpret_cast<const float*>(qkv);
    nrp::StreamMaskDev none{};
    TRY_CUDA(nrp::launch_relpos_attn_f32(q, 3 * D, q + D, 3 * D, q + 2 * D, 3 * D,
                                         reinterpret_cast<const float*>(pbuf),
                                         a->u_dev.as<float>(), a->v_dev.as<float>(), lengths, cd,
                                         none, reinterpret_cast<float*>(cbuf), B, T, T, D, a->H,
                                         st));
  }
  return linear(ctx, st, a->dtype, cbuf, static_cast<int>(BT), D, a->w_out.p, a->out_quant,
                a->s_out.p, a->z_out.p, D, a->has_b_out ? a->b_out.p : nullptr, out, D);
}
