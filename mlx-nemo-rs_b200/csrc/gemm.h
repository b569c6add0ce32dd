// gemm.h -- launchers of the library's kernels (internal, not the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <vector>

namespace nrp {

// Launches `kernel` with programmatic stream serialization: it may start
// while the previous kernel in the stream finishes, and waits for that
// kernel's grid (pdl_wait) before touching memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory limit once per device (function
// attributes belong to each device's context; `done` holds one bit per
// device ordinal).
template <typename F>
cudaError_t smem_attr_once(F* func, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// ---- TMA descriptors (driver entry point resolved through the runtime) ----
// Row-major 2-D tensor [outer, inner] of `elem_bytes` elements, row stride in
// bytes; box (box_inner, box_outer); 128-byte swizzle when box_inner *
// elem_bytes == 128.  Returns false when the driver rejects the map.
bool make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                  uint32_t box_outer, bool swizzle128);
// 3-D tensor [d2, d1, d0] (d0 innermost) with strides in bytes for d1, d2.
bool make_tmap_3d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                  uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                  bool swizzle128);

// Row tiling of a GEMM whose M rows are B utterances of T frames (T > 0):
// row tiles never straddle utterances, and with len != null a tile whose
// first frame is at or past len[b] (device int32 [B]) is skipped -- its
// output rows are written as zeros.  T == 0: flat rows.  In the batched
// form the x map is 3-D [B][T][K] with box (64, 128, 1).
struct RowTiling {
  const int32_t* len = nullptr;
  int T = 0;
  int B = 0;
  // Output rows of utterance b start at y + b * y_bstride (elements); 0
  // means T * ldy (utterances stacked).  A time-major output [T][B][N] is
  // ldy = B * N, y_bstride = N.  Rows t >= T are never written.
  int64_t y_bstride = 0;
  // Input rows of utterance b start at x + b * x_bstride (elements, a
  // multiple of 8); 0 means T * K.
  int64_t x_bstride = 0;
};

// What the GEMM epilogue does with v = acc + bias (f32) before the single
// rounding to bf16:
//   kEpiBias      y = v
//   kEpiSilu      y = v * sigmoid(v)                      (FeedForward::forward)
//   kEpiResidual  y = res + alpha * v; res may alias y     (the block's residuals)
//   kEpiGlu       W's rows come in 256-row tiles [128 value rows | their 128
//                 gate rows]; tile k writes output columns [128k, 128k + 128)
//                 = value * sigmoid(gate), so y has N/2 columns; with len,
//                 rows t >= len[b] are written as zeros (ConvolutionModule's
//                 GLU and padded-frame zeroing)
//   kEpiRelu      y = max(round(acc) + bias, 0): a pointwise conv whose output
//                 is rounded before its bias add, then ReLU (the subsampling)
enum EpiMode { kEpiBias = 0, kEpiSilu = 1, kEpiResidual = 2, kEpiGlu = 3, kEpiRelu = 4 };
struct Epilogue {
  int mode = kEpiBias;
  const __nv_bfloat16* res = nullptr;
  int64_t ldr = 0;     // residual row stride (elements)
  int64_t res_bs = 0;  // residual batch stride under batched tiling (0: T * ldr)
  float alpha = 1.f;
  const int32_t* len = nullptr;  // kEpiGlu, batched tiling
};

// ---- tcgen05 GEMM: y[M,N] = x[M,K] . W[N,K]^T (+ bias) ----
// x map: bf16 [M, K], box (64, 128), swizzle 128.  w: bf16 [N, K] row-major
// (the launcher makes its map for the tile width it picks).  Requires
// K % 64 == 0 and N % 32 == 0.  w_early: no kernel still running on the
// stream writes w (weights uploaded or dequantised ahead), so the kernel may
// load its first W stages before waiting on the previous kernel.
int gemm_smem_bytes();
cudaError_t launch_gemm_bf16(const CUtensorMap& map_x, const void* w,
                             const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int M, int N,
                             int K, int num_sms, int* err, cudaStream_t stream,
                             RowTiling rt = RowTiling(), const Epilogue& ep = Epilogue(),
                             bool w_early = false);
// Quantised W: MLX affine 8-bit, group 64: wq [N, K] bytes (the packed u32
// words read as little-endian bytes), scales/biases bf16 [N, K/64].
cudaError_t launch_gemm_q8(const CUtensorMap& map_x, const uint8_t* wq, const __nv_bfloat16* qs,
                           const __nv_bfloat16* qb, const __nv_bfloat16* bias, __nv_bfloat16* y,
                           int ldy, int M, int N, int K, int num_sms, int* err,
                           cudaStream_t stream, RowTiling rt = RowTiling(),
                           const Epilogue& ep = Epilogue());

// ---- large-M quantised GEMM, first half: w[N,K] bf16 = dequant(wq) ----
// (then the bf16 GEMM): each weight is dequantised once per call instead of
// once per 128-row tile.  Requires K % 64 == 0.
cudaError_t launch_dequant_q8(const uint8_t* wq, const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                              __nv_bfloat16* w, int N, int K, int num_sms, cudaStream_t stream);
// Several weights in one launch (at most kMaxDeqJobs).
struct DeqJob {
  const uint8_t* wq;
  const __nv_bfloat16* qs;
  const __nv_bfloat16* qb;
  __nv_bfloat16* w;
  int N, K;
};
constexpr int kMaxDeqJobs = 12;
struct DeqBatch {
  DeqJob job[kMaxDeqJobs];
  int64_t begin16[kMaxDeqJobs + 1];  // first 16-weight unit of each job, then the total
  int n;
};
cudaError_t launch_dequant_q8_batch(const DeqJob* jobs, int n, int num_sms, cudaStream_t stream);

// ---- small-M quantised GEMM (HBM-bound regime): y[M,N] for M <= 256 ----
// x bf16 [M, K] (row stride K), wq [N, K] bytes, scales/biases bf16
// [N, K/64]; epilogues bias, SiLU, residual (res row stride ldr) and ReLU
// (not GLU).  x and wq 16-byte aligned, K % 64 == 0.
// Each CTA stages its 8..32 code rows in shared memory (K <= kQSmallMaxK).
// err: the context's device error word (a bulk copy that never lands is
// reported there, after a bounded wait).
constexpr int kQSmallMaxM = 256;
constexpr int kQSmallMaxK = 8192;
constexpr int kQSmallMaxSmem = 200 * 1024;
bool qgemm_small_supported(int M, int K, const void* x, const void* wq, const Epilogue& ep);
cudaError_t launch_qgemm_small(const __nv_bfloat16* x, int M, int K, const uint8_t* wq,
                               const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                               const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int N,
                               int num_sms, int* err, cudaStream_t stream,
                               const Epilogue& ep = Epilogue());

// ---- fp32 GEMM (fp32 module dtype): y = x . W^T (+ bias) ----
// The 3xTF32 tcgen05 kernel (gemm_tf32.cu) where gemm_tf32_supported (K a
// multiple of 32, x and w 16-byte aligned), else CUDA-core FFMA tiles.
// num_sms: the device's SM count; err: the context's device error word.
cudaError_t launch_gemm_f32(const float* x, int M, int K, const float* w, int N,
                            const float* bias, float* y, int ldy, int num_sms, int* err,
                            cudaStream_t stream);
bool gemm_tf32_supported(int M, int K, int N, const void* x, const void* w);
cudaError_t launch_gemm_tf32x3(const float* x, int M, int K, const float* w, int N,
                               const float* bias, float* y, int ldy, int num_sms, int* err,
                               cudaStream_t stream);

// ---- offline fused rel-pos attention, bf16, tcgen05 ----
// Where a launch's rows sit in the sequence.  All frame indices are global
// (frames of the whole utterance, Tg per utterance): the P row of query i
// and key j is Tg-1-i+j, key_len and the attention context are in global
// frames.  The launch computes query rows [q_lo, q_hi) of each utterance
// from a q|k|v buffer holding global frames [base, base + tbuf) (row of
// frame g of utterance b at (g - base) * qkv_ts + b * qkv_bs elements, each
// row q | k | v of D each), and keys only from [k_lo, k_hi) (the frames the
// buffer really holds).  p holds P rows [p_base, p_base + p_rows) of the
// global table; rows outside read as zero, so a windowed context needs only
// the rows its relative positions reach.
struct AttnGeom {
  int Tg;
  int tbuf, base;
  int64_t qkv_ts, qkv_bs;  // elements
  int q_lo, q_hi;
  int k_lo, k_hi;
  int p_base, p_rows;
  int out_base;     // global frame of output row 0
  int64_t out_bs;   // output batch stride (elements); rows are D apart
};
// The whole sequence in one buffer [B, T, 3D] and the full P table.
AttnGeom full_geom(int T, int D);
// Relative offsets d = j - i visible under a context: [dmin, dmax] within
// [-(T-1), T-1] (AttentionContext::block_mask, attention.rs:232-272).
struct AttnContextDev {
  int has, left, right, chunked;
};
void visible_offsets(const AttnContextDev& ctx, int T, int& dmin, int& dmax);

// q+u / q+v biases of every head as bf16 pairs (the attention kernel takes
// them as parameters): head h's u at w[128h .. 128h+64), its v at
// w[128h+64 .. 128h+128).
constexpr int kMaxHeadsUV = 16;
struct AttnUV {
  uint32_t w[kMaxHeadsUV * 128];
};

// qkv per geom; p: projected positions per geom; uv_host: [H][128] bf16
// pairs as in AttnUV (H <= kMaxHeadsUV); key_len: [B] int32 (key j visible
// iff j < max(key_len[b], 1)) or null; out: bf16, row of frame i of utterance
// b at b * out_bs + (i - out_base) * D.  sched: two ints, zero before the
// launch and left zero after it (the kernel's item counter); launches that
// share them must not run concurrently.
cudaError_t launch_relpos_attn_bf16(const void* qkv, const void* p, const uint32_t* uv_host,
                                    const int32_t* key_len, AttnContextDev ctx,
                                    const AttnGeom& g, void* out, int B, int H, int* err,
                                    int* sched, int num_sms, cudaStream_t stream);

// ---- generic CUDA-core attention (fp32 module dtype, any head_dim <= 128) ----
// q [B,Tq,D] (row stride ldq), k/v [B,Tk,D] (row strides ldk, ldv), p
// [2Tk-1, D]; masks: key_len (offline pad), ctx (offline context on absolute
// query positions q_off + i), stream (streaming mask: cache C, filled,
// valid, ctx).  Rows without a visible key are 0.
struct StreamMaskDev {
  int has;        // 1: streaming mask in force
  int cache_len;  // C (keys 0..C-1 come from the cache)
  int filled;     // keys j < C - filled are hidden
  int valid;      // query rows i >= valid see nothing
  int left, right, chunked, ctx_has;
};
cudaError_t launch_relpos_attn_f32(const float* q, int ldq, const float* k, int ldk,
                                   const float* v, int ldv, const float* p, const float* u,
                                   const float* vb, const int32_t* key_len, AttnContextDev ctx,
                                   StreamMaskDev sm, float* out, int B, int Tq, int Tk, int D,
                                   int H, cudaStream_t stream);

// ---- streaming attention against ring caches (T = float or bf16 storage) ----
// q [B, T, ldq] (head h at column h*dh), knew/vnew [B, T, ldkv] the chunk's
// projected keys/values, ring caches kc/vc [B, C, D] with the oldest frame at
// slot `head`, p [2(C+T)-1, D], out [B, T, D].
template <typename T>
cudaError_t launch_relpos_attn_stream_simt(const T* q, int ldq, const T* knew, const T* vnew,
                                           int ldkv, const T* kc, const T* vc, int C, int head,
                                           const T* p, const float* u, const float* vb,
                                           StreamMaskDev sm, T* out, int B, int T_, int D, int H,
                                           cudaStream_t stream);

// ---- Conformer block kernels (block_kernels.cu) ----
// LayerNorm over rows of D in {256, 512, 1024, 2048} (gamma/beta f32 [D]),
// optionally followed by SiLU; y may alias x.
cudaError_t launch_layernorm(const __nv_bfloat16* x, const float* gamma, const float* beta,
                             __nv_bfloat16* y, int64_t rows, int D, float eps, bool act_silu,
                             cudaStream_t stream);
// Depthwise conv over time of [B, T, D] (taps wt f32 [K][D], bias [D] or null),
// then y = act((conv + bias) * bn_scale + bn_shift) (scale/shift null = 1/0).
cudaError_t launch_dwconv(const __nv_bfloat16* x, const float* wt, const float* bias,
                          const float* bn_scale, const float* bn_shift, __nv_bfloat16* y, int B,
                          int T, int D, int K, bool causal, bool act_silu, cudaStream_t stream);
cudaError_t launch_scale(__nv_bfloat16* x, int64_t n, float s, cudaStream_t stream);
cudaError_t launch_transpose_btd(const __nv_bfloat16* x, __nv_bfloat16* y, int B, int T, int D,
                                 cudaStream_t stream);
// p[0 .. n) = v
cudaError_t launch_fill_i32(int32_t* p, int v, int n, cudaStream_t stream);

// ---- dw_striding subsampling convolutions (subsampling_kernels.cu) ----
// conv.0 (1 -> C, 3x3, stride 2, + bias, ReLU) of f32 mel frames, optionally
// fused with the first depthwise 3x3 stride-2 conv (+ bias).  Mel element
// (b, t, f) is mel[b * mel_bs + t * mel_ts + f * mel_fs]; frames t >= len[b]
// read as zero (len null: none).  pad = 1, or 2 for causal padding (left 2,
// right 1).  out NHWC bf16: [B][T2][F2][C] fused, else [B][T1][F1][C].
// Weights and biases come as MMA B fragments (subsample_conv0_frags,
// subsample_dw_frags).  Requires C % 32 == 0 and F1 <= 80.
struct SubConvArgs {
  const float* mel = nullptr;
  int64_t mel_bs = 0, mel_ts = 0, mel_fs = 0;
  const int32_t* len = nullptr;
  int len_off = 0;  // subtracted from len[b]: the first frame of a time chunk
  int T = 0, F = 0, T1 = 0, F1 = 0, T2 = 0, F2 = 0, C = 0, pad = 1;
  const uint32_t *f0 = nullptr, *f1 = nullptr;  // conv.0 and depthwise fragments
  __nv_bfloat16* out = nullptr;
};
// Fragment words per (group, lane): 12 (three 16-byte loads).
constexpr int kSubFragWords = 12;
// The host-side fragment layouts (bf16 pairs, low half first), for C
// channels: conv.0 w [C][9], b [C] -> [C/32][32 lanes][12]: for n-tile nt
// of the 32-channel group, words 3nt, 3nt+1 = (w[c][2t], w[c][2t+1]),
// (t == 0 ? w[c][8] : 0, 0) with c = 8 nt + g, word 3nt+2 = (b[8nt+2t],
// b[8nt+2t+1]) (g = lane / 4, t = lane % 4).  Depthwise w [C][9], b [C]
// -> [C/8][32 lanes][12]: words 2j, 2j+1 = tap 2j, 2j+1 of channel c on the
// diagonal (lane's pair (g == 2t ? v : 0, g == 2t+1 ? v : 0)), word 10 =
// the bias pair of channels 2t, 2t+1, word 11 = 0.
void subsample_conv0_frags(const float* w, const float* b, int C, std::vector<uint32_t>& out);
void subsample_dw_frags(const float* w, const float* b, int C, std::vector<uint32_t>& out);
size_t subsample_conv0_smem(int F1, bool fuse);
cudaError_t launch_subsample_conv0(const SubConvArgs& a, int B, bool fuse, cudaStream_t stream);
// y [B][To][Fo][C] = depthwise 3x3 stride 2 + bias of x [B][Ti][Fi][C]
// (both bf16 NHWC); C % 32 == 0.
cudaError_t launch_subsample_dw(const __nv_bfloat16* x, int B, int Ti, int Fi, int C, int pad,
                                const uint32_t* frag, __nv_bfloat16* y, int To, int Fo,
                                int num_sms, cudaStream_t stream);

// ---- streaming attention on tensor cores (attn_stream.cu), bf16 ----
// q|k|v [B, T, 3D] of the chunk, rings kc/vc/hc [B, C, D] (oldest frame at
// slot `head`), p [2(C+T)-1, D], out [B, T, D].  With n_app > 0 (only when
// T <= 16) the kernel also writes new frames src0 .. src0+n_app-1 (K, V
// and the attention input x) into ring slots head .. head+n_app-1 (mod C).
// err: the context's device error word (a bulk copy that never lands).
bool stream_attn_supported(int C, int T, int D, int H);
cudaError_t launch_relpos_attn_stream_mma(const __nv_bfloat16* qkv, const __nv_bfloat16* kc,
                                          const __nv_bfloat16* vc, __nv_bfloat16* hc,
                                          const __nv_bfloat16* x, int C, int head, int n_app,
                                          int src0, const __nv_bfloat16* p, const float* u,
                                          const float* v, StreamMaskDev sm, __nv_bfloat16* out,
                                          int B, int T, int D, int H, int* err,
                                          cudaStream_t stream);

// ---- small elementwise helpers ----
cudaError_t launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n,
                               cudaStream_t stream);
cudaError_t launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n,
                               cudaStream_t stream);
// Packed <-> padded frames.  One launch covers up to kMaxFrameUtts
// utterances: utterance u (padded batch index b0 + u) has len[u] rows, at
// packed rows [off[u], off[u] + len[u]) and padded rows [0, len[u]) of batch
// row b0 + u (bstride bytes apart).  to_padded: packed -> padded, else the
// reverse.  dev_lengths (may be null): len[u] is also written to
// dev_lengths[b0 + u].
constexpr int kMaxFrameUtts = 128;
struct FramesPlan {
  int64_t row_bytes, bstride, b0;
  int64_t off[kMaxFrameUtts];
  int32_t len[kMaxFrameUtts];
};
// A one-warp kernel that waits on an mbarrier nothing arrives on until
// budget_ns have passed, then records kDevTimeoutSelftest in *err and exits:
// the bounded-wait failure path, exercised without a fault.
cudaError_t launch_wait_expiry(int* err, uint64_t budget_ns, cudaStream_t stream);
cudaError_t launch_frames(void* padded, void* packed, const FramesPlan& plan, int n_utts,
                          bool to_padded, int32_t* dev_lengths, cudaStream_t stream);

// Ring append of rows: dst[b, (head + i) % C, :] = src[b, src_off + i, :] for
// i in [0, n), row length `cols` elements of `elem_bytes`.
cudaError_t launch_ring_append(const void* src, int64_t src_bstride, int64_t src_rstride,
                               void* dst, int64_t dst_bstride, int C, int head, int n, int B,
                               int cols, int elem_bytes, cudaStream_t stream);

}  // namespace nrp
