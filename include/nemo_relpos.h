/*
 * nemo_relpos.h -- C ABI of libnemo_relpos.so, a B200 (sm_100a)
 * implementation of the FastConformer encoder's relative-position
 * multi-head self-attention of animaslabs/mlx-nemo-rs (crate mlx-voice).
 *
 * The ABI replaces the reference's `internals` attention-module API and its
 * streaming-cache structs; each declaration names the reference item
 * (file:line, paths relative to the reference project root) it stands in
 * for.  Conventions:
 *   - every function returns an int status: NRP_OK (0) or a negative
 *     NRP_ERR_* code; nrp_last_error() gives this thread's last message;
 *   - tensors are row-major; "device" pointers are caller-owned CUDA memory
 *     on the context's device; "host" pointers are read during the call;
 *   - device work is queued on the caller's cudaStream_t (passed as void*,
 *     NULL = legacy default stream).  A call synchronises nothing once the
 *     library's workspace has grown to the shapes it sees: a call with a
 *     larger shape than any before grows the module's intermediate buffers
 *     with cudaMalloc (which synchronises the device), and a quantised
 *     weight's first use at 256 or more rows makes its kept bf16 copy
 *     (cudaMalloc, then one cudaStreamSynchronize of the caller's stream;
 *     see nrp_context_set_weight_cache).  Warm a module up once at its
 *     largest shape before latency-critical use or stream capture, or use
 *     nrp_attn_forward_noalloc;
 *   - every call that launches work makes its context's device current on
 *     the calling thread (nrp_attn_forward_noalloc restores the caller's);
 *   - a handle is used by one host thread at a time (the reference's
 *     `&mut self` methods); one device per context.
 */
#ifndef NEMO_RELPOS_H
#define NEMO_RELPOS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NRP_ABI_VERSION 1

/* Status codes (the reference's core::error::Error kinds, src/core/error.rs:7-60). */
#define NRP_OK 0
#define NRP_ERR_INVALID -1     /* bad argument or shape (Error::Model / ShapeMismatch) */
#define NRP_ERR_CUDA -2        /* CUDA runtime/driver error (Error::Mlx's role) */
#define NRP_ERR_UNSUPPORTED -3 /* configuration not implemented (Error::NotImplemented) */
#define NRP_ERR_NOMEM -4       /* device allocation failed */
#define NRP_ERR_DEVICE -5      /* a kernel reported a bounded wait that expired */

typedef enum { NRP_DTYPE_F32 = 0, NRP_DTYPE_BF16 = 1 } nrp_dtype;

/* Which projection of RelPositionMultiHeadAttention (attention.rs:333-342). */
typedef enum {
  NRP_LINEAR_Q = 0,
  NRP_LINEAR_K = 1,
  NRP_LINEAR_V = 2,
  NRP_LINEAR_OUT = 3,
  NRP_LINEAR_POS = 4
} nrp_linear_id;

/* AttentionContext (attention.rs:210-216): left/right frames, chunked = the
 * "chunked_limited" style. */
typedef struct {
  int32_t left;
  int32_t right;
  int32_t chunked;
} nrp_att_context;

/* StreamingConfig (src/asr/streaming/core.rs:27-67). */
typedef struct {
  int32_t chunk_size[2];
  int32_t shift_size[2];
  int32_t cache_drop_size;
  int32_t last_channel_cache_size;
  int32_t last_time_cache_size;
  int32_t valid_out_len;
  int32_t pre_encode_cache_size[2];
  int32_t drop_extra_pre_encoded;
  int32_t lookahead_frames;
  int32_t mode_idx;
  int32_t left_context;
  int32_t right_context;
} nrp_streaming_config;

typedef struct nrp_context nrp_context;
typedef struct nrp_attn nrp_attn;
typedef struct nrp_cache nrp_cache;

/* ------------------------------------------------------------- library */
int nrp_abi_version(void);
/* Message of this thread's last failed call ("" if none). */
const char* nrp_last_error(void);

/* ------------------------------------------- host-side logic (no device) */

/* RelPositionalEncoding::get_encoding (attention.rs:131-177) of a table
 * built by RelPositionalEncoding::new(d_model, max_len, _)
 * (attention.rs:35-51, create_pe 59-103): writes [2*seq_len-1, d_model] f32
 * for positions (seq_len-1)..-(seq_len-1).  seq_len == 0 is an error
 * (132-136); seq_len > max_len rebuilds the table at seq_len (137-145). */
int nrp_pe_encoding_host(int d_model, int max_len, int seq_len, float* out);

/* RelPositionalEncoding::xscale (attention.rs:36-40, 186-188). */
float nrp_pe_xscale(int d_model, int xscaling);

/* AttentionContext::new (attention.rs:220-227): writes *out and returns 1
 * ("Some"), or returns 0 ("None") when left < 0 and right < 0.  style is
 * "regular" or "chunked_limited". */
int nrp_att_context_new(int left, int right, const char* style, nrp_att_context* out);

/* AttentionContext::block_mask (attention.rs:232-272) as visibility bytes
 * vis[(i-start)*seq_len + j] (1 = visible). */
int nrp_block_mask_host(const nrp_att_context* context, int start, int end, int seq_len,
                        uint8_t* vis);

/* key_padding_mask (attention.rs:280-294): returns 0 ("None") when no frame
 * is padding, else 1 and, when mask != NULL, writes the additive mask
 * [batch, seq_len] (0 or -inf; each row keeps max(len,1) keys). */
int nrp_key_padding_mask_host(const int32_t* lengths, int batch, int seq_len, float* mask);

/* create_attention_mask (src/asr/modules/encoders/conformer.rs:97-221):
 * vis [tensor_seq_len, max_audio_length] for the query rows of the current
 * chunk.  context == NULL means no att_context_size. */
int nrp_streaming_mask_host(const nrp_att_context* context, int max_audio_length, int cache_len,
                            int filled_cache_len, int tensor_seq_len, int valid_seq_len,
                            uint8_t* vis);

/* compute_streaming_config (src/asr/streaming/core.rs:247-362) for one
 * mode's (left, right) context. */
int nrp_streaming_config_compute(int left, int right, int chunked, int n_layers,
                                 int subsampling_factor, int conv_kernel_size, int causal_conv,
                                 int mode_idx, int max_context, nrp_streaming_config* out);

/* ------------------------------------------------------------- context */
/* One CUDA device; owns the device error word kernels report into. */
int nrp_context_create(int device, nrp_context** out);
int nrp_context_destroy(nrp_context* ctx);
/* Synchronises `stream`, then reads and clears the device error word:
 * NRP_ERR_DEVICE if a kernel gave up on a bounded wait since the last check. */
int nrp_context_check(nrp_context* ctx, void* stream);
/* Failure-path self-test: queues on `stream` a kernel that waits on a
 * barrier nothing ever arrives on for budget_us microseconds (1 .. 10^6) and
 * then gives up, the way every kernel's bounded wait does.  The next
 * nrp_context_check returns NRP_ERR_DEVICE and clears the error; the context
 * stays usable.  No GPU fault is involved. */
int nrp_context_selftest_wait_expiry(nrp_context* ctx, void* stream, int budget_us);
/* Quantised linears with 256 or more rows run as bf16 GEMMs over their
 * weight's dequantised copy.  With the weight cache on (the default), each
 * weight's copy is made on its first such use and kept until its module
 * re-uploads or frees the weight (2 bytes per parameter of device memory:
 * 0.6 GB for a 24-layer d_model-1024 encoder); off, the copy is remade in a
 * scratch buffer on every call (the reference's memory footprint). */
int nrp_context_set_weight_cache(nrp_context* ctx, int enable);

/* get_encoding on the device in the given dtype (f32 table cast like
 * RelPositionalEncoding::set_dtype, attention.rs:180-183): dev_out
 * [2*seq_len-1, d_model]. */
int nrp_pe_encoding(nrp_context* ctx, int d_model, int max_len, int seq_len, int dtype,
                    void* dev_out, void* stream);

/* ------------------------------------------------------ attention module */
/* RelPositionMultiHeadAttention::new (attention.rs:367-406): zero
 * parameters, dtype f32.  head_dim = d_model / n_heads. */
int nrp_attn_create(nrp_context* ctx, int d_model, int n_heads, int use_bias, nrp_attn** out);
int nrp_attn_destroy(nrp_attn* attn);

/* RelPositionMultiHeadAttention::set_dtype (attention.rs:409-423) with
 * LinearLayer::cast (src/core/quantization.rs:92-114): weights, biases,
 * quantisation scales/biases and pos_bias_u/v are rounded to dtype; clears
 * the cached streaming positions. */
int nrp_attn_set_dtype(nrp_attn* attn, int dtype);

/* The pub field cache_drop_size (attention.rs:349-350), set by
 * ConformerEncoder::setup_streaming (conformer.rs:812-817). */
int nrp_attn_set_cache_drop_size(nrp_attn* attn, int cache_drop_size);

/* load_weights for one projection, Standard arm (attention.rs:863-880 via
 * Weights::fetch_linear, src/core/loading.rs:151-158, and load_linear_layer,
 * quantization.rs:327-345): weight host f32 [d_model, d_model] ([out, in]),
 * bias host f32 [d_model] or NULL (linear_pos has none). */
int nrp_attn_load_linear(nrp_attn* attn, int which, const float* weight, const float* bias);

/* Quantized arm (load_linear_layer, quantization.rs:299-326; MLX layout
 * doc 4-8): wq host u32 [d_model, d_model*bits/32], scales/biases host f32
 * [d_model, d_model/group_size] (the file's F16 values widened), bias host
 * f32 [d_model] or NULL.  Supported: bits 8, group_size 64. */
int nrp_attn_load_linear_quantized(nrp_attn* attn, int which, int bits, int group_size,
                                   const uint32_t* wq, const float* scales, const float* biases,
                                   const float* bias);

/* pos_bias_u / pos_bias_v (attention.rs:882-890): host f32 [n_heads, head_dim]. */
int nrp_attn_load_pos_bias(nrp_attn* attn, const float* pos_bias_u, const float* pos_bias_v);

/* RelPositionMultiHeadAttention::forward (attention.rs:446-573):
 * x device [batch, seq_len, d_model] in the module dtype; pos_emb device
 * [2*seq_len-1, d_model] (module dtype); lengths device int32 [batch] or
 * NULL -- the key_padding_mask of attention.rs:280-294 (keys >= max(len,1)
 * hidden; pass NULL when no frame is padding); context NULL for full
 * attention; out device [batch, seq_len, d_model].  Query rows past a
 * sequence's length are unspecified (conformer.rs:1590-1593); this
 * implementation writes finite values there.  bf16 needs head_dim 128. */
int nrp_attn_forward(nrp_attn* attn, void* stream, const void* x, int batch, int seq_len,
                     const void* pos_emb, const int32_t* lengths,
                     const nrp_att_context* context, void* out);

/* No counterpart in the reference.  The same computation as nrp_attn_forward
 * (same arguments and outputs), for callers that cannot let the library
 * allocate device memory -- e.g. an audio thread with a real-time deadline,
 * which cannot wait on cudaMalloc's device synchronisation, or a process
 * whose device memory is handed out by another runtime's allocator.  Its
 * intermediate tensors live in a fixed 32 MiB array in the library's device
 * memory, so it allocates nothing.  The array is committed, and its device
 * address looked up, when the first context on a device is created
 * (nrp_context_create); the device holds it from then until the process
 * exits.  The limit is batch * seq_len * 8 KB + positions * 2 KB <= 32 MiB
 * at d_model 1024 in bf16 (positions = 2 * seq_len - 1, or the rows a
 * context window reaches: 257 for (128, 128)), i.e. about 2.8k frames for
 * one utterance with full context; larger sizes are rejected with
 * NRP_ERR_INVALID.  The module's parameters must already be on the device
 * (one nrp_attn_forward or nrp_attn_forward_with_cache call uploads them);
 * otherwise NRP_ERR_INVALID.  Quantised weights use the bf16 copies that
 * call kept when it ran on 256 or more rows (the context's weight cache);
 * without them the 8-bit GEMM dequantises in its producer, which is slower.
 * The caller's current device is restored on return.  All calls share the
 * array: calls whose work overlaps on the GPU race and must be serialised
 * by the caller. */
int nrp_attn_forward_noalloc(nrp_attn* attn, void* stream, const void* x, int batch, int seq_len,
                             const void* pos_emb, const int32_t* lengths,
                             const nrp_att_context* context, void* out);

/* ---------------------------------------------------- streaming caches */
/* One layer's share of EncoderCache (src/asr/streaming/core.rs:117-127):
 * the attention-input cache last_channel[layer] ([batch, cache_len,
 * d_model], f32, zero-initialised) kept as a ring, plus device K/V rings of
 * its projections so cached frames are not re-projected every chunk. */
int nrp_cache_create(nrp_attn* attn, int batch, int cache_len, nrp_cache** out);
int nrp_cache_destroy(nrp_cache* cache);
/* Zero the cache (EncoderCache::new state). */
int nrp_cache_reset(nrp_cache* cache, void* stream);
/* The ring slot of the oldest cached frame (host state, advanced by every
 * nrp_attn_forward_with_cache).  A caller that replays the device work of a
 * forward_with_cache call (a captured CUDA graph) without running the call
 * sets it to the value that call left.  No counterpart in the reference,
 * whose cache is a tensor that is rebuilt every chunk. */
int nrp_cache_get_head(const nrp_cache* cache, int* head);
int nrp_cache_set_head(nrp_cache* cache, int head);
/* Copy in / out the cache in EncoderCache.last_channel order (oldest frame
 * first): device f32 [batch, cache_len, d_model].  Import re-projects K/V
 * with the module's current weights. */
int nrp_cache_import_h(nrp_cache* cache, const float* h, void* stream);
int nrp_cache_export_h(nrp_cache* cache, float* h, void* stream);

/* RelPositionMultiHeadAttention::forward_with_cache (attention.rs:606-816)
 * as ConformerEncoder::forward_streaming drives it per layer
 * (conformer.rs:883-1000): x device [batch, seq_len, d_model]; pos_emb
 * device [2*(cache_len+seq_len)-1, d_model] (projected once per length and
 * reused, 749-761); filled = the first stream's fill level (clamped to
 * [0, cache_len]), valid = its valid frame count; context NULL = no
 * att_context_size.  The attention mask is create_attention_mask's
 * (conformer.rs:97-221); rows with no visible key give 0 (781-790).  The
 * cache then slides by seq_len - cache_drop_size frames (661-684, 983-1000). */
int nrp_attn_forward_with_cache(nrp_attn* attn, void* stream, const void* x, int batch,
                                int seq_len, const void* pos_emb, nrp_cache* cache, int filled,
                                int valid, const nrp_att_context* context, void* out);

/* ------------------------------------- sequence split over several GPUs */
/* Long-form windowed attention with the sequence cut into contiguous
 * segments, one per GPU (one process per GPU).  The reference runs one
 * device and has no counterpart; each rank computes exactly the rows
 * RelPositionMultiHeadAttention::forward (attention.rs:446-573) gives for its
 * segment, with the keys and values of the frames its window reaches on the
 * neighbouring segments (the halo) received over NCCL. */
typedef struct nrp_halo nrp_halo;
#define NRP_HALO_ID_BYTES 128

/* Copies the valid frames of each utterance of a [B, T, row] tensor:
 * dst[b, :lengths[b]] = src[b, :lengths[b]] (lengths clipped to [0, T], host
 * memory), one cudaMemcpyAsync per utterance on `stream` (cudaMemcpyDefault:
 * pinned host <-> device or device <-> device).  Padded frames are left as
 * they are: a forward's padded rows are unspecified (conformer.rs:1590-1593)
 * and padded input rows reach no valid output row.  *bytes (may be NULL):
 * the bytes queued.  This is the host side of a serving loop that moves only
 * valid frames across PCIe. */
int nrp_copy_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                    int64_t row_bytes, void* stream, int64_t* bytes);

/* Packed frames: a batch's valid frames back to back, utterance b's
 * lengths[b] rows from packed row lengths[0] + ... + lengths[b-1] on (the
 * buffer a serving loop fills per step).  nrp_unpack_frames writes them into
 * rows [0, lengths[b]) of the [B, T, row_bytes] device tensor dst, and
 * nrp_pack_frames reads those rows of src into packed dst.  With `staging`
 * (device memory of at least sum(lengths) * row_bytes bytes) the packed side
 * may be pinned host memory: one cudaMemcpyAsync crosses the link (into or
 * out of staging) and a kernel scatters or gathers the rows on the device;
 * staging NULL means the packed side is device memory.  One copy per
 * direction instead of nrp_copy_frames' one per utterance: with 16
 * utterances moving both ways at once, per-utterance copies ran at 36 GB/s
 * each way on B200 over PCIe, one copy each way at 49 GB/s.  dev_lengths
 * (may be NULL): the kernel also writes lengths[b] there (the device lengths
 * of a key-padding mask), so a step needs no second upload.  lengths is a
 * host array, each in [0, T].  Padded rows are left as they are.  Stream
 * ordered; *bytes (may be NULL): the packed bytes. */
int nrp_unpack_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                      int64_t row_bytes, void* staging, int32_t* dev_lengths, void* stream,
                      int64_t* bytes);
int nrp_pack_frames(void* dst, const void* src, const int32_t* lengths, int B, int T,
                    int64_t row_bytes, void* staging, void* stream, int64_t* bytes);

/* Segment of `rank`: [start, start + len) of seq_len frames cut into nranks
 * pieces of ceil(seq_len / nranks) (the last one ragged; len may be 0). */
int nrp_seq_shard(int seq_len, int nranks, int rank, int* start, int* len);
/* Utterance-parallel replicas (one GPU per rank, no collective on the data
 * path): splits a batch of n utterances over nranks so that their work is
 * balanced.  An utterance of L frames costs L^2 + (4 d_model / 3) L (its
 * attention, 6 d L^2, against its projections, 8 d^2 L).  Longest first,
 * each to the least loaded rank (ties: the lower rank), which is within
 * 4/3 of the best split.  rank_of [n]: the rank of each utterance;
 * rank_cost [nranks] (may be NULL): each rank's total cost. */
int nrp_partition_utterances(const int32_t* lengths, int n, int nranks, int d_model,
                             int32_t* rank_of, double* rank_cost);

/* The halo plan of `rank` under `context` (NULL: full context): its
 * segment, the frames it receives from rank-1 (halo_left) and rank+1
 * (halo_right), and the frames it sends them (its first send_prev and last
 * send_next frames).  The halo of a segment [s, e) is the part of
 * [s + dmin, e + dmax) within the sequence outside it, where dmin..dmax are
 * the key offsets j - i the context makes visible.  NRP_ERR_UNSUPPORTED
 * when a rank would have no frames or a halo would reach past a neighbour. */
typedef struct {
  int start, len;
  int halo_left, halo_right;
  int send_prev, send_next;
} nrp_seq_plan;
int nrp_seq_shard_plan(int seq_len, int nranks, int rank, const nrp_att_context* context,
                       nrp_seq_plan* out);

/* The communicator's unique id (ncclGetUniqueId), made on one rank and
 * handed to every rank by the caller's own means (a store, a broadcast). */
int nrp_halo_unique_id(unsigned char id[NRP_HALO_ID_BYTES]);

/* Joins the communicator of nranks ranks (one per process and device, the
 * context's device).  NCCL (libnccl.so.2) is loaded on first use.  Every
 * wait of the communicator's host side is bounded by timeout_ms: a rank
 * that does not join or answer in time makes the call fail (NRP_ERR_DEVICE)
 * and the communicator is aborted. */
int nrp_halo_comm_create(nrp_context* ctx, const unsigned char id[NRP_HALO_ID_BYTES], int rank,
                         int nranks, int timeout_ms, nrp_halo** out);
int nrp_halo_comm_destroy(nrp_halo* halo);

/* Waits up to the communicator's timeout for the work queued on `stream`;
 * if it has not finished (a peer that never sent its halo), aborts the
 * communicator -- which ends its kernels -- and returns NRP_ERR_DEVICE.
 * An aborted communicator fails every later call. */
int nrp_halo_comm_check(nrp_halo* halo, void* stream);

/* This rank's share of nrp_attn_forward on [batch, seq_len, d_model]:
 * x_local device [batch, len, d_model] = frames [start, start + len) of the
 * sequence (nrp_seq_shard); pos_emb device [2*seq_len-1, d_model], the whole
 * table (only the rows the window reaches are read); lengths device int32
 * [batch] in frames of the whole sequence, or NULL; context: a window that
 * reaches no further than the neighbouring segments (NRP_ERR_UNSUPPORTED
 * otherwise, and for full context); out_local device [batch, len, d_model].
 * bf16 only.  Every rank calls it with the same batch, seq_len and context,
 * in the same order. */
int nrp_attn_forward_seq_sharded(nrp_attn* attn, nrp_halo* halo, void* stream,
                                 const void* x_local, int batch, int seq_len,
                                 const void* pos_emb, const int32_t* lengths,
                                 const nrp_att_context* context, void* out_local);

/* ------------------------------------------------------ conformer block */
/* ConformerBlock (src/asr/modules/encoders/conformer.rs:1617-2028):
 *   x += 0.5 * FF1(LN x); x += MHA(LN x); x += Conv(LN x);
 *   x += 0.5 * FF2(LN x); x = LN x
 * with FeedForward = linear2(SiLU(linear1 x)) (2033-2088) and
 * ConvolutionModule = pointwise_conv2(SiLU(norm(depthwise(GLU(pointwise_conv1
 * x) with padded frames zeroed)))) (2108-2330).  LayerNorms have eps 1e-5;
 * the conv norm is BatchNorm in inference mode (eps 1e-5) or a LayerNorm.
 * Every linear may be standard or MLX 8-bit quantised, like the attention's.
 * The block runs in bf16 (nrp_block_set_dtype(NRP_DTYPE_BF16)) and needs
 * d_model in {256, 512, 1024, 2048}, head_dim 128 and ff_dim % 64 == 0. */
typedef struct nrp_block nrp_block;
typedef enum {
  NRP_BLOCK_FF1_LINEAR1 = 0, /* feed_forward1.linear1 [ff_dim, d_model] */
  NRP_BLOCK_FF1_LINEAR2 = 1, /* feed_forward1.linear2 [d_model, ff_dim] */
  NRP_BLOCK_CONV_PW1 = 2,    /* conv.pointwise_conv1 [2*d_model, d_model] */
  NRP_BLOCK_CONV_PW2 = 3,    /* conv.pointwise_conv2 [d_model, d_model] */
  NRP_BLOCK_FF2_LINEAR1 = 4,
  NRP_BLOCK_FF2_LINEAR2 = 5
} nrp_block_linear_id;
typedef enum {
  NRP_BLOCK_NORM_FF1 = 0,  /* norm_feed_forward1 */
  NRP_BLOCK_NORM_ATT = 1,  /* norm_self_att */
  NRP_BLOCK_NORM_CONV = 2, /* norm_conv */
  NRP_BLOCK_NORM_FF2 = 3,  /* norm_feed_forward2 */
  NRP_BLOCK_NORM_OUT = 4   /* norm_out */
} nrp_block_norm_id;
/* ConformerBlock::new (1661-1692): conv_norm 0 = batch_norm, 1 = layer_norm;
 * causal_conv pads the depthwise conv on the left only. */
int nrp_block_create(nrp_context* ctx, int d_model, int n_heads, int ff_dim, int conv_kernel,
                     int causal_conv, int conv_norm, int use_bias, nrp_block** out);
int nrp_block_destroy(nrp_block* block);
int nrp_block_set_dtype(nrp_block* block, int dtype);
/* The block's RelPositionMultiHeadAttention (owned by the block): load its
 * parameters with nrp_attn_load_*. */
int nrp_block_attn(nrp_block* block, nrp_attn** attn);
/* Weights::fetch_linear for one of the block's linears (FeedForward::
 * load_weights 2074-2088, ConvolutionModule::load_weights 2404-2437): host
 * f32 weight [out, in], bias [out] or NULL; quantised: u32 codes
 * [out, in*bits/32], scales/biases [out, in/group]. */
int nrp_block_load_linear(nrp_block* block, int which, const float* weight, const float* bias);
int nrp_block_load_linear_quantized(nrp_block* block, int which, int bits, int group_size,
                                    const uint32_t* wq, const float* scales,
                                    const float* biases, const float* bias);
/* load_layer_norm (src/core/loading.rs:203-214): gamma, beta host f32 [d_model]. */
int nrp_block_load_norm(nrp_block* block, int which, const float* gamma, const float* beta);
/* load_conv1d for conv.depthwise_conv (loading.rs:216-223): weight host f32
 * in the MLX layout [d_model, kernel, 1]; bias [d_model] or NULL. */
int nrp_block_load_depthwise(nrp_block* block, const float* weight, const float* bias);
/* load_batch_norm for conv.batch_norm (loading.rs:234-252); with conv_norm
 * = layer_norm, gamma/beta are that LayerNorm's and mean/var are ignored. */
int nrp_block_load_conv_norm(nrp_block* block, const float* gamma, const float* beta,
                             const float* running_mean, const float* running_var);
/* ConformerBlock::forward (1693-1870): x, out device [batch, seq_len,
 * d_model] bf16 (out may be x); pos_emb device [2*seq_len-1, d_model];
 * lengths device int32 [batch] or NULL (PaddingMask, 1594-1615: padded keys
 * hidden, padded frames zeroed before the depthwise conv); context NULL
 * for full attention.  Rows past a length are unspecified. */
int nrp_block_forward(nrp_block* block, void* stream, const void* x, int batch, int seq_len,
                      const void* pos_emb, const int32_t* lengths,
                      const nrp_att_context* context, void* out);

/* ConformerBlock::forward_with_cache (conformer.rs:1877-1967) with
 * ConvolutionModule::forward_with_cache (2332-2400), as forward_streaming
 * drives it (883-1000): x, out device [batch, seq_len, d_model] bf16 (out
 * may be x); pos_emb device [2*(C+seq_len)-1, d_model]; attn_cache the
 * block attention's cache (nrp_cache_create on nrp_block_attn, C frames);
 * conv_cache device bf16 [batch, conv_kernel-1, d_model] (time-major; the
 * reference's cache_last_time[layer] is [batch, d_model, conv_kernel-1]):
 * read, then replaced by the last conv_kernel-1 frames of [cache | GLU
 * output]; filled, valid, context as nrp_attn_forward_with_cache; frames
 * t >= valid are zeroed before the depthwise conv (the pad mask, 929-941).
 * The depthwise conv runs without padding over [cache | chunk]. */
int nrp_block_forward_with_cache(nrp_block* block, void* stream, const void* x, int batch,
                                 int seq_len, const void* pos_emb, nrp_cache* attn_cache,
                                 void* conv_cache, int filled, int valid,
                                 const nrp_att_context* context, void* out);

/* EncoderCache on the device (streaming/core.rs:117-185) for an encoder's
 * forward_streaming: per layer the attention's K/V/h ring of cache_len
 * frames (last_channel) and the conv cache [batch, conv_kernel-1, d_model]
 * bf16 (last_time, time-major), and the fill level the streams share
 * (last_channel_len: forward_streaming reads the first stream's,
 * conformer.rs:853-857).  Make it after nrp_encoder_set_dtype(BF16). */
typedef struct nrp_encoder_cache nrp_encoder_cache;

/* ConformerEncoder::forward_from_embeddings (conformer.rs:694-722) over
 * n_layers blocks: x * xscale (sqrt(d_model) when xscaling), the positional
 * table of RelPositionalEncoding(d_model, max_len) for seq_len, every block,
 * then the transpose to [batch, d_model, seq_len]. */
typedef struct nrp_encoder nrp_encoder;
typedef struct nrp_subsampling nrp_subsampling; /* (below) */
int nrp_encoder_create(nrp_context* ctx, int n_layers, int d_model, int n_heads, int ff_dim,
                       int conv_kernel, int causal_conv, int conv_norm, int use_bias,
                       int xscaling, int max_len, nrp_encoder** out);
int nrp_encoder_destroy(nrp_encoder* enc);
int nrp_encoder_block(nrp_encoder* enc, int layer, nrp_block** block);
int nrp_encoder_set_dtype(nrp_encoder* enc, int dtype);
/* x device [batch, seq_len, d_model] bf16 (left unchanged); lengths device
 * int32 [batch] or NULL; out device [batch, d_model, seq_len] bf16. */
int nrp_encoder_forward_from_embeddings(nrp_encoder* enc, void* stream, const void* x, int batch,
                                        int seq_len, const int32_t* lengths,
                                        const nrp_att_context* context, void* out);
/* The encoder's pre_encode (ConformerEncoder::new, conformer.rs:381-420):
 * creates the subsampling the encoder owns and runs in nrp_encoder_forward;
 * *sub is borrowed (load its weights with nrp_subsampling_load_*). */
int nrp_encoder_add_subsampling(nrp_encoder* enc, int feat_in, int subsampling_factor,
                                int conv_channels, int causal_downsampling,
                                nrp_subsampling** sub);
/* ConformerEncoder::forward (475-560): features device f32 [batch, feat_in,
 * frames]; lengths host int32 [batch] mel frames, or NULL (all frames):
 * frames past a length are zeroed, the subsampling, x * xscale, the blocks
 * with the subsampled lengths, the transpose.  out device [batch, d_model,
 * T'] bf16 (T' = nrp_subsampling_output_length(frames)); out_lengths host
 * int32 [batch] (Subsampling::output_lengths, 1387-1411) or NULL. */
int nrp_encoder_forward(nrp_encoder* enc, void* stream, const float* features, int batch,
                        int frames, const int32_t* lengths, const nrp_att_context* context,
                        void* out, int32_t* out_lengths);
int nrp_encoder_cache_create(nrp_encoder* enc, int batch, int cache_len,
                             nrp_encoder_cache** out);
int nrp_encoder_cache_destroy(nrp_encoder_cache* cache);
/* zeros every cache (NeMo starts a stream with zeros), fill level 0 */
int nrp_encoder_cache_reset(nrp_encoder_cache* cache, void* stream);
int nrp_encoder_cache_get_filled(const nrp_encoder_cache* cache, int* filled);
int nrp_encoder_cache_set_filled(nrp_encoder_cache* cache, int filled);
/* layer's attention ring (export/import its h with nrp_cache_export_h /
 * nrp_cache_import_h) and its conv cache (device pointer); either out
 * pointer may be NULL */
int nrp_encoder_cache_layer(nrp_encoder_cache* cache, int layer, nrp_cache** attn_cache,
                            void** conv_cache);
/* copies a layer's conv cache to (to_cache = 0) or from (1) device data
 * bf16 [batch, conv_kernel-1, d_model] */
int nrp_encoder_cache_copy_conv(nrp_encoder_cache* cache, int layer, void* data, int to_cache,
                                void* stream);
/* ConformerEncoder::forward_streaming (conformer.rs:840-1047): features
 * device f32 [batch, feat_in, frames] (a chunk with its pre-encode cache
 * frames in front, as the caller builds it); the subsampling (no mel mask
 * on this path), the first drop_extra_pre_encoded output frames dropped,
 * x * xscale, every block's forward_with_cache against `cache` with the
 * first stream's fill level and valid length (subsampled lengths[0] less
 * the drop; lengths host int32 [batch] mel frames, or NULL: all frames),
 * the transpose; the fill level advances by the frames kept.  out device
 * [batch, d_model, T] bf16 with T = nrp_subsampling_output_length(frames)
 * - drop_extra_pre_encoded; out_lengths host int32 [batch] (subsampled
 * lengths less the drop) and out_frames (T) may be NULL. */
int nrp_encoder_forward_streaming(nrp_encoder* enc, void* stream, const float* features,
                                  int batch, int frames, const int32_t* lengths,
                                  nrp_encoder_cache* cache, int drop_extra_pre_encoded,
                                  const nrp_att_context* context, void* out,
                                  int32_t* out_lengths, int* out_frames);

/* ------------------------------------------ dw_striding subsampling */
/* Subsampling (src/asr/modules/encoders/conformer.rs:1058-1588), the
 * encoder's pre_encode: mel frames [batch, frames, feat_in] -> NHWC
 * [.., 1]; conv.0 (1 -> C, 3x3, stride 2) + ReLU; per further stride a
 * depthwise 3x3 stride-2 conv (groups C), a pointwise 1x1 conv and ReLU;
 * [B, T', F', C] flattened channel-major ([B, T', C * F']) into the `out`
 * linear -> [batch, T', d_model].  strides = log2(subsampling_factor) for
 * 2, 4, 8 (any other factor: 2, as Subsampling::new).  Non-causal convs pad
 * 1 on both sides; causal_downsampling pads (2, 1) on time and frequency
 * (causal_pad_2d, 66-80).  Runs in bf16; conv_channels a power of two in
 * [64, 2048], d_model % 32 == 0. */
typedef enum {
  NRP_FEATURES_BFT = 0, /* [batch, feat_in, frames] (ConformerEncoder::forward's input) */
  NRP_FEATURES_BTF = 1  /* [batch, frames, feat_in] (forward_subsampling_only's) */
} nrp_features_layout;
/* Subsampling::new (1111-1205).  ctx may be NULL for a handle that only
 * answers sizes (feat_out, output_length); its forward then fails. */
int nrp_subsampling_create(nrp_context* ctx, int feat_in, int d_model, int subsampling_factor,
                           int conv_channels, int causal_downsampling, nrp_subsampling** out);
int nrp_subsampling_destroy(nrp_subsampling* sub);
int nrp_subsampling_set_dtype(nrp_subsampling* sub, int dtype);
/* compute_freq_output_size (1220-1244): F', so `out` has C * F' inputs. */
int nrp_subsampling_feat_out(const nrp_subsampling* sub, int* feat_out);
/* Subsampling::output_length (1315-1327): frames after the conv stack (also
 * the time size of the forward's output for an input of `frames`). */
int nrp_subsampling_output_length(const nrp_subsampling* sub, int frames, int* out_frames);
/* load_conv2d (src/core/loading.rs:227-232) for pre_encode.conv.{index}
 * (Subsampling::load_weights, 1557-1588): 0 = conv.0 [C, 3, 3, 1]; 2 + 3i =
 * depthwise i [C, 3, 3, 1]; 3 + 3i = pointwise i [C, 1, 1, C]; host f32 in
 * MLX's layout; bias [C] or NULL (zeros). */
int nrp_subsampling_load_conv(nrp_subsampling* sub, int index, const float* weight,
                              const float* bias);
/* Weights::fetch_linear for pre_encode.out: weight [d_model, C * F'] in the
 * reference's (channel, frequency) column order, bias [d_model] or NULL;
 * quantised: as nrp_attn_load_linear_quantized. */
int nrp_subsampling_load_out(nrp_subsampling* sub, const float* weight, const float* bias);
int nrp_subsampling_load_out_quantized(nrp_subsampling* sub, int bits, int group_size,
                                       const uint32_t* wq, const float* scales,
                                       const float* biases, const float* bias);
/* Subsampling::forward_frames (1413-1555): features device f32 in `layout`;
 * lengths device int32 [batch] or NULL: frames t >= lengths[b] read as zero
 * (ConformerEncoder::forward's mel mask, 484-518); out device
 * [batch, T', d_model] bf16, T' = nrp_subsampling_output_length(frames). */
int nrp_subsampling_forward(nrp_subsampling* sub, void* stream, const float* features, int layout,
                            int batch, int frames, const int32_t* lengths, void* out);
/* Subsampling::forward_frames_chunked (1334-1377): with frames > 0, inputs
 * longer than `frames` mel frames (rounded down to a multiple of the factor)
 * run the conv stack in time chunks, each with twice the receptive field of
 * real neighbouring frames on either side, the frames that saw a chunk's edge
 * padding cropped.  This bounds the activation memory to one chunk's; the
 * output equals the single pass bit for bit.  0 (the default): the whole
 * input at once.  The reference uses 4096 (SUBSAMPLING_CHUNK_FRAMES, 1060). */
int nrp_subsampling_set_chunk_frames(nrp_subsampling* sub, int frames);

/* --------------------------------------------------- linear primitives */
/* LinearLayer::forward, Standard arm (quantization.rs:128-135) on device
 * buffers: y[M,N] = x[M,K] . w[N,K]^T (+ bias[N]), dtype f32 or bf16 for
 * every operand.  bf16 needs K % 64 == 0 and N % 32 == 0. */
int nrp_linear(nrp_context* ctx, void* stream, int dtype, const void* x, int M, int K,
               const void* w, int N, const void* bias, void* y);

/* LinearLayer::forward, Quantized arm (quantization.rs:137-160):
 * y[M,N] = x[M,K] . dequant(wq, scales, biases)^T (+ bias), MLX affine
 * 8-bit, group 64; x, scales, biases, bias, y bf16 on the device; wq device
 * u32 [N, K/4].  M <= 16 runs the HBM-bound GEMV, larger M the tcgen05
 * GEMM with in-register dequantisation. */
int nrp_qlinear(nrp_context* ctx, void* stream, const void* x, int M, int K, const uint32_t* wq,
                const void* scales, const void* biases, int N, int group_size, int bits,
                const void* bias, void* y);

/* ------------------------------------------------------------ profiling */
/* Per-kernel device time from CUDA events the library records on the
 * launching stream around each launch while enabled (the reference has no
 * profiler integration; its timing is end to end, examples/eval.rs:158-215). */
typedef enum {
  NRP_KERNEL_GEMM_BF16 = 0,   /* tcgen05 projection GEMM */
  NRP_KERNEL_GEMM_Q8 = 1,     /* tcgen05 GEMM, 8-bit weights dequantised in smem */
  NRP_KERNEL_QGEMV = 2,       /* small-M 8-bit GEMV */
  NRP_KERNEL_GEMM_F32 = 3,    /* f32 CUDA-core GEMM */
  NRP_KERNEL_ATTN_SM100 = 4,  /* fused offline rel-pos attention, tcgen05 */
  NRP_KERNEL_ATTN_SIMT = 5,   /* f32 offline attention, CUDA cores */
  NRP_KERNEL_ATTN_STREAM = 6, /* streaming attention against the ring cache */
  NRP_KERNEL_RING_APPEND = 7, /* streaming cache slide */
  NRP_KERNEL_LAYERNORM = 8,   /* the block's LayerNorms */
  NRP_KERNEL_DWCONV = 9,      /* depthwise conv + BatchNorm + SiLU */
  NRP_KERNEL_ELEMENTWISE = 10, /* input scaling, transposes, copies */
  NRP_KERNEL_DEQUANT = 11,    /* 8-bit weights to bf16 (large-M quantised GEMM) */
  NRP_KERNEL_SUBSAMPLE = 12,  /* the subsampling's direct (non-GEMM) convolutions */
  NRP_KERNEL_KINDS = 13
} nrp_kernel_kind;
int nrp_profile_enable(nrp_context* ctx, int enable);
int nrp_profile_reset(nrp_context* ctx);
/* Synchronises on the recorded events; writes launches and total ms of `kind`. */
int nrp_profile_read(nrp_context* ctx, int kind, int64_t* launches, double* total_ms);
/* The recorded launches since the last reset in the order the host issued
 * them: kinds[i] (nrp_kernel_kind) and ms[i] for i < min(*count, capacity);
 * *count = the number recorded.  Synchronises on the recorded events. */
int nrp_profile_launches(nrp_context* ctx, int* kinds, float* ms, int64_t capacity,
                         int64_t* count);

#ifdef __cplusplus
}
#endif
#endif
