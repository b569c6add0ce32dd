/*
 * relpos_oracle.h -- CPU restatement of the reference's rel-pos MHA path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * implementation: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product library (libnemo_relpos.so) never
 * links or calls it.
 *
 * Reference: animaslabs/mlx-nemo-rs (crate mlx-voice 0.3.0).  The reference
 * is Rust over MLX (Metal/Accelerate, macOS only) and cannot be built or run
 * here, so this is a restatement of its algorithm; each function cites the
 * reference file:line it follows.  Parity is pinned by the reference's own
 * known-answer and property tests (src/asr/modules/encoders/attention.rs
 * tests 901-1357, src/asr/streaming/core.rs 392-438, src/core/quantization.rs
 * 414-468), restated in tests/test_oracle_golden.py against
 * tests/golden/reference_kats.json.  MLX's own kernels (quantized_matmul,
 * fast::scaled_dot_product_attention) have no golden vectors in the
 * reference: their arithmetic is restated from MLX's published semantics.
 *
 * All tensors are row-major float32 unless stated otherwise.
 */
#ifndef RELPOS_ORACLE_H
#define RELPOS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- positional encoding (attention.rs:59-103, 131-177) ---- */
/* pe: [2*max_len-1, d_model] for positions (max_len-1) .. -(max_len-1). */
void orc_create_pe(int d_model, int max_len, float *pe);
/* out: [2*seq_len-1, d_model]; slice of the max_len table, or a table built
 * at seq_len when seq_len > max_len.  Returns 0, or -1 for seq_len == 0. */
int orc_get_encoding(int d_model, int max_len, int seq_len, float *out);

/* ---- rel_shift by pad/reshape/slice (attention.rs:832-855) ---- */
/* x, out: [bh, seq_len, pos_len] */
void orc_rel_shift(const float *x, int bh, int seq_len, int pos_len, float *out);

/* ---- masks ---- */
/* AttentionContext::block_mask (attention.rs:232-272): vis[(i-start)*seq_len+j]
 * = 1 when query i sees key j. */
void orc_block_mask(int left, int right, int chunked, int start, int end,
                    int seq_len, uint8_t *vis);
/* query_block_size (attention.rs:202-206) */
int orc_query_block_size(int batch_heads, int seq_len, int64_t max_score_elements);
/* create_attention_mask (conformer.rs:97-221): vis [tensor_seq_len, max_audio_length] */
void orc_create_attention_mask(int left, int right, int chunked,
                               int max_audio_length, int cache_len,
                               int filled_cache_len, int tensor_seq_len,
                               int valid_seq_len, uint8_t *vis);

/* ---- linear layers (quantization.rs:126-162) ---- */
/* y[M,N] = x[M,K] . W[N,K]^T (+ bias[N]) */
void orc_linear(const float *x, int M, int K, const float *w, int N,
                const float *bias, float *y);
/* MLX affine dequantisation: w[n,k] = scale[n,k/g] * q[n,k] + bias[n,k/g],
 * q packed (32/bits) per uint32 along k, lowest bits first. */
void orc_dequantize(const uint32_t *wq, const float *scales, const float *biases,
                    int N, int K, int group_size, int bits, float *w);
/* MLX affine quantisation (round to nearest of (w - min)/scale), the format
 * `mlx.core.quantize` writes: per group scale = (max-min)/(2^bits-1),
 * bias = min.  Used to build quantised test weights. */
void orc_quantize(const float *w, int N, int K, int group_size, int bits,
                  uint32_t *wq, float *scales, float *biases);

/* ---- rel-pos multi-head attention ---- */
typedef struct {
  const float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo; /* [D,D], [D] (bias may be NULL) */
  const float *wp;                                    /* linear_pos [D,D], no bias */
  const float *pos_bias_u, *pos_bias_v;               /* [H, dh] */
} orc_mha_weights;

typedef struct {
  int has;      /* 0 = no context limit (AttentionContext::new returned None) */
  int left, right, chunked;
} orc_context;

enum {
  ORC_DIRECT = 0,         /* bd by index arithmetic, no blocking */
  ORC_REFERENCE_ALGO = 1, /* the reference's algorithm: query blocks, materialised
                             (q+v)P^T over pos rows, rel_shift by pad/reshape,
                             additive masks, softmax, PV (attention.rs:458-573) */
};

/* RelPositionMultiHeadAttention::forward_blocked (attention.rs:458-573).
 * x [B,T,D], pos_emb [2T-1, D], lengths [B] or NULL (key_padding_mask,
 * attention.rs:280-294), ctx or NULL, out [B,T,D].
 * bf16 != 0 rounds to bfloat16 where the reference's bf16 graph does.
 * max_score_elements: query-block budget (2^26 in the reference); <= 0 means
 * one block.  Returns 0 or -1 on bad arguments. */
int orc_mha_forward(const float *x, int B, int T, int D, int H,
                    const orc_mha_weights *w, const float *pos_emb,
                    const int32_t *lengths, const orc_context *ctx, int mode,
                    int bf16, int64_t max_score_elements, float *out);

/* Core attention on already projected tensors (no linears):
 * q [B,Tq,D], k/v [B,Tk,D], p [2Tk-1, D] (projected positions), u/v [H,dh],
 * vis [Tq,Tk] (shared over batch) or NULL, key_len [B] or NULL
 * (key j visible iff j < max(key_len[b],1)), ctx or NULL (offline context
 * mask on absolute positions q_offset+i vs j).  Rows with no visible key
 * give 0.  out [B,Tq,D] (heads concatenated). */
void orc_relpos_attention(const float *q, const float *k, const float *v,
                          const float *p, const float *u, const float *vb,
                          int B, int Tq, int Tk, int D, int H,
                          const uint8_t *vis, const int32_t *key_len,
                          const orc_context *ctx, int q_offset, float *out);

/* RelPositionMultiHeadAttention::forward_with_cache (attention.rs:606-816)
 * for one layer.  x [B,T,D]; cache [B,C,D] (full buffer) or NULL (C ignored);
 * pos_emb [2(C+T)-1, D]; mask [T, C+T] (1 = visible, shared over the batch)
 * or NULL; mask_is_bool selects the unfused path that zeroes rows with no
 * visible key (attention.rs:781-790); new_cache [B, max(T-drop,0) + C - ..]:
 * exactly concat(cache[q_keep:], x[:q_keep]) with q_keep = max(T-drop, 0),
 * i.e. [B, C, D] when cache != NULL (caller-sized), [B, q_keep, D] when NULL.
 * Returns the number of frames in new_cache per batch row. */
int orc_mha_forward_with_cache(const float *x, int B, int T, int D, int H,
                               const orc_mha_weights *w, const float *pos_emb,
                               const float *cache, int C, const uint8_t *mask,
                               int mask_is_bool, int cache_drop_size, int bf16,
                               float *out, float *new_cache);

/* One streaming layer step as ConformerEncoder::forward_streaming drives it
 * (conformer.rs:883-1000): mask from create_attention_mask with the first
 * stream's fill/valid, memo rule (all visible -> no mask; valid < T -> bool
 * mask; else additive), forward_with_cache, then the cache re-padded to C
 * (zeros in front) or truncated to the newest C frames.  h_cache [B,C,D] is
 * updated in place.  Returns the next fill level min(filled + keep, C). */
int orc_stream_layer_step(const float *x, int B, int T, int D, int H,
                          const orc_mha_weights *w, const float *pos_emb,
                          float *h_cache, int C, int filled, int valid,
                          int left, int right, int chunked, int cache_drop_size,
                          int bf16, float *out);

/* One linear of a Conformer block: w [N, K] f32 (a quantised layer passes
 * its dequantised weights), b [N] or NULL. */
typedef struct {
  const float *w, *b;
} orc_lin;

typedef struct {
  orc_lin ff1_1, ff1_2, pw1, pw2, ff2_1, ff2_2;
  const float *dw_w, *dw_b;               /* depthwise conv [D][K], [D] or NULL */
  const float *cn_g, *cn_b, *cn_m, *cn_v; /* conv norm (m, v: batch norm only) */
  const float *norm_g[5], *norm_b[5];     /* ff1, self_att, conv, ff2, out */
  orc_mha_weights attn;
} orc_block_weights;

/* ConformerBlock::forward (conformer.rs:1693-1870) with FeedForward
 * (2033-2088) and ConvolutionModule::forward (2249-2330): LayerNorm eps
 * 1e-5, SiLU, GLU, padded frames (t >= lengths[b]) zeroed before the
 * depthwise conv (non-causal: (K-1)/2 zeros each side; causal: K-1 on the
 * left), BatchNorm in inference mode (conv_norm 0, eps 1e-5) or LayerNorm
 * (conv_norm 1).  With bf16, every parameter is rounded (set_dtype) and
 * every op's output is rounded as the reference's bf16 graph does.
 * x, out [B, T, D]; pos_emb [2T-1, D]. */
int orc_block_forward(const float *x, int B, int T, int D, int H, int ff, int K,
                      int causal, int conv_norm, const orc_block_weights *w,
                      const float *pos_emb, const int32_t *lengths,
                      const orc_context *ctx, int bf16, float *out);

/* ---- dw_striding subsampling (conformer.rs:1058-1555) ---- */
#define ORC_SUB_MAX_PAIRS 2
typedef struct {
  const float *conv0_w, *conv0_b;                 /* [C, 3, 3, 1], [C] */
  const float *dw_w[ORC_SUB_MAX_PAIRS], *dw_b[ORC_SUB_MAX_PAIRS]; /* [C, 3, 3, 1] */
  const float *pw_w[ORC_SUB_MAX_PAIRS], *pw_b[ORC_SUB_MAX_PAIRS]; /* [C, 1, 1, C] */
  const float *out_w, *out_b;                     /* [d_model, C * F'], [d_model] */
} orc_subsampling_weights;

/* strides = log2(factor) for 2, 4, 8, else 2 (conformer.rs:1118-1123). */
int orc_subsampling_strides(int factor);
/* Subsampling::output_length (1315-1327). */
int orc_subsampling_out_len(int len, int factor, int causal);
/* compute_freq_output_size (1220-1244): F'. */
int orc_subsampling_feat_out(int feat_in, int factor, int causal);
/* Subsampling::forward_frames (1413-1555): x [B, T, F] (already masked by
 * the caller when it should be), out [B, T', d_model].  Biases may be NULL. */
int orc_subsampling_forward(const float *x, int B, int T, int F, int C, int factor,
                            int causal, int d_model, const orc_subsampling_weights *w,
                            int bf16, float *out);

/* One streaming step of a ConformerBlock (forward_with_cache, conformer.rs:
 * 1877-1967, with ConvolutionModule::forward_with_cache 2332-2400) as
 * forward_streaming drives it: h_cache [B,C,D] (the attention input ring,
 * as orc_stream_layer_step) and conv_cache [B,K-1,D] (time-major; the last
 * K-1 GLU frames) are updated in place; frames t >= valid are zeroed before
 * the depthwise conv.  x, out [B,T,D]; pos_emb [2(C+T)-1, D].  Returns the
 * next fill level. */
int orc_stream_block_step(const float *x, int B, int T, int D, int H, int ff, int K,
                          int conv_norm, const orc_block_weights *w, const float *pos_emb,
                          float *h_cache, int C, float *conv_cache, int filled, int valid,
                          int left, int right, int chunked, int cache_drop_size, int bf16,
                          float *out);

/* bfloat16 round-to-nearest-even of a float (what an MLX astype does). */
float orc_bf16_round(float x);
void orc_bf16_round_array(float *x, int64_t n);

/* Threads the oracle may use (OpenMP); <= 0 = library default. */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
