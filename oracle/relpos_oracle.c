/*
 * relpos_oracle.c -- CPU restatement of the reference's rel-pos MHA path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load this.
 *
 * Every function cites the reference file:line it restates, relative to the
 * reference project root (animaslabs/mlx-nemo-rs).  Arithmetic is float32
 * like the reference's f32 graph; `bf16` arguments round to bfloat16 at the
 * points where the reference's bf16 graph materialises bf16 arrays.
 */
#include "relpos_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void orc_set_threads(int n) {
  g_threads = n;
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ bf16 */
float orc_bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan: keep (quiet nan) */
    if (u & 0x007fffffu) u |= 0x00400000u;
    u &= 0xffff0000u;
  } else {
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    u &= 0xffff0000u;
  }
  float y;
  memcpy(&y, &u, 4);
  return y;
}

void orc_bf16_round_array(float *x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) x[i] = orc_bf16_round(x[i]);
}

/* ------------------------------------------------- positional encoding */
/* RelPositionalEncoding::create_pe, attention.rs:59-103.  Positions run from
 * (max_len-1) down to -(max_len-1); div_term[k] = exp(-(2k) * ln(1e4)/d)
 * computed in f32; angles = pos * div_term (broadcast multiply, 79);
 * pe[:, 2k] = sin, pe[:, 2k+1] = cos (85-89). */
void orc_create_pe(int d_model, int max_len, float *pe) {
  const int pe_len = 2 * max_len - 1;
  const int half = d_model / 2;
  float *div = (float *)malloc(sizeof(float) * (size_t)half);
  const float lnf = logf(10000.0f) / (float)d_model;
  for (int k = 0; k < half; ++k) div[k] = expf(-((float)(2 * k)) * lnf);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < pe_len; ++r) {
    const float pos = (float)(max_len - 1 - r);
    float *row = pe + (size_t)r * d_model;
    for (int k = 0; k < half; ++k) {
      const float a = pos * div[k];
      row[2 * k] = sinf(a);
      row[2 * k + 1] = cosf(a);
    }
  }
  free(div);
}

/* RelPositionalEncoding::get_encoding, attention.rs:131-177: an empty
 * sequence is an error (132-136); past max_len the table is rebuilt at
 * seq_len (137-145); else the slice [max_len-seq_len, max_len+seq_len-1). */
int orc_get_encoding(int d_model, int max_len, int seq_len, float *out) {
  if (seq_len <= 0) return -1;
  if (seq_len > max_len) {
    orc_create_pe(d_model, seq_len, out);
    return 0;
  }
  const int pe_len = 2 * max_len - 1;
  float *pe = (float *)malloc(sizeof(float) * (size_t)pe_len * d_model);
  orc_create_pe(d_model, max_len, pe);
  const int start = max_len - seq_len;
  memcpy(out, pe + (size_t)start * d_model,
         sizeof(float) * (size_t)(2 * seq_len - 1) * d_model);
  free(pe);
  return 0;
}

/* ---------------------------------------------------------- rel_shift */
/* rel_shift, attention.rs:832-855: pad one zero column on the left
 * ([.., pos_len+1]), reshape to [pos_len+1, seq_len], drop the first row,
 * reshape back to [seq_len, pos_len].  Done literally on the flat buffer. */
void orc_rel_shift(const float *x, int bh, int seq_len, int pos_len, float *out) {
  const size_t padded = (size_t)seq_len * (pos_len + 1);
#pragma omp parallel for schedule(static)
  for (int b = 0; b < bh; ++b) {
    const float *xb = x + (size_t)b * seq_len * pos_len;
    float *ob = out + (size_t)b * seq_len * pos_len;
    /* flat index f of the padded [seq_len, pos_len+1] buffer */
    for (size_t o = 0; o < (size_t)seq_len * pos_len; ++o) {
      const size_t f = o + (size_t)seq_len; /* skip first row of [pos_len+1, seq_len] */
      (void)padded;
      const size_t row = f / (size_t)(pos_len + 1);
      const size_t col = f % (size_t)(pos_len + 1);
      ob[o] = col == 0 ? 0.0f : xb[row * pos_len + (col - 1)];
    }
  }
}

/* ---------------------------------------------------------------- masks */
/* AttentionContext::block_mask, attention.rs:232-272. */
static inline int ctx_visible(int left, int right, int chunked, int i, int j) {
  if (chunked && right >= 0) {
    const int chunk = right + 1;
    const int left_chunks = left >= 0 ? left / chunk : 10000;
    /* floor_divide on non-negative ints */
    const int diff = i / chunk - j / chunk;
    return diff >= 0 && diff <= left_chunks;
  }
  const int offset = j - i;
  int vis = left < 0 ? 1 : (offset >= -(left > 0 ? left : 0));
  if (!chunked && right >= 0) vis = vis && (offset <= right);
  return vis;
}

void orc_block_mask(int left, int right, int chunked, int start, int end,
                    int seq_len, uint8_t *vis) {
  for (int i = start; i < end; ++i)
    for (int j = 0; j < seq_len; ++j)
      vis[(size_t)(i - start) * seq_len + j] =
          (uint8_t)ctx_visible(left, right, chunked, i, j);
}

/* query_block_size, attention.rs:202-206 */
int orc_query_block_size(int batch_heads, int seq_len, int64_t max_score_elements) {
  int64_t per_row = (int64_t)batch_heads * 2 * (int64_t)seq_len;
  if (per_row < 1) per_row = 1;
  int64_t r = max_score_elements / per_row;
  const int64_t hi = seq_len > 1 ? seq_len : 1;
  if (r < 1) r = 1;
  if (r > hi) r = hi;
  return (int)r;
}

/* create_attention_mask (conformer.rs:97-221) with apply_triu (227-249),
 * apply_tril (255-277) and create_chunked_limited_mask (293-323).
 * vis[i, j] for query rows i in [0, tensor_seq_len) (absolute cache_len+i)
 * and keys j in [0, max_audio_length). */
void orc_create_attention_mask(int left, int right, int chunked,
                               int max_audio_length, int cache_len,
                               int filled_cache_len, int tensor_seq_len,
                               int valid_seq_len, uint8_t *vis) {
  const int offset = cache_len - filled_cache_len;
  for (int ii = 0; ii < tensor_seq_len; ++ii) {
    const int i = cache_len + ii;
    for (int j = 0; j < max_audio_length; ++j) {
      int m = 1;
      if (chunked) {
        if (right == -1) {
          if (left >= 0) m = (j - i) >= -left;
        } else {
          const int chunk = right + 1;
          const int lc = left >= 0 ? left / chunk : 10000;
          const int diff = i / chunk - j / chunk;
          m = diff >= 0 && diff <= lc;
        }
      } else {
        if (left >= 0) m = m && ((j - i) >= -left);
        if (right >= 0) m = m && ((j - i) <= right);
      }
      if (offset > 0) m = m && (j >= offset);
      if (valid_seq_len < tensor_seq_len) m = m && (ii < valid_seq_len);
      vis[(size_t)ii * max_audio_length + j] = (uint8_t)m;
    }
  }
}

/* ------------------------------------------------------------- linears */
/* LinearLayer::forward, Standard arm (quantization.rs:128-135):
 * y = x . W^T (+ b).  W is transposed once so the inner loop runs over
 * contiguous output columns. */
void orc_linear(const float *x, int M, int K, const float *w, int N,
                const float *bias, float *y) {
  float *wt = (float *)malloc(sizeof(float) * (size_t)K * N);
#pragma omp parallel for schedule(static)
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) wt[(size_t)k * N + n] = w[(size_t)n * K + k];
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i) {
    float *yr = y + (size_t)i * N;
    const float *xr = x + (size_t)i * K;
    for (int n = 0; n < N; ++n) yr[n] = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float a = xr[k];
      const float *wr = wt + (size_t)k * N;
      for (int n = 0; n < N; ++n) yr[n] += a * wr[n];
    }
    if (bias)
      for (int n = 0; n < N; ++n) yr[n] += bias[n];
  }
  free(wt);
}

/* quantized_matmul's dequantisation (quantization.rs:137-160, layout doc
 * 4-8): weight u32 [N, K/(32/bits)], scales/biases [N, K/group];
 * w = scale * q + bias, values packed lowest bits first. */
void orc_dequantize(const uint32_t *wq, const float *scales, const float *biases,
                    int N, int K, int group_size, int bits, float *w) {
  const int per = 32 / bits;
  const uint32_t maskv = (bits == 32) ? 0xffffffffu : ((1u << bits) - 1u);
  const int kq = K / per, kg = K / group_size;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      const uint32_t word = wq[(size_t)n * kq + k / per];
      const uint32_t q = (word >> (bits * (k % per))) & maskv;
      const float s = scales[(size_t)n * kg + k / group_size];
      const float b = biases[(size_t)n * kg + k / group_size];
      w[(size_t)n * K + k] = s * (float)q + b;
    }
}

void orc_quantize(const float *w, int N, int K, int group_size, int bits,
                  uint32_t *wq, float *scales, float *biases) {
  const int per = 32 / bits;
  const int levels = (1 << bits) - 1;
  const int kq = K / per, kg = K / group_size;
  memset(wq, 0, sizeof(uint32_t) * (size_t)N * kq);
  for (int n = 0; n < N; ++n)
    for (int g = 0; g < kg; ++g) {
      const float *wg = w + (size_t)n * K + (size_t)g * group_size;
      float lo = wg[0], hi = wg[0];
      for (int e = 1; e < group_size; ++e) {
        lo = wg[e] < lo ? wg[e] : lo;
        hi = wg[e] > hi ? wg[e] : hi;
      }
      float s = (hi - lo) / (float)levels;
      if (s < 1e-12f) s = 1e-12f;
      scales[(size_t)n * kg + g] = s;
      biases[(size_t)n * kg + g] = lo;
      for (int e = 0; e < group_size; ++e) {
        int q = (int)lrintf((wg[e] - lo) / s);
        q = q < 0 ? 0 : (q > levels ? levels : q);
        const int k = g * group_size + e;
        wq[(size_t)n * kq + k / per] |= (uint32_t)q << (bits * (k % per));
      }
    }
}

/* ------------------------------------------------------------ attention */
static inline float dot(const float *a, const float *b, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* Direct form of the attention core: for query i and key j the positional
 * score reads projected position row r = Tq-1-i+j, which is what
 * rel_shift + truncation leaves in column j (attention.rs:1248-1282 proves
 * out[i][j] = in[i][Tq-1-i+j]).  Scores: ((q+u).k + (q+v).p_r) / sqrt(dh)
 * (attend, attention.rs:299-318: SDPA scale multiplies bd too). */
void orc_relpos_attention(const float *q, const float *k, const float *v,
                          const float *p, const float *u, const float *vb,
                          int B, int Tq, int Tk, int D, int H,
                          const uint8_t *vis, const int32_t *key_len,
                          const orc_context *ctx, int q_offset, float *out) {
  const int dh = D / H;
  const float scale = 1.0f / sqrtf((float)dh);
#pragma omp parallel
  {
    float *sc = (float *)malloc(sizeof(float) * (size_t)Tk);
    uint8_t *ok = (uint8_t *)malloc((size_t)Tk);
    float *qu = (float *)malloc(sizeof(float) * (size_t)dh);
    float *qv = (float *)malloc(sizeof(float) * (size_t)dh);
#pragma omp for collapse(3) schedule(static)
    for (int b = 0; b < B; ++b)
      for (int h = 0; h < H; ++h)
        for (int i = 0; i < Tq; ++i) {
          const float *qi = q + ((size_t)b * Tq + i) * D + (size_t)h * dh;
          for (int d = 0; d < dh; ++d) {
            qu[d] = qi[d] + u[(size_t)h * dh + d];
            qv[d] = qi[d] + vb[(size_t)h * dh + d];
          }
          int kl = Tk;
          if (key_len) {
            kl = key_len[b] < 1 ? 1 : key_len[b];
            if (kl > Tk) kl = Tk;
          }
          float mx = -INFINITY;
          int any = 0;
          for (int j = 0; j < Tk; ++j) {
            int m = j < kl;
            if (vis) m = m && vis[(size_t)i * Tk + j];
            if (ctx && ctx->has)
              m = m && ctx_visible(ctx->left, ctx->right, ctx->chunked, q_offset + i, j);
            ok[j] = (uint8_t)m;
            if (!m) continue;
            any = 1;
            const float *kj = k + ((size_t)b * Tk + j) * D + (size_t)h * dh;
            const float *pr = p + (size_t)(Tq - 1 - i + j) * D + (size_t)h * dh;
            sc[j] = (dot(qu, kj, dh) + dot(qv, pr, dh)) * scale;
            if (sc[j] > mx) mx = sc[j];
          }
          float *oi = out + ((size_t)b * Tq + i) * D + (size_t)h * dh;
          for (int d = 0; d < dh; ++d) oi[d] = 0.0f;
          if (!any) continue;
          float sum = 0.0f;
          for (int j = 0; j < Tk; ++j)
            if (ok[j]) {
              sc[j] = expf(sc[j] - mx);
              sum += sc[j];
            }
          const float inv = 1.0f / sum;
          for (int j = 0; j < Tk; ++j)
            if (ok[j]) {
              const float wj = sc[j] * inv;
              const float *vj = v + ((size_t)b * Tk + j) * D + (size_t)h * dh;
              for (int d = 0; d < dh; ++d) oi[d] += wj * vj[d];
            }
        }
    free(sc);
    free(ok);
    free(qu);
    free(qv);
  }
}

/* The reference's own algorithm for one query block (attention.rs:517-551):
 * bd = (q+v) . P_slice^T over positions (seq_len-end) .. (2*seq_len-1-start),
 * rel_shift, truncate to seq_len, mask = bd*scale + ctx_mask + key_mask,
 * SDPA(q+u, k, v, scale, mask). */
static void ref_algo_block(const float *qu, const float *qv, const float *k,
                           const float *v, const float *pproj, int B, int H,
                           int T, int dh, int D, int start, int end,
                           const int32_t *lengths, const orc_context *ctx,
                           int bf16, float *ctx_out /* [B,T,D] */) {
  const int rows = end - start;
  const int pos_cols = T + rows - 1; /* (2T-1-start) - (T-end) */
  const int p0 = T - end;
  const float scale = 1.0f / sqrtf((float)dh);
  uint8_t *cmask = NULL;
  if (ctx && ctx->has) {
    cmask = (uint8_t *)malloc((size_t)rows * T);
    orc_block_mask(ctx->left, ctx->right, ctx->chunked, start, end, T, cmask);
  }
  const size_t bd_elems = (size_t)B * H * rows * pos_cols;
  float *bd = (float *)malloc(sizeof(float) * bd_elems);
  float *bds = (float *)malloc(sizeof(float) * bd_elems);
  /* matrix_bd = matmul(q_v, p_slice) : [B,H,rows,pos_cols] */
#pragma omp parallel for collapse(3) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
      for (int r = 0; r < rows; ++r) {
        const float *qr = qv + ((size_t)b * T + start + r) * D + (size_t)h * dh;
        float *o = bd + (((size_t)b * H + h) * rows + r) * pos_cols;
        for (int c = 0; c < pos_cols; ++c) {
          float s = dot(qr, pproj + (size_t)(p0 + c) * D + (size_t)h * dh, dh);
          o[c] = bf16 ? orc_bf16_round(s) : s;
        }
      }
  orc_rel_shift(bd, B * H, rows, pos_cols, bds);
  free(bd);
#pragma omp parallel
  {
    float *sc = (float *)malloc(sizeof(float) * (size_t)T);
#pragma omp for collapse(3) schedule(static)
    for (int b = 0; b < B; ++b)
      for (int h = 0; h < H; ++h)
        for (int r = 0; r < rows; ++r) {
          const float *bdr = bds + (((size_t)b * H + h) * rows + r) * pos_cols;
          const float *qr = qu + ((size_t)b * T + start + r) * D + (size_t)h * dh;
          int kl = T;
          if (lengths) {
            kl = lengths[b] < 1 ? 1 : lengths[b];
          }
          float mx = -INFINITY;
          for (int j = 0; j < T; ++j) {
            /* attend(): mask = bd * scale (in bd's dtype) + additive masks */
            float m = bdr[j] * scale;
            if (bf16) m = orc_bf16_round(m);
            if (cmask && !cmask[(size_t)r * T + j]) m = -INFINITY;
            if (lengths && j >= kl) m = -INFINITY;
            const float s = dot(qr, k + ((size_t)b * T + j) * D + (size_t)h * dh, dh) * scale + m;
            sc[j] = s;
            if (s > mx) mx = s;
          }
          float *o = ctx_out + ((size_t)b * T + start + r) * D + (size_t)h * dh;
          for (int d = 0; d < dh; ++d) o[d] = 0.0f;
          if (mx == -INFINITY) { /* every key hidden: softmax of nothing */
            for (int d = 0; d < dh; ++d) o[d] = NAN;
            continue;
          }
          float sum = 0.0f;
          for (int j = 0; j < T; ++j) {
            sc[j] = expf(sc[j] - mx);
            sum += sc[j];
          }
          const float inv = 1.0f / sum;
          for (int j = 0; j < T; ++j) {
            const float wj = sc[j] * inv;
            if (wj == 0.0f) continue;
            const float *vj = v + ((size_t)b * T + j) * D + (size_t)h * dh;
            for (int d = 0; d < dh; ++d) o[d] += wj * vj[d];
          }
        }
    free(sc);
  }
  free(bds);
  free(cmask);
}

static float *dup_round(const float *src, size_t n, int bf16) {
  if (!src) return NULL;
  float *d = (float *)malloc(sizeof(float) * n);
  memcpy(d, src, sizeof(float) * n);
  if (bf16) orc_bf16_round_array(d, (int64_t)n);
  return d;
}

typedef struct {
  float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo, *wp, *u, *v;
} owned_weights;

/* RelPositionMultiHeadAttention::set_dtype (attention.rs:409-423): every
 * parameter is cast to the compute dtype. */
static void cast_weights(const orc_mha_weights *w, int D, int H, int bf16,
                         owned_weights *o) {
  const size_t dd = (size_t)D * D;
  o->wq = dup_round(w->wq, dd, bf16);
  o->bq = dup_round(w->bq, D, bf16);
  o->wk = dup_round(w->wk, dd, bf16);
  o->bk = dup_round(w->bk, D, bf16);
  o->wv = dup_round(w->wv, dd, bf16);
  o->bv = dup_round(w->bv, D, bf16);
  o->wo = dup_round(w->wo, dd, bf16);
  o->bo = dup_round(w->bo, D, bf16);
  o->wp = dup_round(w->wp, dd, bf16);
  o->u = dup_round(w->pos_bias_u, (size_t)D, bf16);
  o->v = dup_round(w->pos_bias_v, (size_t)D, bf16);
  (void)H;
}

static void free_weights(owned_weights *o) {
  free(o->wq); free(o->bq); free(o->wk); free(o->bk); free(o->wv);
  free(o->bv); free(o->wo); free(o->bo); free(o->wp); free(o->u); free(o->v);
}

/* y = linear(x) then rounded like a bf16 matmul + bias output. */
static void linear_r(const float *x, int M, int K, const float *w, int N,
                     const float *bias, int bf16, float *y) {
  if (bf16 && bias) {
    /* matmul output is bf16, then the bias add rounds again */
    orc_linear(x, M, K, w, N, NULL, y);
    orc_bf16_round_array(y, (int64_t)M * N);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < M; ++i)
      for (int n = 0; n < N; ++n)
        y[(size_t)i * N + n] = orc_bf16_round(y[(size_t)i * N + n] + bias[n]);
  } else {
    orc_linear(x, M, K, w, N, bias, y);
    if (bf16) orc_bf16_round_array(y, (int64_t)M * N);
  }
}

/* RelPositionMultiHeadAttention::forward / forward_blocked,
 * attention.rs:446-573. */
int orc_mha_forward(const float *x, int B, int T, int D, int H,
                    const orc_mha_weights *w, const float *pos_emb,
                    const int32_t *lengths, const orc_context *ctx, int mode,
                    int bf16, int64_t max_score_elements, float *out) {
  if (B <= 0 || T <= 0 || D <= 0 || H <= 0 || D % H) return -1;
  const int dh = D / H;
  const int P = 2 * T - 1;
  const size_t n = (size_t)B * T * D;
  owned_weights ow;
  cast_weights(w, D, H, bf16, &ow);
  float *xx = dup_round(x, n, bf16);
  float *pe = dup_round(pos_emb, (size_t)P * D, bf16);
  float *q = (float *)malloc(sizeof(float) * n);
  float *k = (float *)malloc(sizeof(float) * n);
  float *v = (float *)malloc(sizeof(float) * n);
  float *pp = (float *)malloc(sizeof(float) * (size_t)P * D);
  float *cx = (float *)malloc(sizeof(float) * n);
  /* 478-480, 493 */
  linear_r(xx, B * T, D, ow.wq, D, ow.bq, bf16, q);
  linear_r(xx, B * T, D, ow.wk, D, ow.bk, bf16, k);
  linear_r(xx, B * T, D, ow.wv, D, ow.bv, bf16, v);
  linear_r(pe, P, D, ow.wp, D, NULL, bf16, pp);
  /* key mask semantics of key_padding_mask (280-294): None when no frame
   * is padding */
  const int32_t *kl = NULL;
  if (lengths) {
    for (int b = 0; b < B; ++b)
      if (lengths[b] < T) kl = lengths;
  }
  if (mode == ORC_DIRECT) {
    orc_relpos_attention(q, k, v, pp, ow.u, ow.v, B, T, T, D, H, NULL, kl, ctx,
                         0, cx);
  } else {
    /* q_with_bias_u / q_with_bias_v (506-508), bf16 adds round */
    float *qu = (float *)malloc(sizeof(float) * n);
    float *qv = (float *)malloc(sizeof(float) * n);
#pragma omp parallel for schedule(static)
    for (size_t e = 0; e < n; ++e) {
      const int col = (int)(e % (size_t)D);
      float a = q[e] + ow.u[col], c = q[e] + ow.v[col];
      qu[e] = bf16 ? orc_bf16_round(a) : a;
      qv[e] = bf16 ? orc_bf16_round(c) : c;
    }
    const int64_t budget = max_score_elements > 0 ? max_score_elements : INT64_MAX;
    const int block = orc_query_block_size(B * H, T, budget);
    for (int start = 0; start < T; start += block) {
      const int end = start + block < T ? start + block : T;
      ref_algo_block(qu, qv, k, v, pp, B, H, T, dh, D, start, end, kl, ctx,
                     bf16, cx);
    }
    free(qu);
    free(qv);
  }
  (void)dh;
  if (bf16) orc_bf16_round_array(cx, (int64_t)n);
  /* linear_out (565) */
  linear_r(cx, B * T, D, ow.wo, D, ow.bo, bf16, out);
  free(xx); free(pe); free(q); free(k); free(v); free(pp); free(cx);
  free_weights(&ow);
  return 0;
}

/* forward_with_cache, attention.rs:606-816. */
int orc_mha_forward_with_cache(const float *x, int B, int T, int D, int H,
                               const orc_mha_weights *w, const float *pos_emb,
                               const float *cache, int C, const uint8_t *mask,
                               int mask_is_bool, int cache_drop_size, int bf16,
                               float *out, float *new_cache) {
  const int q_keep = T - cache_drop_size > 0 ? T - cache_drop_size : 0;
  const int total = cache ? C + T : T;
  const int P = 2 * total - 1;
  owned_weights ow;
  cast_weights(w, D, H, bf16, &ow);
  float *kv_in = (float *)malloc(sizeof(float) * (size_t)B * total * D);
  /* kv_input = concat(cache, x) along time (650) */
  for (int b = 0; b < B; ++b) {
    if (cache)
      memcpy(kv_in + (size_t)b * total * D, cache + (size_t)b * C * D,
             sizeof(float) * (size_t)C * D);
    memcpy(kv_in + ((size_t)b * total + (total - T)) * D, x + (size_t)b * T * D,
           sizeof(float) * (size_t)T * D);
  }
  int nc_len;
  /* new cache = concat(cache[q_keep:], x[:q_keep]) (665-684), or x[:q_keep]
   * without a cache (689-694) */
  if (cache) {
    if (q_keep > 0) {
      const int keep_old = C - q_keep > 0 ? C - q_keep : 0;
      nc_len = keep_old + q_keep;
      for (int b = 0; b < B; ++b) {
        float *nb = new_cache + (size_t)b * nc_len * D;
        if (keep_old)
          memcpy(nb, cache + ((size_t)b * C + q_keep) * D,
                 sizeof(float) * (size_t)keep_old * D);
        memcpy(nb + (size_t)keep_old * D, x + (size_t)b * T * D,
               sizeof(float) * (size_t)q_keep * D);
      }
    } else {
      nc_len = C;
      memcpy(new_cache, cache, sizeof(float) * (size_t)B * C * D);
    }
  } else {
    nc_len = q_keep;
    for (int b = 0; b < B; ++b)
      memcpy(new_cache + (size_t)b * q_keep * D, x + (size_t)b * T * D,
             sizeof(float) * (size_t)q_keep * D);
  }
  float *xx = dup_round(x, (size_t)B * T * D, bf16);
  if (bf16) orc_bf16_round_array(kv_in, (int64_t)B * total * D);
  float *pe = dup_round(pos_emb, (size_t)P * D, bf16);
  float *q = (float *)malloc(sizeof(float) * (size_t)B * T * D);
  float *k = (float *)malloc(sizeof(float) * (size_t)B * total * D);
  float *v = (float *)malloc(sizeof(float) * (size_t)B * total * D);
  float *pp = (float *)malloc(sizeof(float) * (size_t)P * D);
  float *cx = (float *)malloc(sizeof(float) * (size_t)B * T * D);
  linear_r(xx, B * T, D, ow.wq, D, ow.bq, bf16, q);      /* 718 */
  linear_r(kv_in, B * total, D, ow.wk, D, ow.bk, bf16, k); /* 721 */
  linear_r(kv_in, B * total, D, ow.wv, D, ow.bv, bf16, v); /* 722 */
  linear_r(pe, P, D, ow.wp, D, NULL, bf16, pp);          /* 755 */
  /* The fused SDPA with an additive mask and the unfused boolean path
   * agree on every row that sees a key; rows that see nothing are zero on
   * the boolean path (786-789) and would be NaN on the additive one, which
   * the encoder never builds (conformer.rs:907-921). */
  (void)mask_is_bool;
  orc_relpos_attention(q, k, v, pp, ow.u, ow.v, B, T, total, D, H, mask, NULL,
                       NULL, 0, cx);
  if (bf16) orc_bf16_round_array(cx, (int64_t)B * T * D);
  linear_r(cx, B * T, D, ow.wo, D, ow.bo, bf16, out); /* 807 */
  free(kv_in); free(xx); free(pe); free(q); free(k); free(v); free(pp); free(cx);
  free_weights(&ow);
  return nc_len;
}

/* ConformerEncoder::forward_streaming's per-layer attention handling,
 * conformer.rs:883-1037. */
int orc_stream_layer_step(const float *x, int B, int T, int D, int H,
                          const orc_mha_weights *w, const float *pos_emb,
                          float *h_cache, int C, int filled, int valid,
                          int left, int right, int chunked, int cache_drop_size,
                          int bf16, float *out) {
  const int total = C + T;
  if (filled < 0) filled = 0;
  if (filled > C) filled = C;
  if (valid > T) valid = T;
  uint8_t *vis = (uint8_t *)malloc((size_t)T * total);
  orc_create_attention_mask(left, right, chunked, total, C, filled, T, valid, vis);
  int all_visible = 1;
  for (size_t e = 0; e < (size_t)T * total; ++e)
    if (!vis[e]) { all_visible = 0; break; }
  const uint8_t *mask = all_visible ? NULL : vis;
  const int is_bool = !all_visible && valid < T;
  const int q_keep = T - cache_drop_size > 0 ? T - cache_drop_size : 0;
  const int nc_cap = C + T;
  float *nc = (float *)malloc(sizeof(float) * (size_t)B * nc_cap * D);
  const int nc_len = orc_mha_forward_with_cache(x, B, T, D, H, w, pos_emb,
                                                h_cache, C, mask, is_bool,
                                                cache_drop_size, bf16, out, nc);
  /* re-pad with zeros in front or keep the newest C frames (983-1000) */
  for (int b = 0; b < B; ++b) {
    float *hb = h_cache + (size_t)b * C * D;
    const float *nb = nc + (size_t)b * nc_len * D;
    if (nc_len < C) {
      memset(hb, 0, sizeof(float) * (size_t)(C - nc_len) * D);
      memcpy(hb + (size_t)(C - nc_len) * D, nb, sizeof(float) * (size_t)nc_len * D);
    } else {
      memcpy(hb, nb + (size_t)(nc_len - C) * D, sizeof(float) * (size_t)C * D);
    }
  }
  free(nc);
  free(vis);
  /* fill level: min(len + keep, C) (1027-1037) */
  const int next = filled + q_keep < C ? filled + q_keep : C;
  return next;
}

/* ------------------------------------------------------ Conformer block */

static inline float rnd(float v, int bf16) { return bf16 ? orc_bf16_round(v) : v; }

/* nn::LayerNorm (eps 1e-5): f32 statistics, one rounding of the output
 * (MLX's fused layer norm). g, b already in the compute dtype. */
static void layer_norm_r(const float *x, int64_t rows, int D, const float *g,
                         const float *b, int bf16, float *y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * D;
    double s = 0.0;
    for (int c = 0; c < D; ++c) s += xr[c];
    const float mean = (float)(s / D);
    double q = 0.0;
    for (int c = 0; c < D; ++c) {
      const double d = xr[c] - mean;
      q += d * d;
    }
    const float inv = 1.0f / sqrtf((float)(q / D) + 1e-5f);
    for (int c = 0; c < D; ++c)
      y[r * D + c] = rnd((xr[c] - mean) * inv * g[c] + b[c], bf16);
  }
}

/* sigmoid and x * sigmoid(x) as two rounded ops (mlx nn::silu). */
static inline float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

static void silu_r(float *x, int64_t n, int bf16) {
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < n; ++e) x[e] = rnd(x[e] * rnd(sigm(x[e]), bf16), bf16);
}

/* FeedForward (2081-2087) and the half-step residual (1723-1726). */
static void ff_residual(float *xx, int64_t M, int D, int ff, const orc_lin *l1,
                        const orc_lin *l2, const float *g, const float *b, int bf16,
                        float *h, float *hid, float *tmp) {
  layer_norm_r(xx, M, D, g, b, bf16, h);
  linear_r(h, (int)M, D, l1->w, ff, l1->b, bf16, hid);
  silu_r(hid, M * ff, bf16);
  linear_r(hid, (int)M, ff, l2->w, D, l2->b, bf16, tmp);
  const float half = 0.5f;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < M * D; ++e) xx[e] = rnd(xx[e] + rnd(half * tmp[e], bf16), bf16);
}

int orc_block_forward(const float *x, int B, int T, int D, int H, int ff, int K,
                      int causal, int conv_norm, const orc_block_weights *w,
                      const float *pos_emb, const int32_t *lengths,
                      const orc_context *ctx, int bf16, float *out) {
  if (B <= 0 || T <= 0 || D <= 0 || H <= 0 || D % H || ff <= 0 || K <= 0) return -1;
  const int64_t M = (int64_t)B * T;
  const size_t n = (size_t)M * D;
  /* set_dtype: every block parameter in the compute dtype */
  float *ng[5], *nb[5];
  for (int i = 0; i < 5; ++i) {
    ng[i] = dup_round(w->norm_g[i], D, bf16);
    nb[i] = dup_round(w->norm_b[i], D, bf16);
  }
  const orc_lin *src[6] = {&w->ff1_1, &w->ff1_2, &w->pw1, &w->pw2, &w->ff2_1, &w->ff2_2};
  const int lin_n[6] = {ff, D, 2 * D, D, ff, D}, lin_k[6] = {D, ff, D, D, D, ff};
  orc_lin L[6];
  for (int i = 0; i < 6; ++i) {
    L[i].w = dup_round(src[i]->w, (size_t)lin_n[i] * lin_k[i], bf16);
    L[i].b = dup_round(src[i]->b, (size_t)lin_n[i], bf16);
  }
  float *dw_w = dup_round(w->dw_w, (size_t)D * K, bf16);
  float *dw_b = dup_round(w->dw_b, D, bf16);
  float *cn_g = dup_round(w->cn_g, D, bf16), *cn_b = dup_round(w->cn_b, D, bf16);
  float *cn_m = conv_norm == 0 ? dup_round(w->cn_m, D, bf16) : NULL;
  float *cn_v = conv_norm == 0 ? dup_round(w->cn_v, D, bf16) : NULL;
  const float eps = rnd(1e-5f, bf16);  /* bn.eps cast to the dtype (2130) */
  /* PaddingMask::new (1604-1614): None when nothing is padded */
  const int32_t *kl = NULL;
  if (lengths)
    for (int b = 0; b < B; ++b)
      if (lengths[b] < T) kl = lengths;

  float *xx = dup_round(x, n, bf16);
  float *h = (float *)malloc(sizeof(float) * n);
  float *tmp = (float *)malloc(sizeof(float) * n);
  float *hid = (float *)malloc(sizeof(float) * (size_t)M * (ff > 2 * D ? ff : 2 * D));
  float *glu = (float *)malloc(sizeof(float) * n);

  /* 1703-1726 */
  ff_residual(xx, M, D, ff, &L[0], &L[1], ng[0], nb[0], bf16, h, hid, tmp);
  /* 1750-1785: x += self_attn(LN x) */
  layer_norm_r(xx, M, D, ng[1], nb[1], bf16, h);
  orc_mha_forward(h, B, T, D, H, &w->attn, pos_emb, kl, ctx, ORC_DIRECT, bf16,
                  0, tmp);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < (int64_t)n; ++e) xx[e] = rnd(xx[e] + tmp[e], bf16);
  /* 1797-1824: x += conv(LN x) */
  layer_norm_r(xx, M, D, ng[2], nb[2], bf16, h);
  linear_r(h, (int)M, D, L[2].w, 2 * D, L[2].b, bf16, hid); /* pointwise_conv1 */
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < M; ++r) {
    const int b = (int)(r / T), t = (int)(r % T);
    const int valid = !kl || t < kl[b];
    for (int c = 0; c < D; ++c) {
      const float a = hid[r * 2 * D + c], g = hid[r * 2 * D + D + c];
      const float v = rnd(a * rnd(sigm(g), bf16), bf16); /* GLU 2275-2281 */
      glu[r * D + c] = valid ? v : 0.0f;                 /* 2282-2285 */
    }
  }
  const int pad = causal ? K - 1 : (K - 1) / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t)
      for (int c = 0; c < D; ++c) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
          const int ts = t + k - pad;
          if (ts >= 0 && ts < T) acc += dw_w[(size_t)c * K + k] * glu[((size_t)b * T + ts) * D + c];
        }
        if (dw_b) acc = rnd(acc, bf16) + dw_b[c];
        h[((size_t)b * T + t) * D + c] = rnd(acc, bf16);
      }
  if (conv_norm == 0) {
    /* BatchNorm, inference: (x - mean) * rsqrt(var + eps) * weight + bias */
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < (int64_t)n; ++e) {
      const int c = (int)(e % D);
      const float xm = rnd(h[e] - cn_m[c], bf16);
      const float inv = rnd(1.0f / sqrtf(rnd(cn_v[c] + eps, bf16)), bf16);
      const float nv = rnd(xm * inv, bf16);
      h[e] = rnd(rnd(nv * cn_g[c], bf16) + cn_b[c], bf16);
    }
  } else {
    layer_norm_r(h, M, D, cn_g, cn_b, bf16, h);
  }
  silu_r(h, (int64_t)n, bf16);
  linear_r(h, (int)M, D, L[3].w, D, L[3].b, bf16, tmp); /* pointwise_conv2 */
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < (int64_t)n; ++e) xx[e] = rnd(xx[e] + tmp[e], bf16);
  /* 1826-1858 */
  ff_residual(xx, M, D, ff, &L[4], &L[5], ng[3], nb[3], bf16, h, hid, tmp);
  /* 1861: final norm */
  layer_norm_r(xx, M, D, ng[4], nb[4], bf16, out);

  free(xx); free(h); free(tmp); free(hid); free(glu);
  for (int i = 0; i < 5; ++i) { free(ng[i]); free(nb[i]); }
  for (int i = 0; i < 6; ++i) { free((void *)L[i].w); free((void *)L[i].b); }
  free(dw_w); free(dw_b); free(cn_g); free(cn_b); free(cn_m); free(cn_v);
  return 0;
}

/* ------------------------------------------ dw_striding subsampling */

/* Subsampling::new (conformer.rs:1118-1123): strides = log2(factor) for
 * 2, 4, 8; any other factor gets 2. */
int orc_subsampling_strides(int factor) {
  return factor == 2 ? 1 : factor == 4 ? 2 : factor == 8 ? 3 : 2;
}

/* One stride-2, kernel-3 conv along an axis (conformer.rs:1306-1326 and the
 * conv output size): causal pads (k-1, s-1) = (2, 1), floor(n/2) + 1;
 * otherwise padding 1 on both sides, floor((n-1)/2) + 1 (floor division,
 * so 0 -> 0). */
static int sub_conv_len(int n, int causal) {
  if (causal) {
    const int p = n;  /* n + (k-1) + (s-1) - k */
    return (p >= 0 ? p / 2 : -((-p + 1) / 2)) + 1;
  }
  const int p = n - 1;
  return (p >= 0 ? p / 2 : -((-p + 1) / 2)) + 1;
}

/* Subsampling::output_length (1315-1327). */
int orc_subsampling_out_len(int len, int factor, int causal) {
  const int s = orc_subsampling_strides(factor);
  for (int i = 0; i < s; ++i) len = sub_conv_len(len, causal);
  return len > 0 ? len : 0;
}

/* compute_freq_output_size (1220-1244). */
int orc_subsampling_feat_out(int feat_in, int factor, int causal) {
  const int s = orc_subsampling_strides(factor);
  int f = feat_in;
  for (int i = 0; i < s; ++i) f = causal ? f / 2 + 1 : (f + 2 - 3) / 2 + 1;
  return f;
}

/* A 3x3 stride-2 conv over NHWC x [B, Ti, Fi, cin] -> y [B, To, Fo, C]:
 * cin == 1 is the first conv (every output channel reads channel 0),
 * cin == C the depthwise one (groups = C); w [C, 3, 3, 1] (MLX layout),
 * input (2*to + kt - pad, 2*fo + kf - pad), zero outside the input.  The
 * conv output is rounded, then the bias add (nn::Conv2d::forward), then the
 * optional ReLU. */
static void sub_conv3x3_s2(const float *x, int B, int Ti, int Fi, int cin, int C,
                           int pad, const float *w, const float *bias, int relu,
                           int bf16, float *y, int To, int Fo) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int to = 0; to < To; ++to)
      for (int fo = 0; fo < Fo; ++fo)
        for (int c = 0; c < C; ++c) {
          const int ci = cin == 1 ? 0 : c;
          float acc = 0.0f;
          for (int kt = 0; kt < 3; ++kt) {
            const int ti = 2 * to + kt - pad;
            if (ti < 0 || ti >= Ti) continue;
            for (int kf = 0; kf < 3; ++kf) {
              const int fi = 2 * fo + kf - pad;
              if (fi < 0 || fi >= Fi) continue;
              acc += x[(((size_t)b * Ti + ti) * Fi + fi) * cin + ci] * w[c * 9 + kt * 3 + kf];
            }
          }
          float v = rnd(acc, bf16);
          if (bias) v = rnd(v + bias[c], bf16);
          if (relu && v < 0.0f) v = 0.0f;
          y[(((size_t)b * To + to) * Fo + fo) * C + c] = v;
        }
}

/* Subsampling::forward_frames (conformer.rs:1413-1555), dw_striding:
 *   x [B, T, F] -> NHWC [B, T, F, 1]; (causal_pad_2d, 66-80: (2, 1) on time
 *   and frequency, then padding 0; otherwise padding 1)
 *   conv.0 (1 -> C, 3x3, stride 2) + ReLU
 *   per further stride: depthwise 3x3 stride 2 (groups C), pointwise 1x1
 *   (C -> C), ReLU
 *   [B, T', F', C] -> [B, T', C, F'] -> [B, T', C*F'] -> out linear.
 * With bf16 every parameter and the input are rounded (set_dtype, 1098-1108,
 * and the encoder's as_dtype, 519) and every op's output too.
 * out [B, T', d_model], T' = orc_subsampling_out_len(T). */
int orc_subsampling_forward(const float *x, int B, int T, int F, int C, int factor,
                            int causal, int d_model, const orc_subsampling_weights *w,
                            int bf16, float *out) {
  if (B <= 0 || T <= 0 || F <= 0 || C <= 0 || d_model <= 0) return -1;
  const int S = orc_subsampling_strides(factor);
  const int pad = causal ? 2 : 1;
  int Ti = T, Fi = F;
  float *cur = dup_round(x, (size_t)B * T * F, bf16);
  int cin = 1;
  for (int s = 0; s < S; ++s) {
    const int To = sub_conv_len(Ti, causal), Fo = sub_conv_len(Fi, causal);
    const size_t n = (size_t)B * To * Fo * C;
    float *y = (float *)malloc(sizeof(float) * n);
    float *cw = dup_round(s == 0 ? w->conv0_w : w->dw_w[s - 1], (size_t)C * 9, bf16);
    float *cb = dup_round(s == 0 ? w->conv0_b : w->dw_b[s - 1], (size_t)C, bf16);
    sub_conv3x3_s2(cur, B, Ti, Fi, cin, C, pad, cw, cb, s == 0, bf16, y, To, Fo);
    free(cw);
    free(cb);
    free(cur);
    cur = y;
    if (s > 0) {
      /* pointwise conv: w [C, 1, 1, C] is a [C, C] linear, then ReLU */
      float *pw = dup_round(w->pw_w[s - 1], (size_t)C * C, bf16);
      float *pb = dup_round(w->pw_b[s - 1], (size_t)C, bf16);
      float *z = (float *)malloc(sizeof(float) * n);
      linear_r(cur, (int)(n / C), C, pw, C, pb, bf16, z);
#pragma omp parallel for schedule(static)
      for (int64_t e = 0; e < (int64_t)n; ++e)
        if (z[e] < 0.0f) z[e] = 0.0f;
      free(pw);
      free(pb);
      free(cur);
      cur = z;
    }
    Ti = To;
    Fi = Fo;
    cin = C;
  }
  /* 1519-1536: [B, T', F', C] -> [B, T', C, F'] flattened */
  const int K = C * Fi;
  float *flat = (float *)malloc(sizeof(float) * (size_t)B * Ti * K);
#pragma omp parallel for collapse(2) schedule(static)
  for (int r = 0; r < B * Ti; ++r)
    for (int f = 0; f < Fi; ++f)
      for (int c = 0; c < C; ++c)
        flat[(size_t)r * K + (size_t)c * Fi + f] = cur[((size_t)r * Fi + f) * C + c];
  free(cur);
  float *ow = dup_round(w->out_w, (size_t)d_model * K, bf16);
  float *ob = dup_round(w->out_b, (size_t)d_model, bf16);
  linear_r(flat, B * Ti, K, ow, d_model, ob, bf16, out);
  free(ow);
  free(ob);
  free(flat);
  return 0;
}

/* ------------------------------------------- streaming Conformer block */

/* ConformerBlock::forward_with_cache (conformer.rs:1877-1967) as
 * ConformerEncoder::forward_streaming drives it (883-1000): FF1 half step;
 * the attention on LN(x) through orc_stream_layer_step (mask from the
 * first stream's fill level and valid length, ring slide and re-pad of
 * h_cache [B,C,D] in place); ConvolutionModule::forward_with_cache
 * (2332-2400): pointwise_conv1 + GLU, frames t >= valid zeroed (the pad mask,
 * 929-941), concatenated after conv_cache [B,K-1,D] (time-major here; the
 * reference keeps [B,D,K-1]), the new conv cache = the last K-1 frames of
 * the concatenation, the depthwise conv over it without padding (T outputs),
 * the conv norm, SiLU, pointwise_conv2; FF2 half step; final LayerNorm.
 * Rounding as orc_block_forward.  Returns the next fill level. */
int orc_stream_block_step(const float *x, int B, int T, int D, int H, int ff, int K,
                          int conv_norm, const orc_block_weights *w, const float *pos_emb,
                          float *h_cache, int C, float *conv_cache, int filled, int valid,
                          int left, int right, int chunked, int cache_drop_size, int bf16,
                          float *out) {
  if (B <= 0 || T <= 0 || D <= 0 || H <= 0 || D % H || ff <= 0 || K <= 0) return -1;
  const int64_t M = (int64_t)B * T;
  const size_t n = (size_t)M * D;
  float *ng[5], *nb[5];
  for (int i = 0; i < 5; ++i) {
    ng[i] = dup_round(w->norm_g[i], D, bf16);
    nb[i] = dup_round(w->norm_b[i], D, bf16);
  }
  const orc_lin *src[6] = {&w->ff1_1, &w->ff1_2, &w->pw1, &w->pw2, &w->ff2_1, &w->ff2_2};
  const int lin_n[6] = {ff, D, 2 * D, D, ff, D}, lin_k[6] = {D, ff, D, D, D, ff};
  orc_lin L[6];
  for (int i = 0; i < 6; ++i) {
    L[i].w = dup_round(src[i]->w, (size_t)lin_n[i] * lin_k[i], bf16);
    L[i].b = dup_round(src[i]->b, (size_t)lin_n[i], bf16);
  }
  float *dw_w = dup_round(w->dw_w, (size_t)D * K, bf16);
  float *dw_b = dup_round(w->dw_b, D, bf16);
  float *cn_g = dup_round(w->cn_g, D, bf16), *cn_b = dup_round(w->cn_b, D, bf16);
  float *cn_m = conv_norm == 0 ? dup_round(w->cn_m, D, bf16) : NULL;
  float *cn_v = conv_norm == 0 ? dup_round(w->cn_v, D, bf16) : NULL;
  const float eps = rnd(1e-5f, bf16);
  if (valid > T) valid = T;
  if (valid < 0) valid = 0;

  float *xx = dup_round(x, n, bf16);
  float *h = (float *)malloc(sizeof(float) * n);
  float *tmp = (float *)malloc(sizeof(float) * n);
  float *hid = (float *)malloc(sizeof(float) * (size_t)M * (ff > 2 * D ? ff : 2 * D));
  const int Tc = K - 1 + T;
  float *cat = (float *)malloc(sizeof(float) * (size_t)B * Tc * D);

  ff_residual(xx, M, D, ff, &L[0], &L[1], ng[0], nb[0], bf16, h, hid, tmp);
  /* x += MHA(LN x) with the cache */
  layer_norm_r(xx, M, D, ng[1], nb[1], bf16, h);
  const int next = orc_stream_layer_step(h, B, T, D, H, &w->attn, pos_emb, h_cache, C, filled,
                                         valid, left, right, chunked, cache_drop_size, bf16, tmp);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < (int64_t)n; ++e) xx[e] = rnd(xx[e] + tmp[e], bf16);
  /* x += Conv(LN x) with the cache */
  layer_norm_r(xx, M, D, ng[2], nb[2], bf16, h);
  linear_r(h, (int)M, D, L[2].w, 2 * D, L[2].b, bf16, hid);
  for (int b = 0; b < B; ++b) {
    memcpy(cat + (size_t)b * Tc * D, conv_cache + (size_t)b * (K - 1) * D,
           sizeof(float) * (size_t)(K - 1) * D);
    for (int t = 0; t < T; ++t)
      for (int c = 0; c < D; ++c) {
        const int64_t r = (int64_t)b * T + t;
        const float a = hid[r * 2 * D + c], g = hid[r * 2 * D + D + c];
        const float v = rnd(a * rnd(sigm(g), bf16), bf16);
        cat[((size_t)b * Tc + K - 1 + t) * D + c] = t < valid ? v : 0.0f;
      }
    memcpy(conv_cache + (size_t)b * (K - 1) * D, cat + ((size_t)b * Tc + T) * D,
           sizeof(float) * (size_t)(K - 1) * D);
  }
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int t = 0; t < T; ++t)
      for (int c = 0; c < D; ++c) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k)
          acc += dw_w[(size_t)c * K + k] * cat[((size_t)b * Tc + t + k) * D + c];
        if (dw_b) acc = rnd(acc, bf16) + dw_b[c];
        h[((size_t)b * T + t) * D + c] = rnd(acc, bf16);
      }
  if (conv_norm == 0) {
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < (int64_t)n; ++e) {
      const int c = (int)(e % D);
      const float xm = rnd(h[e] - cn_m[c], bf16);
      const float inv = rnd(1.0f / sqrtf(rnd(cn_v[c] + eps, bf16)), bf16);
      const float nv = rnd(xm * inv, bf16);
      h[e] = rnd(rnd(nv * cn_g[c], bf16) + cn_b[c], bf16);
    }
  } else {
    layer_norm_r(h, M, D, cn_g, cn_b, bf16, h);
  }
  silu_r(h, (int64_t)n, bf16);
  linear_r(h, (int)M, D, L[3].w, D, L[3].b, bf16, tmp);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < (int64_t)n; ++e) xx[e] = rnd(xx[e] + tmp[e], bf16);
  ff_residual(xx, M, D, ff, &L[4], &L[5], ng[3], nb[3], bf16, h, hid, tmp);
  layer_norm_r(xx, M, D, ng[4], nb[4], bf16, out);

  free(xx); free(h); free(tmp); free(hid); free(cat);
  for (int i = 0; i < 5; ++i) { free(ng[i]); free(nb[i]); }
  for (int i = 0; i < 6; ++i) { free((void *)L[i].w); free((void *)L[i].b); }
  free(dw_w); free(dw_b); free(cn_g); free(cn_b); free(cn_m); free(cn_v);
  return next;
}
