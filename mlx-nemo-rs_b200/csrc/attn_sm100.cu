// attn_sm100.cu -- fused offline relative-position attention on tcgen05.
//
// Computes, per (batch b, head h, 128-query tile), what the reference's
// RelPositionMultiHeadAttention::forward_blocked does between the
// projections (src/asr/modules/encoders/attention.rs:501-556):
//
//   S[i,j] = ((q_i + u) . k_j + rel_shift((q + v) . P^T)[i,j]) / sqrt(dh)
//   out_i  = softmax_j(S[i,j] + mask) . V
//
// without materialising the [rows, 2T-1] positional score matrix.
//
// Positional term.  rel_shift leaves column j of row i holding P row
// r = T-1-i+j (attention.rs:1248-1282).  For query tile [i0, i0+128) and key
// tile t (keys j0+128t ..) the rows needed are rbase+128t + x with
// x = 127-il+jl in [0, 255) (il, jl: row/key within the tiles), i.e. P chunks
// t and t+1 of 128 rows each (chunk c = rows rbase+128c ..).  The product
// BD_c = Q . P_c^T depends only on the chunk, so each chunk is multiplied
// once and kept in a two-slot TMEM ring for the two key tiles that read it:
// per key tile the tensor cores do S (128 cols), one BD chunk (128) and P.V
// (128) -- exactly the algorithmic work.  Each row reads its 128 BD columns
// at offset 127-il: a per-lane skew, done in registers with a 5-stage
// predicated barrel shift over a 64-column window.
//
// Biases.  The CTA's query tile is staged once and turned into two bf16
// tiles, q+u (A operand of the content product) and q+v (A operand of the
// positional product) -- the same bf16 adds as the reference's
// q_with_bias_u / q_with_bias_v (attention.rs:506-508).
//
// Masks.  Key padding (attention.rs:280-294) and AttentionContext windows
// (attention.rs:232-272) reduce to one visible key interval per query row.
//
// Geometry.  Frame indices are global (AttnGeom): a launch may cover a
// slice of the query rows, read q|k|v from a buffer that starts at any frame
// and has any row and batch strides (the time-major halo buffer of a
// sequence-split forward), and read only the slice of the P table that its
// relative positions reach -- TMA loads of P rows outside that slice, and of
// frames outside the buffer, return zeros, and every pair they feed is masked.
//
// Memory.  Shared: q+u, q+v, one {K tile, P chunk} stage, 2 x V,
// probabilities (the bf16 A operand of P.V) -- 224 KB.  TMEM: S [0,128), BD
// slots [128,256) and [256,384), O [384,512).  The MMAs of key tile t+1 run
// while the softmax of tile t finishes (its TMEM reads come first); the
// next {K, P} stage loads as soon as the tile's MMAs have read it and V is
// loaded a tile ahead.
//
// Warps 0-7 (softmax): warp w owns TMEM lane quadrant w&3 (one query row
// per thread) and key half w>>2 (64 keys); the two threads of a row swap
// their row maxima through shared memory.  Warp 8: TMEM owner; its lane 0
// issues every TMA load and MMA.  Online softmax in the log2 domain; the
// output is rescaled only when a row maximum grows by more than 2^8 (exact:
// the final normalisation uses the same maximum).  Every wait is bounded.
#include <math.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kDh = 128;
constexpr int kTile = 128;
constexpr uint32_t kHalf = kTile * 64 * 2;  // 16 KB: 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kHalf;  // 32 KB: 128 rows x 128 bf16
constexpr int kSoftmaxThreads = 256;
constexpr int kSoftmaxWarps = kSoftmaxThreads / 32;
constexpr int kThreads = kSoftmaxThreads + 32;

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t kOffQu = 0;
constexpr uint32_t kOffQv = kOffQu + kTileBytes;
constexpr uint32_t kOffK = kOffQv + kTileBytes;
constexpr uint32_t kOffP = kOffK + kTileBytes;
constexpr uint32_t kOffV = kOffP + kTileBytes;       // 2 slots
constexpr uint32_t kOffPr = kOffV + 2 * kTileBytes;
constexpr uint32_t kOffX = kOffPr + kTileBytes;      // [2 parity][2 halves][128] f32
constexpr uint32_t kOffBar = kOffX + 2048;

struct Bars {
  uint64_t q, prep, p0, kp, v[2], s, sfree, p, o, x;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kSmemBytes = kOffBar + sizeof(Bars);
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr uint32_t kStageTx = 2 * kTileBytes;  // K tile + P chunk

// 2^x with the MUFU approximation (flush-to-zero; inputs here are <= 8).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One arrival per warp, after every lane's prior writes (each lane fenced
// what it needs before calling this).
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Bounded wait whose outcome is the same for every lane of the warp (the
// tcgen05 loads/stores that follow are warp-collective).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const bool mine = mbar_wait(bar, parity, err, code);
  return __all_sync(0xffffffffu, mine);
}

// Visible key interval [lo, hi) of query row i (AttentionContext::block_mask,
// attention.rs:232-272, intersected with key_padding_mask, 280-294).
__device__ __forceinline__ void row_interval(const AttnContextDev& c, int i, int kbeg, int kend,
                                             int& lo, int& hi) {
  lo = kbeg;
  hi = kend;
  if (!c.has) return;
  if (c.chunked && c.right >= 0) {
    const int chunk = c.right + 1;
    const int lc = c.left >= 0 ? c.left / chunk : 10000;
    const int ci = i / chunk;
    lo = max(lo, (ci - lc) * chunk);
    hi = min(hi, (ci + 1) * chunk);
  } else {
    if (c.left >= 0) lo = max(lo, i - c.left);
    if (!c.chunked && c.right >= 0) hi = min(hi, i + c.right + 1);
  }
}

// 8 consecutive MMAs over the 128-deep head dimension (two 64-column
// swizzled halves of each operand, 32 bytes per K=16 step).
__device__ __forceinline__ void mma_k128(uint32_t tmem_d, uint32_t a, uint32_t b, uint32_t idesc,
                                         bool acc_first) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
    umma_ss(tmem_d, sdesc_sw128(a + off, 16, 1024), sdesc_sw128(b + off, 16, 1024), idesc,
            (k > 0) || acc_first);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_kernel(const __grid_constant__ CUtensorMap map_qkv,  // [B][tbuf][3D] bf16
                       const __grid_constant__ CUtensorMap map_p,    // [p_rows][D] bf16
                       const float* __restrict__ pos_u, const float* __restrict__ pos_v,
                       const __grid_constant__ CUtensorMap map_out,  // [B][rows][D] bf16
                       const int32_t* __restrict__ key_len, AttnContextDev ctx, AttnGeom g,
                       __nv_bfloat16* __restrict__ out, int H, int pf_stride, int* err) {
  // Dynamic shared memory starts 1024-byte aligned when, as here, the kernel
  // has no static shared memory; checked, since the swizzle atoms need it.
  extern __shared__ __align__(1024) uint8_t smem[];
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(err, 0, kDevBadArgs);
    return;
  }
  uint8_t* sQu = smem + kOffQu;
  uint8_t* sQv = smem + kOffQv;
  uint8_t* sK = smem + kOffK;
  uint8_t* sP = smem + kOffP;
  uint8_t* sV = smem + kOffV;
  uint8_t* sPr = smem + kOffPr;

  const int warp = warp_id();
  const int lane = lane_id();
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int D = H * kDh;
  const int i0 = g.q_lo + qt * kTile;  // global frame of the tile's first row

  // Keys visible to any row of this tile: one interval [jlo, jhi) of global
  // frames, within the frames the buffer holds.
  int klen = g.Tg;
  if (key_len) klen = min(g.Tg, max(key_len[b], 1));
  const int kend = min(klen, g.k_hi);
  int jlo, jhi;
  {
    int lo0, hi0, lo1, hi1;
    const int i1 = min(i0 + kTile - 1, g.q_hi - 1);
    row_interval(ctx, i0, g.k_lo, kend, lo0, hi0);
    row_interval(ctx, i1, g.k_lo, kend, lo1, hi1);
    jlo = min(lo0, lo1);
    jhi = max(hi0, hi1);
  }
  // Query tiles wholly past the utterance's length are padding: their
  // outputs are unspecified in the reference (conformer.rs:1590-1593) and
  // are written as zeros here.
  const bool padded_tile = key_len && i0 >= klen;
  const int j0 = jlo;
  const int nt = (jhi > jlo && !padded_tile) ? (jhi - j0 + kTile - 1) / kTile : 0;
  // first P row of chunk 0, as a row of the p buffer (may be negative:
  // rows outside the buffer load as zeros and only meet masked pairs)
  const int rbase = g.Tg - kTile - i0 + j0 - g.p_base;

  if (nt == 0) {  // no visible key (padding): zeros, without barriers or TMEM
    const int rows = min(kTile, g.q_hi - i0);
    __nv_bfloat16* ob = out + static_cast<size_t>(b) * g.out_bs + h * kDh;
    for (int k = threadIdx.x; k < rows * 16; k += blockDim.x) {
      const int rr = k >> 4, c = k & 15;
      *reinterpret_cast<uint4*>(ob + static_cast<size_t>(i0 + rr - g.out_base) * D + c * 8) =
          make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->q, 1);
    mbar_init(&bars->prep, kSoftmaxWarps);
    mbar_init(&bars->p0, 1);
    mbar_init(&bars->kp, 1);
    mbar_init(&bars->v[0], 1);
    mbar_init(&bars->v[1], 1);
    mbar_init(&bars->s, 1);
    mbar_init(&bars->sfree, kSoftmaxWarps);
    mbar_init(&bars->p, kSoftmaxWarps);
    mbar_init(&bars->o, 1);
    mbar_init(&bars->x, kSoftmaxWarps);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort;

  if (warp == 8) {
    // ------------------------------------------------ TMA + MMA issuer
    if (lane == 0 && nt > 0) {
      const int qcol = h * kDh, kcol = D + h * kDh, vcol = 2 * D + h * kDh;
      prefetch_tensormap(&map_qkv);
      prefetch_tensormap(&map_p);
      auto load_stage = [&](int t) {  // K_t and P chunk t+1
        mbar_arrive_expect_tx(&bars->kp, kStageTx);
        const int jt = j0 + t * kTile - g.base;
        tma_load_3d(sK, &map_qkv, &bars->kp, kcol, jt, b);
        tma_load_3d(sK + kHalf, &map_qkv, &bars->kp, kcol + 64, jt, b);
        const int prow = rbase + (t + 1) * kTile;
        tma_load_2d(sP, &map_p, &bars->kp, h * kDh, prow);
        tma_load_2d(sP + kHalf, &map_p, &bars->kp, h * kDh + 64, prow);
      };
      auto load_v = [&](int t) {
        uint64_t* bar = &bars->v[t & 1];
        uint8_t* dst = sV + (t & 1) * kTileBytes;
        mbar_arrive_expect_tx(bar, kTileBytes);
        tma_load_3d(dst, &map_qkv, bar, vcol, j0 + t * kTile - g.base, b);
        tma_load_3d(dst + kHalf, &map_qkv, bar, vcol + 64, j0 + t * kTile - g.base, b);
      };
      mbar_arrive_expect_tx(&bars->q, kTileBytes);
      tma_load_3d(sQu, &map_qkv, &bars->q, qcol, i0 - g.base, b);
      tma_load_3d(sQu + kHalf, &map_qkv, &bars->q, qcol + 64, i0 - g.base, b);
      // P chunk 0 is only read by the first BD MMA, so it is staged in the
      // probability buffer, which is free until the first softmax.
      mbar_arrive_expect_tx(&bars->p0, kTileBytes);
      tma_load_2d(sPr, &map_p, &bars->p0, h * kDh, rbase);
      tma_load_2d(sPr + kHalf, &map_p, &bars->p0, h * kDh + 64, rbase);
      load_stage(0);
      // The CTA that will start about one CTA-duration from now (index +
      // pf_stride, one per SM) finds its first Q, K and V tiles in L2: their
      // DRAM latency would otherwise sit on its prologue.
      {
        const int nx = gridDim.x, ny = gridDim.y;
        const int nxt = blockIdx.x + nx * (blockIdx.y + ny * blockIdx.z) + pf_stride;
        if (nxt < nx * ny * static_cast<int>(gridDim.z)) {
          const int qt2 = nxt % nx, h2 = (nxt / nx) % ny, b2 = nxt / (nx * ny);
          const int i2 = g.q_lo + qt2 * kTile;
          int klen2 = g.Tg;
          if (key_len) klen2 = min(g.Tg, max(key_len[b2], 1));
          if (!(key_len && i2 >= klen2)) {
            int lo0, hi0, lo1, hi1;
            row_interval(ctx, i2, g.k_lo, min(klen2, g.k_hi), lo0, hi0);
            row_interval(ctx, min(i2 + kTile - 1, g.q_hi - 1), g.k_lo, min(klen2, g.k_hi), lo1,
                         hi1);
            const int j2 = min(lo0, lo1) - g.base;
            for (int half = 0; half < 2; ++half) {
              tma_prefetch_3d(&map_qkv, h2 * kDh + 64 * half, i2 - g.base, b2);
              tma_prefetch_3d(&map_qkv, D + h2 * kDh + 64 * half, j2, b2);
              tma_prefetch_3d(&map_qkv, 2 * D + h2 * kDh + 64 * half, j2, b2);
            }
          }
        }
      }

      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t aQu = smem_u32(sQu), aQv = smem_u32(sQv), aK = smem_u32(sK);
      const uint32_t aV = smem_u32(sV), aP = smem_u32(sP), aPr = smem_u32(sPr);
      auto pv = [&](int t) {  // O (+)= probabilities(t) . V_t
        tc_fence_after();
        const uint32_t vb = aV + (t & 1) * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t offa = (k >> 2) * kHalf + (k & 3) * 32;
          umma_ss(tmem + 384, sdesc_sw128(aPr + offa, 16, 1024),
                  sdesc_sw128(vb + k * 2048, kHalf, 1024), idesc_pv, (t > 0) || (k > 0));
        }
        umma_commit(&bars->o);
      };
      bool ok = mbar_wait(&bars->prep, 0, err, kDevTimeoutEpi) &&
                mbar_wait(&bars->p0, 0, err, kDevTimeoutLoad);
      if (ok) {
        tc_fence_after();
        mma_k128(tmem + 128, aQv, aPr, idesc_kk, false);  // BD_0 -> slot 0
      }
      for (int t = 0; t < nt && ok; ++t) {
        ok = mbar_wait(&bars->kp, t & 1, err, kDevTimeoutLoad);
        if (ok && t > 0) ok = mbar_wait(&bars->sfree, (t - 1) & 1, err, kDevTimeoutEpi);
        if (!ok) break;
        tc_fence_after();
        mma_k128(tmem, aQu, aK, idesc_kk, false);  // S_t
        mma_k128(tmem + 128 + 128 * ((t + 1) & 1), aQv, aP, idesc_kk, false);  // BD_{t+1}
        umma_commit(&bars->s);
        if (t == 0) {  // V is first read after a whole softmax pass: load it
          load_v(0);   // behind the first MMAs' operands
          if (nt > 1) load_v(1);
        }
        // the stage is free once these MMAs have read it
        ok = mbar_wait(&bars->s, t & 1, err, kDevTimeoutMma);
        if (!ok) break;
        if (t + 1 < nt) load_stage(t + 1);
        if (t > 0) {  // P.V of the previous tile, then V for tile t+1 into its slot
          ok = mbar_wait(&bars->p, (t - 1) & 1, err, kDevTimeoutEpi) &&
               mbar_wait(&bars->v[(t - 1) & 1], ((t - 1) >> 1) & 1, err, kDevTimeoutLoad);
          if (!ok) break;
          pv(t - 1);
          ok = mbar_wait(&bars->o, (t - 1) & 1, err, kDevTimeoutMma);
          if (!ok) break;
          if (t + 1 < nt) load_v(t + 1);
        }
      }
      if (ok) {  // P.V of the last tile
        const int t = nt - 1;
        ok = mbar_wait(&bars->p, t & 1, err, kDevTimeoutEpi) &&
             mbar_wait(&bars->v[t & 1], (t >> 1) & 1, err, kDevTimeoutLoad);
        if (ok) pv(t);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------- softmax threads
    const int quad = warp & 3;
    const int kh = warp >> 2;           // key half of each tile
    const int il = quad * 32 + lane;    // row within the tile == TMEM lane
    const int i = i0 + il;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    int rlo, rhi;
    row_interval(ctx, min(i, g.q_hi - 1), g.k_lo, kend, rlo, rhi);
    const float scale_log2 = 1.4426950408889634f * rsqrtf(static_cast<float>(kDh));
    // the output is rescaled when a row maximum grows by more than 2^8
    // (log2 units), i.e. 8 / scale_log2 in raw score units
    const float rescale_raw = 8.f / scale_log2;
    const int shift = 31 - lane;
    const bool s16 = shift & 16, s8 = shift & 8, s4 = shift & 4, s2 = shift & 2, s1 = shift & 1;
    // keys every row of this warp sees: no per-element mask inside it
    const int wlo = __reduce_max_sync(0xffffffffu, rlo);
    const int whi = __reduce_min_sync(0xffffffffu, rhi);
    float* xbuf = reinterpret_cast<float*>(smem + kOffX);  // [parity][half][row] exchange
    uint32_t xphase = 0;
    float m_ref = -INFINITY;  // raw-score maximum the output is scaled by
    float l = 0.f;            // this thread's share of the row sum
    bool ok = true;
    // ---- q+u and q+v tiles (bf16 adds, attention.rs:506-508), once per CTA.
    // This thread's 64 u and v values are fetched before the wait for the Q
    // tile, so their latency overlaps the TMA.
    if (nt > 0) {
      const int tid = threadIdx.x;  // 0..255: row tid/2, 64-column half tid&1
      const int row = tid >> 1, half = tid & 1;
      float4 u4[16], v4[16];
      const float4* ug = reinterpret_cast<const float4*>(pos_u + h * kDh + half * 64);
      const float4* vg = reinterpret_cast<const float4*>(pos_v + h * kDh + half * 64);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        u4[k] = __ldg(ug + k);
        v4[k] = __ldg(vg + k);
      }
      ok = warp_wait(&bars->q, 0, err, kDevTimeoutLoad);
      if (ok) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t off = half * kHalf + sw128_offset(row, ch);
          const uint4 q = *reinterpret_cast<const uint4*>(sQu + off);
          const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
          const float uu[8] = {u4[2 * ch].x, u4[2 * ch].y, u4[2 * ch].z, u4[2 * ch].w,
                               u4[2 * ch + 1].x, u4[2 * ch + 1].y, u4[2 * ch + 1].z,
                               u4[2 * ch + 1].w};
          const float vv[8] = {v4[2 * ch].x, v4[2 * ch].y, v4[2 * ch].z, v4[2 * ch].w,
                               v4[2 * ch + 1].x, v4[2 * ch + 1].y, v4[2 * ch + 1].z,
                               v4[2 * ch + 1].w};
          uint32_t wu[4], wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[e]));
            wu[e] = pack_bf16x2(f.x + uu[2 * e], f.y + uu[2 * e + 1]);
            wv[e] = pack_bf16x2(f.x + vv[2 * e], f.y + vv[2 * e + 1]);
          }
          *reinterpret_cast<uint4*>(sQu + off) = make_uint4(wu[0], wu[1], wu[2], wu[3]);
          *reinterpret_cast<uint4*>(sQv + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        fence_proxy_async_smem();
      }
      warp_arrive(&bars->prep);
    }
    for (int t = 0; t < nt && ok; ++t) {
      const uint32_t par = t & 1;
      if (__any_sync(0xffffffffu, *abort_flag)) { ok = false; break; }
      if (!warp_wait(&bars->s, par, err, kDevTimeoutMma)) { ok = false; break; }
      tc_fence_after();
      const int jt = j0 + t * kTile;
      // ---- pass 1: 64 scores (log2 domain, masked) into registers
      float sc[64];
      float mxp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mxp[e] = -INFINITY;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        const int jl0 = 64 * kh + 32 * sub;
        const int col0 = 96 - 32 * quad + jl0;  // BD window start (chunk-pair coords)
        uint32_t sr[32], w0[32], w1[32];
        tmem_ld32(trow + jl0, sr);
        const int x0 = col0, x1 = col0 + 32;
        tmem_ld32(trow + 128 + 128 * ((t + (x0 >> 7)) & 1) + (x0 & 127), w0);
        tmem_ld32(trow + 128 + 128 * ((t + (x1 >> 7)) & 1) + (x1 & 127), w1);
        tmem_ld_wait();
        float a[64];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          a[x] = __uint_as_float(w0[x]);
          a[x + 32] = __uint_as_float(w1[x]);
        }
        // a[e] <- a[shift + e]: barrel shift by the lane's skew (selects)
#pragma unroll
        for (int x = 0; x < 47; ++x) a[x] = s16 ? a[x + 16] : a[x];
#pragma unroll
        for (int x = 0; x < 39; ++x) a[x] = s8 ? a[x + 8] : a[x];
#pragma unroll
        for (int x = 0; x < 35; ++x) a[x] = s4 ? a[x + 4] : a[x];
#pragma unroll
        for (int x = 0; x < 33; ++x) a[x] = s2 ? a[x + 2] : a[x];
#pragma unroll
        for (int x = 0; x < 32; ++x) a[x] = s1 ? a[x + 1] : a[x];
        const int jb = jt + jl0;
        // raw scores s + bd (the scale is applied inside exp2 below)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          add_f32x2(sc[32 * sub + e], sc[32 * sub + e + 1], __uint_as_float(sr[e]),
                    __uint_as_float(sr[e + 1]), a[e], a[e + 1]);
        if (!(jb >= wlo && jb + 32 <= whi)) {  // some key hidden from some row
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int j = jb + e;
            sc[32 * sub + e] = (j >= rlo && j < rhi) ? sc[32 * sub + e] : -INFINITY;
          }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) mxp[e & 7] = fmaxf(mxp[e & 7], sc[32 * sub + e]);
      }
      float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      tc_fence_before();
      warp_arrive(&bars->sfree);  // S and BD slot t&1 may be overwritten
      // ---- previous P.V done: O is stable, the probability buffer is free
      if (t > 0 && !warp_wait(&bars->o, par ^ 1, err, kDevTimeoutMma)) { ok = false; break; }
      // ---- swap row maxima with the other key half's thread; the two parity
      // buffers let one sync per tile suffice (a thread cannot write the
      // buffer of parity p again before its partner passed this sync)
      xbuf[xphase * 256 + kh * 128 + il] = mx;
      warp_arrive(&bars->x);
      if (!warp_wait(&bars->x, xphase, err, kDevTimeoutEpi)) { ok = false; break; }
      mx = fmaxf(mx, xbuf[xphase * 256 + (kh ^ 1) * 128 + il]);
      xphase ^= 1;
      float alpha = 1.f;
      if (mx > m_ref + rescale_raw) {  // also taken when m_ref is -inf and mx finite
        alpha = (m_ref == -INFINITY) ? 1.f : exp2f((m_ref - mx) * scale_log2);
        m_ref = mx;
      }
      l *= alpha;
      if (t > 0) {
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            const uint32_t col = 384 + 64 * kh + 16 * c;
            uint32_t o[16];
            tmem_ld16(trow + col, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(trow + col, o);
          }
          tmem_st_wait();
        }
      }
      // ---- pass 2: probabilities -> shared memory (bf16 A operand of P.V)
      // a row that has seen no key yet keeps m_ref = -inf: subtract 0 so
      // its -inf scores give exp2(-inf) = 0 rather than NaN
      // p = 2^((score - m) * scale): one packed FMA per pair, then MUFU
      const float nms = m_ref == -INFINITY ? 0.f : -m_ref * scale_log2;
      uint8_t* prow = sPr + kh * kHalf;
      float lp[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) lp[e] = 0.f;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x0, x1;
          fma_f32x2(x0, x1, sc[8 * ch + 2 * e], sc[8 * ch + 2 * e + 1], scale_log2, nms);
          const float p0 = fast_exp2(x0);
          const float p1 = fast_exp2(x1);
          add_f32x2(lp[2 * e], lp[2 * e + 1], lp[2 * e], lp[2 * e + 1], p0, p1);
          pk[e] = pack_bf16x2(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + sw128_offset(il, ch)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(&bars->p);
    }
    // ---- epilogue: out = O / l over both key halves
    if (ok) ok = warp_wait(&bars->o, (nt - 1) & 1, err, kDevTimeoutMma);
    float inv = 0.f;
    if (ok) {
      tc_fence_after();
      xbuf[xphase * 256 + kh * 128 + il] = l;
      warp_arrive(&bars->x);
      ok = warp_wait(&bars->x, xphase, err, kDevTimeoutEpi);
      if (ok) {
        const float lt = l + xbuf[xphase * 256 + (kh ^ 1) * 128 + il];
        inv = lt > 0.f ? 1.f / lt : 0.f;
      }
    }
    // The normalised tile goes to shared memory in the TMA layout (the q+u
    // tile's buffer: every MMA that read it completed before O did) and
    // leaves in two bulk tensor stores; rows past q_hi fall outside the
    // output map and are not written.
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t o[32];
      if (ok) {
        tmem_ld32(trow + 384 + 64 * kh + 32 * c, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0u;
      }
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pk[e] = pack_bf16x2(__uint_as_float(o[8 * v + 2 * e]) * inv,
                              __uint_as_float(o[8 * v + 2 * e + 1]) * inv);
        *reinterpret_cast<uint4*>(sQu + kh * kHalf + sw128_offset(il, 4 * c + v)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, kSoftmaxThreads);
    if (threadIdx.x == 0) {
      tma_store_3d(&map_out, sQu, h * kDh, i0 - g.out_base, b);
      tma_store_3d(&map_out, sQu + kHalf, h * kDh + 64, i0 - g.out_base, b);
      bulk_commit();
      bulk_wait_all();
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

AttnGeom full_geom(int T, int D) {
  AttnGeom g;
  g.Tg = T;
  g.tbuf = T;
  g.base = 0;
  g.qkv_ts = 3ll * D;
  g.qkv_bs = 3ll * D * T;
  g.q_lo = 0;
  g.q_hi = T;
  g.k_lo = 0;
  g.k_hi = T;
  g.p_base = 0;
  g.p_rows = 2 * T - 1;
  g.out_base = 0;
  g.out_bs = static_cast<int64_t>(T) * D;
  return g;
}

void visible_offsets(const AttnContextDev& c, int T, int& dmin, int& dmax) {
  dmin = -(T - 1);
  dmax = T - 1;
  if (!c.has) return;
  if (c.chunked && c.right >= 0) {
    // row i of chunk ci sees keys [(ci - lc) * chunk, (ci + 1) * chunk)
    const long long chunk = c.right + 1;
    const long long lc = c.left >= 0 ? c.left / chunk : 10000;
    const long long lo = -(lc * chunk + chunk - 1);
    if (lo > dmin) dmin = static_cast<int>(lo);
    dmax = static_cast<int>(chunk - 1 < dmax ? chunk - 1 : dmax);
  } else {
    if (c.left >= 0) dmin = -c.left;
    if (!c.chunked && c.right >= 0) dmax = c.right;
  }
  dmin = dmin < -(T - 1) ? -(T - 1) : dmin;
  dmax = dmax > T - 1 ? T - 1 : dmax;
  if (dmax < dmin) dmax = dmin;  // nothing visible: keep a valid 1-row window
}

cudaError_t launch_relpos_attn_bf16(const void* qkv, const void* p, const float* u,
                                    const float* v, const int32_t* key_len, AttnContextDev ctx,
                                    const AttnGeom& g, void* out, int B, int H, int* err,
                                    int num_sms, cudaStream_t stream) {
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(relpos_attn_kernel, static_cast<int>(kSmemBytes), attr))
    return e;
  const int D = H * kDh;
  if (g.q_hi <= g.q_lo || g.tbuf <= 0 || g.p_rows <= 0 || B <= 0 || B > 65535)
    return cudaErrorInvalidValue;
  if (g.q_lo < g.base || g.q_hi > g.base + g.tbuf || g.k_lo < g.base ||
      g.k_hi > g.base + g.tbuf || g.k_lo < 0 || g.k_hi > g.Tg || g.q_lo < g.out_base)
    return cudaErrorInvalidValue;
  CUtensorMap map_qkv, map_p, map_out;
  if (!make_tmap_3d(&map_qkv, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3ull * D, g.tbuf, B,
                    static_cast<uint64_t>(g.qkv_ts) * 2, static_cast<uint64_t>(g.qkv_bs) * 2, 64,
                    kTile, 1, true) ||
      !make_tmap_2d(&map_p, p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, g.p_rows,
                    static_cast<uint64_t>(D) * 2, 64, kTile, true) ||
      !make_tmap_3d(&map_out, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, g.q_hi - g.out_base,
                    B, static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(g.out_bs) * 2, 64,
                    kTile, 1, true))
    return cudaErrorInvalidValue;
  dim3 grid((g.q_hi - g.q_lo + kTile - 1) / kTile, H, B);
  relpos_attn_kernel<<<grid, kThreads, kSmemBytes, stream>>>(
      map_qkv, map_p, u, v, map_out, key_len, ctx, g, static_cast<__nv_bfloat16*>(out), H,
      num_sms > 0 ? num_sms : 148, err);
  return cudaGetLastError();
}

}  // namespace nrp
