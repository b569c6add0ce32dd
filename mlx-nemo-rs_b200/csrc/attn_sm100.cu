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
// Biases.  Each query tile is staged once and turned into two bf16 tiles,
// q+u (A operand of the content product) and q+v (A operand of the
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
// Grid.  Persistent, one CTA per SM (relpos_attn_kernel below): the work
// items (query tile, head, utterance) come from a counter the grid shares,
// so SMs stay balanced, and each item's loads and first MMAs run under the
// previous item's last tile.
//
// Softmax (warps 0-7): warp w owns TMEM lane quadrant w&3 (one query row per
// thread) and key half w>>2 (64 keys); the two threads of a row swap their
// row maxima through shared memory.  Online softmax in the log2 domain; the
// output is rescaled only when a row maximum grows by more than 2^8 (exact:
// the final normalisation uses the same maximum).  Every wait is bounded.
//
// The softmax tile loop is bound by instruction fetch as much as by its
// pipes, so code size counts: each role's per-item work is inlined once.
#include <math.h>

#include <cstring>

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
constexpr int kHelperWarps = 3;  // warps 9-11
constexpr int kThreads = kSoftmaxThreads + 32 + 32 * kHelperWarps;  // + the issuer warp

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
  uint64_t q, prep, p0, kp, v[2], s, sfree, p, o, x[4], ob, ofree, dfull[2], dempty[2];
  uint32_t tmem_base;
  int abort;
  int desc[2][8];  // item descriptors, helper -> issuer and softmax (nt < 0: done)
};
static_assert(sizeof(Bars) <= 256, "barrier block");
constexpr uint32_t kOffOrder = kOffBar + 256;  // utterances by decreasing length (u8)
constexpr size_t kSmemBytes = kOffOrder + 256;
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr uint32_t kStageTx = 2 * kTileBytes;  // K tile + P chunk
// Batches up to this size are worked longest utterance first.
constexpr int kMaxSortedBatch = 256;

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

// One work item: query tile qt of head h of utterance b, with the key
// interval [j0, j0 + 128 nt) every row of the tile may see (nt = 0: the tile
// is padding or sees no key).
struct Item {
  int b, h, i0, j0, nt, rbase, kend;
};

__device__ __forceinline__ Item make_item(int r, int X, int H, const int32_t* key_len,
                                          const AttnContextDev& ctx, const AttnGeom& g) {
  Item it;
  const int qt = r % X;
  it.h = (r / X) % H;
  it.b = r / (X * H);
  it.i0 = g.q_lo + qt * kTile;  // global frame of the tile's first row
  int klen = g.Tg;
  if (key_len) klen = min(g.Tg, max(key_len[it.b], 1));
  it.kend = min(klen, g.k_hi);
  int lo0, hi0, lo1, hi1;
  row_interval(ctx, it.i0, g.k_lo, it.kend, lo0, hi0);
  row_interval(ctx, min(it.i0 + kTile - 1, g.q_hi - 1), g.k_lo, it.kend, lo1, hi1);
  // Query tiles wholly past the utterance's length are padding: their
  // outputs are unspecified in the reference (conformer.rs:1590-1593) and
  // are written as zeros here.
  const bool padded = key_len && it.i0 >= klen;
  it.j0 = min(lo0, lo1);
  const int jhi = max(hi0, hi1);
  it.nt = (jhi > it.j0 && !padded) ? (jhi - it.j0 + kTile - 1) / kTile : 0;
  // first P row of chunk 0, as a row of the p buffer (may be negative:
  // rows outside the buffer load as zeros and only meet masked pairs)
  it.rbase = g.Tg - kTile - it.i0 + it.j0 - g.p_base;
  return it;
}

// The last CTA to finish resets the grid's item counter for the next launch.
__device__ __forceinline__ void release_sched(int* sched) {
  __threadfence();
  if (atomicAdd(sched + 1, 1) == static_cast<int>(gridDim.x) - 1) {
    atomicExch(sched, 0);
    atomicExch(sched + 1, 0);
  }
}

// Persistent: one CTA per SM, four roles.
//   helpers (warps 9-11) warp 9 takes a CTA's first item by its block
//           index and the rest from a counter shared by the grid (sched[0]:
//           items from gridDim.x on; the last CTA to finish resets sched[0..1]), in
//           order of decreasing utterance length, writes padding tiles as
//           zeros and hands each item with keys to the other roles through a
//           two-slot descriptor ring; the three build the item's q+u/q+v
//           tiles once the issuer has loaded its Q tile.
//   issuer  (warp 8, one thread) TMA loads and MMAs.
//   softmax (warps 0-7) the scores, probabilities and the epilogue.
// Barrier phases run on per-CTA counters: gt over the CTA's key tiles, ic
// over its items, dc over descriptors.  Item k's prologue hides under item
// k-1's last tile: after item k-1's last S/BD MMAs the issuer loads Q_k,
// {K_0, P_1} and P chunk 0 (into the free V slot of item k's first tile),
// issues item k-1's last P.V, and issues BD_0, S_0, BD_1 once the helper has
// built the q+u/q+v tiles; the softmax warps meanwhile finish item k-1 and
// write its output.  Item k-1's output is staged in the V slot of its last
// tile; item k's V_1 goes to that slot after the bulk store has read it
// (ofree).
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_kernel(const __grid_constant__ CUtensorMap map_qkv,  // [B][tbuf][3D] bf16
                       const __grid_constant__ CUtensorMap map_p,    // [p_rows][D] bf16
                       const __grid_constant__ AttnUV uv,            // q biases, bf16 pairs
                       const __grid_constant__ CUtensorMap map_out,  // [B][rows][D] bf16
                       const int32_t* __restrict__ key_len, AttnContextDev ctx, AttnGeom g,
                       __nv_bfloat16* __restrict__ out, int B, int H, int* err, int* sched) {
  // Dynamic shared memory starts 1024-byte aligned when, as here, the kernel
  // has no static shared memory; checked, since the swizzle atoms need it.
  extern __shared__ __align__(1024) uint8_t smem[];
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) {
      atomicCAS(err, 0, kDevBadArgs);
      release_sched(sched);
    }
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
  const int D = H * kDh;
  const int X = (g.q_hi - g.q_lo + kTile - 1) / kTile;  // query tiles per utterance
  const int n_items = X * H * B;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q, 1);
    mbar_init(&bars->prep, kHelperWarps);
    mbar_init(&bars->p0, 1);
    mbar_init(&bars->kp, 1);
    mbar_init(&bars->v[0], 1);
    mbar_init(&bars->v[1], 1);
    mbar_init(&bars->s, 1);
    mbar_init(&bars->sfree, kSoftmaxWarps);
    mbar_init(&bars->p, kSoftmaxWarps);
    mbar_init(&bars->o, 1);
    for (int k = 0; k < 4; ++k) mbar_init(&bars->x[k], 2);  // the two warps of a quadrant
    mbar_init(&bars->ob, kSoftmaxWarps);
    mbar_init(&bars->ofree, 1);
    mbar_init(&bars->dfull[0], 1);
    mbar_init(&bars->dfull[1], 1);
    // read by the issuer, the softmax warps and the helpers
    mbar_init(&bars->dempty[0], 1 + kSoftmaxWarps + kHelperWarps);
    mbar_init(&bars->dempty[1], 1 + kSoftmaxWarps + kHelperWarps);
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
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 8) {
    // ------------------------------------------------ TMA + MMA issuer
    if (lane == 0) {
      prefetch_tensormap(&map_qkv);
      prefetch_tensormap(&map_p);
      prefetch_tensormap(&map_out);
      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t aQu = smem_u32(sQu), aQv = smem_u32(sQv), aK = smem_u32(sK);
      const uint32_t aV = smem_u32(sV), aP = smem_u32(sP), aPr = smem_u32(sPr);
      auto pv = [&](uint32_t gi, bool acc) {  // O (+)= probabilities . V of tile gi
        tc_fence_after();
        const uint32_t vb = aV + (gi & 1) * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t offa = (k >> 2) * kHalf + (k & 3) * 32;
          umma_ss(tmem + 384, sdesc_sw128(aPr + offa, 16, 1024),
                  sdesc_sw128(vb + k * 2048, kHalf, 1024), idesc_pv, acc || (k > 0));
        }
        umma_commit(&bars->o);
      };
      uint32_t gt = 0, ic = 0, dc = 0;
      bool pending = false, acc_last = false;  // the previous item's last P.V
      uint32_t g_last = 0;
      bool ok = true;
      while (ok) {
        Item it;
        ok = mbar_wait(&bars->dfull[dc & 1], (dc >> 1) & 1, err, kDevTimeoutEpi);
        if (!ok) break;
        {
          const volatile int* d = bars->desc[dc & 1];
          it.b = d[0];
          it.h = d[1];
          it.i0 = d[2];
          it.j0 = d[3];
          it.nt = d[4];
          it.rbase = d[5];
          mbar_arrive(&bars->dempty[dc & 1]);
          ++dc;
        }
        const int kcol = D + it.h * kDh, vcol = 2 * D + it.h * kDh;
        auto load_stage = [&](int t) {  // K_t and P chunk t+1
          mbar_arrive_expect_tx(&bars->kp, kStageTx);
          const int jt = it.j0 + t * kTile - g.base;
          tma_load_3d(sK, &map_qkv, &bars->kp, kcol, jt, it.b);
          tma_load_3d(sK + kHalf, &map_qkv, &bars->kp, kcol + 64, jt, it.b);
          const int prow = it.rbase + (t + 1) * kTile;
          tma_load_2d(sP, &map_p, &bars->kp, it.h * kDh, prow);
          tma_load_2d(sP + kHalf, &map_p, &bars->kp, it.h * kDh + 64, prow);
        };
        auto load_v = [&](int t, uint32_t gi) {  // V_t into the slot of tile gi
          uint64_t* bar = &bars->v[gi & 1];
          uint8_t* dst = sV + (gi & 1) * kTileBytes;
          mbar_arrive_expect_tx(bar, kTileBytes);
          tma_load_3d(dst, &map_qkv, bar, vcol, it.j0 + t * kTile - g.base, it.b);
          tma_load_3d(dst + kHalf, &map_qkv, bar, vcol + 64, it.j0 + t * kTile - g.base, it.b);
        };
        // P chunk 0 is only read by the first BD MMA: staged in the V slot of
        // the item's first tile (its last reader, tile gt-2, has completed:
        // the s commit waited for item k-1 covers every earlier MMA), where
        // V_0 follows once BD_0 has completed
        uint8_t* p0buf = sV + (gt & 1) * kTileBytes;
        if (it.nt > 0) {
          // Q and the first {K, P} stage: every MMA of the previous item that
          // read those buffers has completed (its s was waited below)
          mbar_arrive_expect_tx(&bars->q, kTileBytes);
          tma_load_3d(sQu, &map_qkv, &bars->q, it.h * kDh, it.i0 - g.base, it.b);
          tma_load_3d(sQu + kHalf, &map_qkv, &bars->q, it.h * kDh + 64, it.i0 - g.base, it.b);
          load_stage(0);
          mbar_arrive_expect_tx(&bars->p0, kTileBytes);
          tma_load_2d(p0buf, &map_p, &bars->p0, it.h * kDh, it.rbase);
          tma_load_2d(p0buf + kHalf, &map_p, &bars->p0, it.h * kDh + 64, it.rbase);
        }
        if (pending) {  // the previous item's last P.V (also after the last item)
          ok = mbar_wait(&bars->p, g_last & 1, err, kDevTimeoutEpi) &&
               mbar_wait(&bars->v[g_last & 1], (g_last >> 1) & 1, err, kDevTimeoutLoad);
          if (!ok) break;
          pv(g_last, acc_last);
          pending = false;
        }
        if (it.nt < 0) break;
        // BD_0 once the q+u / q+v tiles are ready and the previous item's
        // last pass 1 released the S and BD columns
        ok = mbar_wait(&bars->prep, ic & 1, err, kDevTimeoutEpi) &&
             mbar_wait(&bars->p0, ic & 1, err, kDevTimeoutLoad);
        if (ok && ic > 0) ok = mbar_wait(&bars->sfree, g_last & 1, err, kDevTimeoutEpi);
        if (!ok) break;
        tc_fence_after();
        mma_k128(tmem + 128, aQv, smem_u32(p0buf), idesc_kk, false);  // BD_0 -> slot 0
        for (int t = 0; t < it.nt && ok; ++t) {
          const uint32_t gi = gt + t;
          ok = mbar_wait(&bars->kp, gi & 1, err, kDevTimeoutLoad);
          if (ok && t > 0) ok = mbar_wait(&bars->sfree, (gi - 1) & 1, err, kDevTimeoutEpi);
          if (!ok) break;
          tc_fence_after();
          mma_k128(tmem, aQu, aK, idesc_kk, false);  // S_t
          mma_k128(tmem + 128 + 128 * ((t + 1) & 1), aQv, aP, idesc_kk, false);  // BD_{t+1}
          umma_commit(&bars->s);
          // the stage (and, for t = 0, P chunk 0) is free once these MMAs
          // have read it
          ok = mbar_wait(&bars->s, gi & 1, err, kDevTimeoutMma);
          if (!ok) break;
          if (t + 1 < it.nt) load_stage(t + 1);
          if (t == 0) {
            load_v(0, gi);
            // The previous item's output is staged in the other V slot until
            // its bulk store has read it.  Waiting here for every item (not
            // only before V_1 goes there) also covers the next item's P
            // chunk 0, which lands in that slot when this item's tile count
            // is odd.
            if (ic > 0) ok = mbar_wait(&bars->ofree, (ic - 1) & 1, err, kDevTimeoutEpi);
            if (!ok) break;
            if (it.nt > 1) load_v(1, gi + 1);
          }
          if (t > 0) {  // P.V of the previous tile, then V for tile t+1 into its slot
            ok = mbar_wait(&bars->p, (gi - 1) & 1, err, kDevTimeoutEpi) &&
                 mbar_wait(&bars->v[(gi - 1) & 1], ((gi - 1) >> 1) & 1, err, kDevTimeoutLoad);
            if (!ok) break;
            pv(gi - 1, t > 1);
            ok = mbar_wait(&bars->o, (gi - 1) & 1, err, kDevTimeoutMma);
            if (!ok) break;
            if (t + 1 < it.nt) load_v(t + 1, gi + 1);
          }
        }
        if (!ok) break;
        pending = true;
        g_last = gt + it.nt - 1;
        acc_last = it.nt > 1;
        gt += it.nt;
        ++ic;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 9) {
    // ------------------------------------------------ helpers
    // ---- q+u and q+v tiles of head h (bf16 adds, attention.rs:506-508),
    // once the issuer has loaded the item's Q tile (every MMA of the
    // previous item that read the q+v buffer completed before that load was
    // issued).  The three helper warps share the 128 x 2 (row, 64-column
    // half) units; a thread keeps one half, so its 32 u and 32 v pairs (the
    // kernel parameters) are loaded once.
    auto build_q_tiles = [&](int h) {
      const int t3 = (warp - 9) * 32 + lane;
      const int half = t3 & 1;
      const uint32_t* uh = uv.w + h * 128 + half * 32;
      uint32_t uw[32], vw[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        uw[k] = uh[k];
        vw[k] = uh[64 + k];
      }
#pragma unroll 1
      for (int row = t3 >> 1; row < kTile; row += 16 * kHelperWarps) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t off = half * kHalf + sw128_offset(row, ch);
          const uint4 q = *reinterpret_cast<const uint4*>(sQu + off);
          *reinterpret_cast<uint4*>(sQu + off) =
              make_uint4(add_bf16x2(q.x, uw[4 * ch]), add_bf16x2(q.y, uw[4 * ch + 1]),
                         add_bf16x2(q.z, uw[4 * ch + 2]), add_bf16x2(q.w, uw[4 * ch + 3]));
          *reinterpret_cast<uint4*>(sQv + off) =
              make_uint4(add_bf16x2(q.x, vw[4 * ch]), add_bf16x2(q.y, vw[4 * ch + 1]),
                         add_bf16x2(q.z, vw[4 * ch + 2]), add_bf16x2(q.w, vw[4 * ch + 3]));
        }
      }
      fence_proxy_async_smem();
    };
    // ---- warp 9 is the scheduler.  Utterances by decreasing length (ties
    // by index): the warp ranks them from one load of the lengths.
    uint8_t* order = smem + kOffOrder;
    const bool sorted = key_len && B <= kMaxSortedBatch;
    if (warp == 9 && sorted) {
      constexpr int kPer = kMaxSortedBatch / 32;
      int len[kPer], rank[kPer];
#pragma unroll
      for (int m = 0; m < kPer; ++m) {
        const int t = lane + 32 * m;
        len[m] = t < B ? key_len[t] : 0;
        rank[m] = 0;
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        if (32 * k >= B) break;
        const int n = min(32, B - 32 * k);
        for (int j = 0; j < n; ++j) {
          const int lu = __shfl_sync(0xffffffffu, len[k], j);
          const int u = 32 * k + j;
#pragma unroll
          for (int m = 0; m < kPer; ++m) {
            const int t = lane + 32 * m;
            rank[m] += (lu > len[m]) || (lu == len[m] && u < t);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < kPer; ++m) {
        const int t = lane + 32 * m;
        if (t < B) order[rank[m]] = static_cast<uint8_t>(t);  // ranks are a permutation
      }
    }
    __syncwarp();
    uint32_t pc = 0, ic = 0, dc = 0;
    bool ok = true;
    const int per_b = X * H;
    bool first = true;  // a CTA's first item is its block index; then the counter
    while (true) {
      if (warp == 9) {
        // the next item with keys; padding tiles are written as zeros here
        Item it;
        while (true) {
          int qn = static_cast<int>(blockIdx.x);
          if (!first) {
            if (lane == 0) qn = atomicAdd(sched, 1) + static_cast<int>(gridDim.x);
            qn = __shfl_sync(0xffffffffu, qn, 0);
          }
          first = false;
          if (qn >= n_items || !ok) {
            it.nt = -1;
            break;
          }
          const int ub = qn / per_b, rem = qn - ub * per_b;
          it = make_item((sorted ? order[ub] : ub) * per_b + rem, X, H, key_len, ctx, g);
          if (it.nt > 0) break;
          const int rows = min(kTile, g.q_hi - it.i0);
          __nv_bfloat16* ob = out + static_cast<size_t>(it.b) * g.out_bs + it.h * kDh;
          for (int k = lane; k < rows * 16; k += 32) {
            const int rr = k >> 4, c = k & 15;
            *reinterpret_cast<uint4*>(ob + static_cast<size_t>(it.i0 + rr - g.out_base) * D +
                                      c * 8) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        if (__any_sync(0xffffffffu, *abort_flag)) {
          ok = false;
          it.nt = -1;
        }
        // publish; the slot is free once the issuer and the softmax warps have
        // read the item two back
        const uint32_t slot = pc & 1;
        if (pc >= 2 && !warp_wait(&bars->dempty[slot], ((pc >> 1) - 1) & 1, err, kDevTimeoutEpi)) {
          ok = false;
          it.nt = -1;
        }
        if (lane == 0) {
          int* d = bars->desc[slot];
          d[0] = it.b;
          d[1] = it.h;
          d[2] = it.i0;
          d[3] = it.j0;
          d[4] = it.nt;
          d[5] = it.rbase;
          d[6] = it.kend;
          mbar_arrive(&bars->dfull[slot]);
          if (it.nt > 0)  // its first Q, K and V tiles into L2
            for (int half = 0; half < 2; ++half) {
              tma_prefetch_3d(&map_qkv, it.h * kDh + 64 * half, it.i0 - g.base, it.b);
              tma_prefetch_3d(&map_qkv, D + it.h * kDh + 64 * half, it.j0 - g.base, it.b);
              tma_prefetch_3d(&map_qkv, 2 * D + it.h * kDh + 64 * half, it.j0 - g.base, it.b);
            }
        }
        ++pc;
      }
      // ---- every helper: the next item from the ring, then its share of
      // the item's q+u/q+v tiles
      if (!warp_wait(&bars->dfull[dc & 1], (dc >> 1) & 1, err, kDevTimeoutEpi)) break;
      const int h = bars->desc[dc & 1][1], nt = bars->desc[dc & 1][4];
      warp_arrive(&bars->dempty[dc & 1]);
      ++dc;
      if (nt < 0) break;
      ok = warp_wait(&bars->q, ic & 1, err, kDevTimeoutLoad);
      if (ok) build_q_tiles(h);
      warp_arrive(&bars->prep);
      ++ic;
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
  } else {
    // ------------------------------------------------- softmax threads
    const int tid = threadIdx.x;        // 0..255
    const int quad = warp & 3;
    const int kh = warp >> 2;           // key half of each tile
    const int il = quad * 32 + lane;    // row within the tile == TMEM lane
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float scale_log2 = 1.4426950408889634f * rsqrtf(static_cast<float>(kDh));
    // the output is rescaled when a row maximum grows by more than 2^8
    // (log2 units), i.e. 8 / scale_log2 in raw score units
    const float rescale_raw = 8.f / scale_log2;
    const int shift = 31 - lane;
    // the shift's stages are selects (a selection on the FMA pipe, b*f +
    // a*(1-f), measured slower: the loop is instruction-fetch bound, and it
    // doubles the instructions of a stage)
    const bool s16 = shift & 16, s8 = shift & 8, s4 = shift & 4, s2 = shift & 2, s1 = shift & 1;
    float* xbuf = reinterpret_cast<float*>(smem + kOffX);  // [parity][half][row] exchange
    uint32_t xphase = 0, gt = 0, ic = 0, ec = 0, dc = 0;
    bool ok = true;
    // the previous item, whose epilogue runs once the next item's q+u/q+v
    // tiles are done
    bool pending = false;
    int pb = 0, ph = 0, pi0 = 0;
    uint32_t pg_last = 0;
    float pl = 0.f;
    auto epilogue = [&]() {  // out = O / l over both key halves
      ok = warp_wait(&bars->o, pg_last & 1, err, kDevTimeoutMma);
      float inv = 0.f;
      if (ok) {
        tc_fence_after();
        xbuf[xphase * 256 + kh * 128 + il] = pl;
        warp_arrive(&bars->x[quad]);
        ok = warp_wait(&bars->x[quad], xphase, err, kDevTimeoutEpi);
        if (ok) {
          const float lt = pl + xbuf[xphase * 256 + (kh ^ 1) * 128 + il];
          inv = lt > 0.f ? 1.f / lt : 0.f;
        }
        xphase ^= 1;
      }
      // The normalised tile goes to shared memory in the TMA layout (the V
      // slot of the item's last tile: its P.V completed with O) and leaves
      // in two bulk tensor stores; rows past q_hi fall outside the output
      // map and are not written.
      uint8_t* stage = sV + (pg_last & 1) * kTileBytes;
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
          *reinterpret_cast<uint4*>(stage + kh * kHalf + sw128_offset(il, 4 * c + v)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(&bars->ob);
      if (tid == 0) {
        if (mbar_wait(&bars->ob, ec & 1, err, kDevTimeoutEpi)) {
          tma_store_3d(&map_out, stage, ph * kDh, pi0 - g.out_base, pb);
          tma_store_3d(&map_out, stage + kHalf, ph * kDh + 64, pi0 - g.out_base, pb);
          bulk_commit();
          bulk_wait_read<0>();
        } else {
          ok = false;
        }
        mbar_arrive(&bars->ofree);  // the issuer may load into the slot again
      }
      if (warp == 0) ok = __all_sync(0xffffffffu, ok);  // lane 0 may have failed the wait
      ++ec;
    };
    while (ok) {
      if (!warp_wait(&bars->dfull[dc & 1], (dc >> 1) & 1, err, kDevTimeoutEpi)) {
        ok = false;
        break;
      }
      Item it;
      {
        const volatile int* d = bars->desc[dc & 1];
        it.b = d[0];
        it.h = d[1];
        it.i0 = d[2];
        it.j0 = d[3];
        it.nt = d[4];
        it.kend = d[6];
        warp_arrive(&bars->dempty[dc & 1]);
        ++dc;
      }
      if (pending) {  // the previous item's output (also after the last item)
        epilogue();
        pending = false;
        if (!ok) break;
      }
      if (it.nt < 0) break;
      if (__any_sync(0xffffffffu, *abort_flag)) { ok = false; break; }
      // ---- the item's key tiles
      const int i = it.i0 + il;
      int rlo, rhi;
      row_interval(ctx, min(i, g.q_hi - 1), g.k_lo, it.kend, rlo, rhi);
      // keys every row of this warp sees: no per-element mask inside it
      const int wlo = __reduce_max_sync(0xffffffffu, rlo);
      const int whi = __reduce_min_sync(0xffffffffu, rhi);
      float m_ref = -INFINITY;  // raw-score maximum the output is scaled by
      float l = 0.f;            // this thread's share of the row sum
      for (int t = 0; t < it.nt && ok; ++t) {
        const uint32_t gi = gt + t;
        const uint32_t par = gi & 1;
        if (__any_sync(0xffffffffu, *abort_flag)) { ok = false; break; }
        if (!warp_wait(&bars->s, par, err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const int jt = it.j0 + t * kTile;
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
          // a[e] <- a[shift + e]: barrel shift by the lane's skew
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
        warp_arrive(&bars->x[quad]);
        if (!warp_wait(&bars->x[quad], xphase, err, kDevTimeoutEpi)) { ok = false; break; }
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
      if (!ok) break;
      pending = true;
      pb = it.b;
      ph = it.h;
      pi0 = it.i0;
      pg_last = gt + it.nt - 1;
      pl = l;
      gt += it.nt;
      ++ic;
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) release_sched(sched);
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

cudaError_t launch_relpos_attn_bf16(const void* qkv, const void* p, const uint32_t* uv_host,
                                    const int32_t* key_len, AttnContextDev ctx,
                                    const AttnGeom& g, void* out, int B, int H, int* err,
                                    int* sched, int num_sms, cudaStream_t stream) {
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(relpos_attn_kernel, static_cast<int>(kSmemBytes), attr))
    return e;
  const int D = H * kDh;
  if (g.q_hi <= g.q_lo || g.tbuf <= 0 || g.p_rows <= 0 || B <= 0 || H <= 0 ||
      H > kMaxHeadsUV || !uv_host || !sched)
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
  AttnUV uv;
  std::memcpy(uv.w, uv_host, sizeof(uint32_t) * 128 * H);
  const int64_t n_items = static_cast<int64_t>((g.q_hi - g.q_lo + kTile - 1) / kTile) * H * B;
  if (n_items > INT32_MAX) return cudaErrorInvalidValue;
  const int sms = num_sms > 0 ? num_sms : 148;
  const int grid = static_cast<int>(n_items < sms ? n_items : sms);  // one CTA per SM
  return launch_pdl(relpos_attn_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, map_qkv,
                    map_p, uv, map_out, key_len, ctx, g, static_cast<__nv_bfloat16*>(out), B, H,
                    err, sched);
}

}  // namespace nrp
