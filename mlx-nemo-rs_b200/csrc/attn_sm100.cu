// attn_sm100.cu -- fused offline relative-position attention on tcgen05.
//
// Computes, per (batch b, head h, 128-query tile), what the reference's
// RelPositionMultiHeadAttention::forward_blocked does between the
// projections (src/asr/modules/encoders/attention.rs:501-556):
//
//   S[i,j]  = ((q_i + u) . k_j + rel_shift((q + v) . P^T)[i,j]) / sqrt(dh)
//   out_i   = softmax_j(S[i,j] + mask) . V
//
// without materialising the [rows, 2T-1] positional score matrix.  rel_shift
// leaves column j of row i holding P row r = T-1-i+j (attention.rs:1248-1282),
// so for a 128x128 (query, key) tile starting at (i0, j0) the positional
// term needs the 255 consecutive P rows starting at T-128-i0+j0.  The kernel
// computes Q . P_window^T (128 x 256) with two N=128 MMAs and, per row,
// reads the 128 columns starting at 127-il (il = row within the tile): a
// per-lane skew done in registers with a 5-stage predicated barrel shift.
// The u/v bias terms are split off as per-key (u.k_j) and per-position
// (v.p_r) scalars computed from the staged tiles, so one Q tile serves both
// products.  Masks (key padding, AttentionContext windows) reduce to one
// visible key interval per query row.
//
// Memory: Q/K/V tiles and a 2-slot ring of 128-row P chunks staged by TMA
// (128B swizzle), probabilities written back to shared memory as the bf16 A
// operand of the P.V MMA.  TMEM: scores [0,128), positional window
// [128,384), output accumulator [384,512).  Online softmax in the log2
// domain; the output is rescaled only when a row's running maximum grows
// by more than 2^8 (exact: the final normalisation uses the same maximum).
//
// Warps 0-3: one query row per thread (TMEM lane = row).  Warp 4: TMEM
// owner; its lane 0 issues every TMA load and MMA.
#include <math.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kDh = 128;
constexpr int kTile = 128;
constexpr uint32_t kHalf = kTile * 64 * 2;   // 16 KB: 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kHalf;   // 32 KB: 128 rows x 128 bf16
constexpr int kThreads = 160;

struct AttnSmem {
  uint64_t bar_q, bar_kp, bar_v, bar_bias, bar_s, bar_sfree, bar_p, bar_o, bar_sync;
  uint32_t tmem_base;
  int abort;
  float kb[2][kTile];     // u . k_j for the keys of tile t (slot t & 1)
  float pb[3][kTile];     // v . p_r for P chunk c (slot c % 3)
  float u[kDh];
  float v[kDh];
};

// smem: Q | K | V | P slot 0 | P slot 1 | probabilities | AttnSmem
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + kTileBytes;
constexpr uint32_t kOffP = kOffV + kTileBytes;
constexpr uint32_t kOffPr = kOffP + 2 * kTileBytes;
constexpr uint32_t kOffMeta = kOffPr + kTileBytes;
constexpr size_t kSmemBytes = 1024 + kOffMeta + sizeof(AttnSmem);

// Bounded wait whose outcome is the same for every lane of the warp (the
// tcgen05 loads/stores that follow are warp-collective).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const bool mine = mbar_wait(bar, parity, err, code);
  return __all_sync(0xffffffffu, mine);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// dot of a 128-element bf16 row of a [128 x 128] K-major SW128 tile (two
// 64-column halves) with a float vector in shared memory.
__device__ __forceinline__ float row_dot(const uint8_t* tile, int row, const float* vec) {
  float acc = 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const uint4 q = *reinterpret_cast<const uint4*>(tile + half * kHalf + sw128_offset(row, ch));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
        const float2 f = __bfloat1622float2(b2);
        const int col = half * 64 + ch * 8 + 2 * e;
        acc = fmaf(f.x, vec[col], acc);
        acc = fmaf(f.y, vec[col + 1], acc);
      }
    }
  }
  return acc;
}

// Visible key interval [lo, hi) of query row i (AttentionContext::block_mask,
// attention.rs:232-272, intersected with key_padding_mask, 280-294).
__device__ __forceinline__ void row_interval(const AttnContextDev& c, int i, int kend, int& lo,
                                             int& hi) {
  lo = 0;
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

__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_kernel(const __grid_constant__ CUtensorMap map_qkv,  // [B][T][3D] bf16
                       const __grid_constant__ CUtensorMap map_p,    // [2T-1][D] bf16
                       const float* __restrict__ pos_u, const float* __restrict__ pos_v,
                       const int32_t* __restrict__ key_len, AttnContextDev ctx,
                       __nv_bfloat16* __restrict__ out, int T, int H, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = base + kOffQ;
  uint8_t* sK = base + kOffK;
  uint8_t* sV = base + kOffV;
  uint8_t* sP = base + kOffP;
  uint8_t* sPr = base + kOffPr;
  AttnSmem* ss = reinterpret_cast<AttnSmem*>(base + kOffMeta);

  const int warp = warp_id();
  const int lane = lane_id();
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int D = H * kDh;
  const int i0 = qt * kTile;

  // Keys visible to any row of this tile: one interval [jlo, jhi).
  int kend = T;
  if (key_len) kend = min(T, max(key_len[b], 1));
  int jlo, jhi;
  {
    int lo0, hi0, lo1, hi1;
    const int i1 = min(i0 + kTile - 1, T - 1);
    row_interval(ctx, i0, kend, lo0, hi0);
    row_interval(ctx, i1, kend, lo1, hi1);
    jlo = max(0, min(lo0, lo1));
    jhi = min(kend, max(hi0, hi1));
  }
  // Query tiles wholly past the utterance's length are padding: their
  // outputs are unspecified in the reference (conformer.rs:1590-1593) and
  // are written as zeros here.
  const bool padded_tile = key_len && i0 >= kend;
  const int nt = (jhi > jlo && !padded_tile) ? (jhi - jlo + kTile - 1) / kTile : 0;
  const int j0 = jlo;
  const int rbase = T - kTile - i0 + j0;  // first P row of chunk 0

  if (threadIdx.x == 0) {
    mbar_init(&ss->bar_q, 1);
    mbar_init(&ss->bar_kp, 1);
    mbar_init(&ss->bar_v, 1);
    mbar_init(&ss->bar_bias, 128);
    mbar_init(&ss->bar_s, 1);
    mbar_init(&ss->bar_sfree, 128);
    mbar_init(&ss->bar_p, 128);
    mbar_init(&ss->bar_o, 1);
    mbar_init(&ss->bar_sync, 128);
    ss->abort = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kDh) {
    ss->u[threadIdx.x] = pos_u[h * kDh + threadIdx.x];
    ss->v[threadIdx.x] = pos_v[h * kDh + threadIdx.x];
  }
  if (warp == 4) {
    tmem_alloc(&ss->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ss->tmem_base;
  volatile int* abort_flag = &ss->abort;

  if (warp == 4) {
    // ------------------------------------------------ TMA + MMA issuer
    if (lane == 0 && nt > 0) {
      const int qcol = h * kDh, kcol = D + h * kDh, vcol = 2 * D + h * kDh;
      prefetch_tensormap(&map_qkv);
      prefetch_tensormap(&map_p);
      mbar_arrive_expect_tx(&ss->bar_q, kTileBytes);
      tma_load_3d(sQ, &map_qkv, &ss->bar_q, qcol, i0, b);
      tma_load_3d(sQ + kHalf, &map_qkv, &ss->bar_q, qcol + 64, i0, b);
      mbar_arrive_expect_tx(&ss->bar_kp, 3 * kTileBytes);
      tma_load_3d(sK, &map_qkv, &ss->bar_kp, kcol, j0, b);
      tma_load_3d(sK + kHalf, &map_qkv, &ss->bar_kp, kcol + 64, j0, b);
      for (int c = 0; c < 2; ++c) {
        uint8_t* dst = sP + c * kTileBytes;
        tma_load_2d(dst, &map_p, &ss->bar_kp, h * kDh, rbase + c * kTile);
        tma_load_2d(dst + kHalf, &map_p, &ss->bar_kp, h * kDh + 64, rbase + c * kTile);
      }
      mbar_arrive_expect_tx(&ss->bar_v, kTileBytes);
      tma_load_3d(sV, &map_qkv, &ss->bar_v, vcol, j0, b);
      tma_load_3d(sV + kHalf, &map_qkv, &ss->bar_v, vcol + 64, j0, b);

      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);
      const uint32_t aP = smem_u32(sP), aPr = smem_u32(sPr);
      bool ok = mbar_wait(&ss->bar_q, 0, err, kDevTimeoutLoad);
      for (int t = 0; t < nt && ok; ++t) {
        const uint32_t par = t & 1;
        ok = mbar_wait(&ss->bar_kp, par, err, kDevTimeoutLoad);
        if (ok && t > 0) ok = mbar_wait(&ss->bar_sfree, par ^ 1, err, kDevTimeoutEpi);
        if (!ok) break;
        tc_fence_after();
        // S = Q . K^T  -> TMEM [0, 128)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
          umma_ss(tmem, sdesc_sw128(aQ + off, 16, 1024), sdesc_sw128(aK + off, 16, 1024),
                  idesc_kk, k > 0);
        }
        // BD = Q . [P chunk t ; P chunk t+1]^T -> TMEM [128, 384)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t pslot = aP + ((t + half) & 1) * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
            umma_ss(tmem + 128 + 128 * half, sdesc_sw128(aQ + off, 16, 1024),
                    sdesc_sw128(pslot + off, 16, 1024), idesc_kk, k > 0);
          }
        }
        umma_commit(&ss->bar_s);
        ok = mbar_wait(&ss->bar_s, par, err, kDevTimeoutMma) &&
             mbar_wait(&ss->bar_bias, par, err, kDevTimeoutEpi);
        if (!ok) break;
        if (t + 1 < nt) {
          // K tile t+1 and P chunk t+2 (into the slot chunk t used)
          const int jn = j0 + (t + 1) * kTile;
          mbar_arrive_expect_tx(&ss->bar_kp, 2 * kTileBytes);
          tma_load_3d(sK, &map_qkv, &ss->bar_kp, kcol, jn, b);
          tma_load_3d(sK + kHalf, &map_qkv, &ss->bar_kp, kcol + 64, jn, b);
          uint8_t* dst = sP + (t & 1) * kTileBytes;
          const int prow = rbase + (t + 2) * kTile;
          tma_load_2d(dst, &map_p, &ss->bar_kp, h * kDh, prow);
          tma_load_2d(dst + kHalf, &map_p, &ss->bar_kp, h * kDh + 64, prow);
        }
        ok = mbar_wait(&ss->bar_p, par, err, kDevTimeoutEpi) &&
             mbar_wait(&ss->bar_v, par, err, kDevTimeoutLoad);
        if (!ok) break;
        tc_fence_after();
        // O += probabilities . V -> TMEM [384, 512); V is MN-major (dh contiguous)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t offa = (k >> 2) * kHalf + (k & 3) * 32;
          umma_ss(tmem + 384, sdesc_sw128(aPr + offa, 16, 1024),
                  sdesc_sw128(aV + k * 2048, kHalf, 1024), idesc_pv, (t > 0) || (k > 0));
        }
        umma_commit(&ss->bar_o);
        ok = mbar_wait(&ss->bar_o, par, err, kDevTimeoutMma);
        if (!ok) break;
        if (t + 1 < nt) {
          const int jn = j0 + (t + 1) * kTile;
          mbar_arrive_expect_tx(&ss->bar_v, kTileBytes);
          tma_load_3d(sV, &map_qkv, &ss->bar_v, vcol, jn, b);
          tma_load_3d(sV + kHalf, &map_qkv, &ss->bar_v, vcol + 64, jn, b);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------- softmax threads
    const int il = warp * 32 + lane;  // row within the tile == TMEM lane
    const int i = i0 + il;
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    int rlo, rhi;
    row_interval(ctx, min(i, T - 1), kend, rlo, rhi);
    const float scale_log2 = 1.4426950408889634f * rsqrtf(static_cast<float>(kDh));
    const int shift = 31 - lane;
    float m_ref = -INFINITY;  // log2-domain running maximum the output is scaled by
    float l = 0.f;
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      const uint32_t par = t & 1;
      if (__any_sync(0xffffffffu, *abort_flag)) { ok = false; break; }
      if (!warp_wait(&ss->bar_kp, par, err, kDevTimeoutLoad)) { ok = false; break; }
      // Per-key and per-position bias scalars.  kb is double-buffered and pb
      // is a 3-slot ring, so a warp one tile ahead never overwrites what a
      // slower warp still reads; bar_sync keeps warps within one tile.
      ss->kb[t & 1][il] = row_dot(sK, il, ss->u);
      if (t == 0) ss->pb[0][il] = row_dot(sP, il, ss->v);
      ss->pb[(t + 1) % 3][il] = row_dot(sP + ((t + 1) & 1) * kTileBytes, il, ss->v);
      mbar_arrive(&ss->bar_bias);
      mbar_arrive(&ss->bar_sync);
      if (!warp_wait(&ss->bar_sync, par, err, kDevTimeoutEpi)) { ok = false; break; }
      if (!warp_wait(&ss->bar_s, par, err, kDevTimeoutMma)) { ok = false; break; }
      tc_fence_after();
      const int jt = j0 + t * kTile;
      const float* kbt = ss->kb[t & 1];
      // ---- pass 1: scores (log2 domain, masked) back into TMEM [0,128)
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32], w0[32], w1[32];
        const int col0 = 96 - 32 * warp + 32 * c;
        tmem_ld32(trow + 32 * c, sr);
        tmem_ld32(trow + 128 + col0, w0);
        tmem_ld32(trow + 128 + col0 + 32, w1);
        tmem_ld_wait();
        float a[64];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          a[x] = __uint_as_float(w0[x]);
          a[x + 32] = __uint_as_float(w1[x]);
        }
        // out[e] = a[shift + e]: barrel shift by the lane's skew (selects)
        {
          const bool s16 = shift & 16, s8 = shift & 8, s4 = shift & 4, s2 = shift & 2,
                     s1 = shift & 1;
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
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int jl = 32 * c + e;
          const int j = jt + jl;
          const int x = 127 - il + jl;  // P row within the 256-row window
          const float pbv = ss->pb[(t + (x >> 7)) % 3][x & 127];
          float sc = (__uint_as_float(sr[e]) + kbt[jl] + a[e] + pbv) * scale_log2;
          sc = (j >= rlo && j < rhi) ? sc : -INFINITY;
          mx = fmaxf(mx, sc);
          sr[e] = __float_as_uint(sc);
        }
        tmem_st32(trow + 32 * c, sr);
      }
      tmem_st_wait();
      // ---- online-softmax bookkeeping
      float alpha = 1.f;
      if (mx > m_ref + 8.f) {  // also taken when m_ref is -inf and mx finite
        alpha = (m_ref == -INFINITY) ? 1.f : exp2f(m_ref - mx);
        m_ref = mx;
      }
      l *= alpha;
      if (t > 0) {
        if (!warp_wait(&ss->bar_o, par ^ 1, err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t o[16];
            tmem_ld16(trow + 384 + 16 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(trow + 384 + 16 * c, o);
          }
          tmem_st_wait();
        }
      }
      // ---- pass 2: probabilities -> shared memory (bf16, A operand of P.V)
      const bool live = m_ref != -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32];
        tmem_ld32(trow + 32 * c, sr);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = live ? exp2f(__uint_as_float(sr[2 * e]) - m_ref) : 0.f;
          const float p1 = live ? exp2f(__uint_as_float(sr[2 * e + 1]) - m_ref) : 0.f;
          l += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        uint8_t* half = sPr + (c >> 1) * kHalf;
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<uint4*>(half + sw128_offset(il, (c & 1) * 4 + v)) =
              make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
      tc_fence_before();
      mbar_arrive(&ss->bar_sfree);
      fence_proxy_async_smem();
      mbar_arrive(&ss->bar_p);
    }
    // ---- epilogue: out = O / l
    if (ok && nt > 0) ok = warp_wait(&ss->bar_o, (nt - 1) & 1, err, kDevTimeoutMma);
    if (ok) tc_fence_after();
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      if (ok && nt > 0) {
        tmem_ld32(trow + 384 + 32 * c, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0u;
      }
      if (i < T) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = pack_bf16x2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<size_t>(b) * T + i) * D +
                                              h * kDh + 32 * c);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
    }
    if (!ok) *abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t launch_relpos_attn_bf16(const void* qkv, const void* p, const float* u,
                                    const float* v, const int32_t* key_len, AttnContextDev ctx,
                                    void* out, int B, int T, int H, int* err, int num_sms,
                                    cudaStream_t stream) {
  (void)num_sms;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(relpos_attn_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int D = H * kDh;
  CUtensorMap map_qkv, map_p;
  if (!make_tmap_3d(&map_qkv, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3ull * D, T, B,
                    3ull * D * 2, 3ull * D * 2 * T, 64, kTile, 1, true))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&map_p, p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, 2ull * T - 1,
                    static_cast<uint64_t>(D) * 2, 64, kTile, true))
    return cudaErrorInvalidValue;
  dim3 grid((T + kTile - 1) / kTile, H, B);
  relpos_attn_kernel<<<grid, kThreads, kSmemBytes, stream>>>(
      map_qkv, map_p, u, v, key_len, ctx, static_cast<__nv_bfloat16*>(out), T, H, err);
  return cudaGetLastError();
}

}  // namespace nrp
