// gemm_sm100.cu -- Y[M,N] = X[M,K] . W[N,K]^T (+ bias[N]) on tcgen05.
//
// Serves LinearLayer::forward (reference: src/core/quantization.rs:126-162)
// for the rel-pos MHA projections: the Standard arm (bf16 W staged by TMA)
// and the Quantized arm (MLX affine 8-bit, group 64: W = scale*q + bias),
// where producer warps dequantise u8 weights straight into the swizzled
// shared-memory B tile, so the dequantised matrix never exists in HBM.
//
// Tiling: 128 x 256 output tile per CTA step (128 x 128, 128 x 192 or, for
// problems whose 128-wide tiles fill at most half the SMs, 128 x 64 when
// that fills the persistent grid's one wave better), K in 64-element stages
// (one 128-byte swizzle atom per row; also exactly one quantisation group), a
// 4-deep TMA/mbarrier pipeline, and two 256-column TMEM accumulators so the
// epilogue of tile t overlaps the MMAs of tile t+1.  The grid is persistent
// (one CTA per SM, tiles strided by gridDim.x).
//
// Warp roles (bf16: 6 warps; quantised: 10 warps):
//   warp 0      TMA producer for X (and W in the bf16 case)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2-5   epilogue: TMEM -> registers -> +bias -> bf16 -> a 32 x 64
//               swizzled shared-memory slab per warp (double-buffered) ->
//               TMA tensor store (full-sector writes; M/N tails clipped)
//   warps 6-9   (quantised only) u8 -> bf16 dequantising producer for W
#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kBM = 128;
// Output tiles are 128 x kBN with kBN = 256 (large problems), 128 (problems
// with few tiles: twice the CTAs, and 6 pipeline stages in the same budget)
// or 192 (bf16 W: when 128-wide tiles overflow one wave and 192-wide fit it).
constexpr int kBK = 64;
constexpr int kMaxStages = 7;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
template <int kBN>
struct TileCfg {
  static constexpr int kStages = kBN == 64 ? 7 : kBN == 128 ? 6 : 4;
  static constexpr uint32_t kBBytes = kBN * kBK * 2;  // 32 / 24 / 16 / 8 KB
};
constexpr int kEpiWarp0 = 2;
constexpr int kDeqWarp0 = 6;

struct GemmSmem {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kSlabBytes = 32 * 128;  // 32 rows x 64 bf16, 128B-swizzled
constexpr uint32_t kEpiBytes = 4 * 2 * kSlabBytes;  // 4 warps x 2 buffers
constexpr int kMaxBatch = 256;  // batched tiling: utterances per GEMM
// A CTA pair (kPair) shares 256-row x 256-column tiles: each CTA holds its
// own 128 rows of X and half of the tile's W rows (16 KB per stage), so six
// stages fit where one CTA's 128 x 256 tile fits four.
template <int kBN, bool kPair>
struct StageCfg {
  static constexpr int kStages = kPair ? 6 : TileCfg<kBN>::kStages;
  static constexpr uint32_t kBBytes = kPair ? kBN / 2 * kBK * 2 : TileCfg<kBN>::kBBytes;
};
template <int kBN, bool kPair = false>
constexpr size_t smem_bytes() {
  return 1024 /*align slack*/ +
         StageCfg<kBN, kPair>::kStages * (kABytes + StageCfg<kBN, kPair>::kBBytes) + kEpiBytes +
         256 + 4 * (kMaxBatch + 1);
}
static_assert(smem_bytes<256>() <= 232448 && smem_bytes<192>() <= 232448 &&
                  smem_bytes<128>() <= 232448 && smem_bytes<64>() <= 232448 &&
                  smem_bytes<256, true>() <= 232448,
              "shared memory budget");

// v[e] += bias[n + e] for e < 32 (zero past N); 16-byte loads when `vec`.
__device__ __forceinline__ void add_bias32(float* v, const __nv_bfloat16* bias, int n, int N,
                                           bool vec) {
  if (vec && n + 32 <= N) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = *reinterpret_cast<const uint4*>(bias + n + q * 8);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[e]));
        v[q * 8 + 2 * e] += f.x;
        v[q * 8 + 2 * e + 1] += f.y;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] += n + e < N ? __bfloat162float(bias[n + e]) : 0.f;
  }
}
__device__ __forceinline__ void add_bias64(float* v, const __nv_bfloat16* bias, int n, int N,
                                           bool vec) {
  add_bias32(v, bias, n, N, vec);
  add_bias32(v + 32, bias, n + 32, N, vec);
}

template <bool kQuant, int kBN, bool kPair>
__global__ void __launch_bounds__(kQuant ? 320 : 192, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_w,
                   const __grid_constant__ CUtensorMap map_y,  // [M, N] bf16, box (64, 32)
                   const uint8_t* __restrict__ wq,         // quantised: [N, K] bytes
                   const __nv_bfloat16* __restrict__ qs,   // [N, K/64]
                   const __nv_bfloat16* __restrict__ qb,   // [N, K/64]
                   const __nv_bfloat16* __restrict__ bias, // [N] or null
                   int M, int N, int K, RowTiling rt, Epilogue ep, int w_early, int* err) {
  static_assert(!kPair || (!kQuant && kBN == 256), "pair tiles: bf16 W, 256 columns");
  constexpr int kStages = StageCfg<kBN, kPair>::kStages;
  constexpr uint32_t kBBytes = StageCfg<kBN, kPair>::kBBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = base;
  uint8_t* sB = base + kStages * kABytes;
  uint8_t* sE = sB + kStages * kBBytes;
  GemmSmem* ss = reinterpret_cast<GemmSmem*>(sE + kEpiBytes);

  const int warp = warp_id();
  const int lane = lane_id();
  // Row tiles: flat over M, or (batched) per utterance so a tile never
  // straddles two.  In the batched form with lengths, the persistent tile
  // list holds every row tile that has a valid frame first, then the tiles
  // wholly past their utterance's length (which only write zeros), so the
  // skipped work is not left as holes in the static assignment.
  const bool batched = rt.T > 0;
  const int tpb = batched ? (rt.T + kBM - 1) / kBM : 0;
  const int tiles_m = batched ? rt.B * tpb : (M + kBM - 1) / kBM;
  const int tiles_n = (N + kBN - 1) / kBN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = K / kBK;
  // Work items: single tiles, or (kPair) pairs of row tiles 2i, 2i + 1 that
  // share a column tile, CTA rank r of the pair taking row tile 2i + r.
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int num_work = kPair ? ((tiles_m + 1) / 2) * tiles_n : num_tiles;
  const int work0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int work_step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // tile of CTA rank r in work item w; -1 past the last row tile
  auto tile_of = [&](int w, int r) -> int {
    if (!kPair) return w;
    const int tm = 2 * (w / tiles_n) + r;
    return tm < tiles_m ? tm * tiles_n + w % tiles_n : -1;
  };
  int* live_pre = reinterpret_cast<int*>(sE + kEpiBytes + sizeof(GemmSmem));  // [B+1]
  int live_m = tiles_m;  // (set from the lengths after pdl_wait below)
  // list index -> (first row of the tile, its utterance); true = zero-fill tile
  auto tile_rows = [&](int tile, int& r0, int& bb) -> bool {
    const int tm = tile / tiles_n;
    if (!batched) {
      r0 = tm * kBM;
      bb = 0;
      return false;
    }
    if (!rt.len) {
      bb = tm / tpb;
      r0 = (tm - bb * tpb) * kBM;
      return false;
    }
    if (tm < live_m) {  // k-th live row tile
      int b = 0;
      while (live_pre[b + 1] <= tm) ++b;
      bb = b;
      r0 = (tm - live_pre[b]) * kBM;
      return false;
    }
    int k = tm - live_m, b = 0;  // k-th dead row tile
    for (;; ++b) {
      const int dead = tpb - (live_pre[b + 1] - live_pre[b]);
      if (k < dead) break;
      k -= dead;
    }
    bb = b;
    r0 = (live_pre[b + 1] - live_pre[b] + k) * kBM;
    return true;
  };
  // This CTA's rows of work item w (m0, bb), whether they are dead (zeros
  // written) or absent (no row tile: loads fall outside X and read zeros,
  // nothing is written); returns whether the item runs MMAs (a pair runs
  // unless neither of its tiles is live).
  auto work_rows = [&](int w, int& m0, int& bb, bool& dead, bool& absent) -> bool {
    const int t = tile_of(w, static_cast<int>(rank));
    absent = t < 0;
    if (absent) {
      m0 = batched ? tpb * kBM : tiles_m * kBM;
      bb = 0;
      dead = true;
    } else {
      dead = tile_rows(t, m0, bb);
    }
    if (!kPair) return !dead;
    const int to = tile_of(w, static_cast<int>(rank ^ 1u));
    int m1 = 0, b1 = 0;
    const bool other_dead = to < 0 || tile_rows(to, m1, b1);
    return !(dead && other_dead);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ss->full[s], kQuant ? 1 + 4 : 1);  // TMA + one arrival per dequant warp
      mbar_init(&ss->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ss->tfull[b], 1);
      mbar_init(&ss->tempty[b], kPair ? 8 : 4);  // the epilogue warps of the pair
    }
    ss->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (kPair) {
      tmem_alloc_pair(&ss->tmem_base, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&ss->tmem_base, 512);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x);
    if (!kQuant) prefetch_tensormap(&map_w);
  }
  tc_fence_before();
  if (kPair)
    cluster_sync();  // both CTAs' barriers are initialised before either signals them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ss->tmem_base;
  volatile int* abort_flag = &ss->abort;
  // The weights were not written by the kernels before this one (w_early):
  // the first tile's first W stages load before the wait on the previous
  // kernel, so their HBM latency hides under its tail.  Only when the tile
  // list does not depend on device lengths (the first tile is live).
  int pre = 0;
  if (!kQuant && !kPair && w_early && !(batched && rt.len) && warp == 0 && lane == 0 &&
      static_cast<int>(blockIdx.x) < num_tiles) {
    const int n0 = (static_cast<int>(blockIdx.x) % tiles_n) * kBN;
    pre = num_kb < kStages ? num_kb : kStages;
    for (int s = 0; s < pre; ++s) {
      mbar_arrive_expect_tx(&ss->full[s], kABytes + kBBytes);
      tma_load_2d(sB + s * kBBytes, &map_w, &ss->full[s], s * kBK, n0);
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  // the lengths may come from the previous kernel in the stream: read them
  // only after its grid is complete
  if (batched && rt.len) {
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int b = 0; b < rt.B; ++b) {
        live_pre[b] = acc;
        const int L = rt.len[b];
        acc += L <= 0 ? 0 : min(tpb, (L + kBM - 1) / kBM);
      }
      live_pre[rt.B] = acc;
    }
    __syncthreads();
    live_m = live_pre[rt.B];
  }

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int w = work0; w < num_work && !*abort_flag; w += work_step) {
        int m0, bb;
        bool dead, absent;
        if (!work_rows(w, m0, bb, dead, absent)) continue;
        const int n0 = (w % tiles_n) * kBN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t round = it / kStages;
          if (static_cast<int>(it) < pre) {  // W already on its way: X only
            if (batched)
              tma_load_3d(sA + s * kABytes, &map_x, &ss->full[s], kb * kBK, m0, bb);
            else
              tma_load_2d(sA + s * kABytes, &map_x, &ss->full[s], kb * kBK, m0);
            continue;
          }
          if (!mbar_wait(&ss->empty[s], (round & 1) ^ 1, err, kDevTimeoutLoad)) {
            *abort_flag = 1;
            break;
          }
          if (kPair) {
            // both CTAs' stage bytes complete on the leader's barrier, whose
            // single arrival (with the pair's byte count) comes from here
            if (rank == 0) mbar_arrive_expect_tx(&ss->full[s], 2 * (kABytes + kBBytes));
            const uint32_t lb = leader_smem(smem_u32(&ss->full[s]));
            if (batched)
              tma_load_3d_pair(sA + s * kABytes, &map_x, lb, kb * kBK, m0, bb);
            else
              tma_load_2d_pair(sA + s * kABytes, &map_x, lb, kb * kBK, m0);
            tma_load_2d_pair(sB + s * kBBytes, &map_w, lb, kb * kBK,
                             n0 + static_cast<int>(rank) * (kBN / 2));
            continue;
          }
          mbar_arrive_expect_tx(&ss->full[s], kQuant ? kABytes : kABytes + kBBytes);
          if (batched)
            tma_load_3d(sA + s * kABytes, &map_x, &ss->full[s], kb * kBK, m0, bb);
          else
            tma_load_2d(sA + s * kABytes, &map_x, &ss->full[s], kb * kBK, m0);
          if (!kQuant) tma_load_2d(sB + s * kBBytes, &map_w, &ss->full[s], kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    // (a pair's MMAs come from its leader CTA alone)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kPair ? 2 * kBM : kBM, kBN, 0, 0);
      uint32_t it = 0;
      int tc = 0;
      for (int w = work0; w < num_work && !*abort_flag; w += work_step) {
        int m0, bb;
        bool dead, absent;
        if (!work_rows(w, m0, bb, dead, absent)) continue;
        const int buf = tc & 1;
        const uint32_t use = tc >> 1;
        ++tc;
        if (!mbar_wait(&ss->tempty[buf], (use & 1) ^ 1, err, kDevTimeoutEpi)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + buf * kBN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t round = it / kStages;
          if (!mbar_wait(&ss->full[s], round & 1, err, kDevTimeoutLoad)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kABytes);
          const uint32_t b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + k * 32, 16, 1024);
            if (kPair)
              umma_ss_pair(dcol, ad, bd, idesc, (kb | k) != 0);
            else
              umma_ss(dcol, ad, bd, idesc, (kb | k) != 0);
          }
          if (kPair)
            umma_commit_pair_mc(&ss->empty[s], 0x3);  // both CTAs' stages are free
          else
            umma_commit(&ss->empty[s]);
        }
        if (!ok) break;
        if (kPair)
          umma_commit_pair_mc(&ss->tfull[buf], 0x3);  // both CTAs' accumulators
        else
          umma_commit(&ss->tfull[buf]);
      }
    }
  } else if (warp < kEpiWarp0 + 4) {
    // --------------------------------------------------------- epilogue
    const int quad = warp & 3;
    uint8_t* slab = sE + (warp - kEpiWarp0) * 2 * kSlabBytes;
    if (lane == 0) prefetch_tensormap(&map_y);
    int tc = 0;
    uint32_t nslab = 0;
    for (int w = work0; w < num_work && !*abort_flag; w += work_step) {
      int m0, bb;
      bool skip, absent;  // skip: zeros (dead rows); absent: nothing to write
      const bool runs = work_rows(w, m0, bb, skip, absent);
      const int n0 = (w % tiles_n) * kBN;
      const int buf = tc & 1;
      const uint32_t use = tc >> 1;
      const bool glu = ep.mode == kEpiGlu;
      // bias columns come 8 at a time (16-byte loads) when the pointer allows
      const bool bias_vec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
      const int ncols = glu ? kBN / 2 : kBN;  // output columns of the tile
      const int on0 = glu ? n0 / 2 : n0;      // its first output column
      const int n_out = glu ? N / 2 : N;
      const int row = m0 + quad * 32 + lane;  // this thread's row (in its utterance)
      const bool row_in = row < (batched ? rt.T : M);
      bool keep = true;  // GLU: padded frames are zeros
      if (glu && ep.len && batched && !skip) keep = row < ep.len[bb];
      // residual rows are read one 64-column slab ahead; the first slab's
      // loads go out before the wait for the accumulator, under the MMAs
      const bool resid = ep.mode == kEpiResidual && !skip && row_in;
      const __nv_bfloat16* rrow = nullptr;
      if (resid) {
        const int64_t bs = ep.res_bs ? ep.res_bs : static_cast<int64_t>(rt.T) * ep.ldr;
        rrow = ep.res + (batched ? bb * bs : 0) + static_cast<int64_t>(row) * ep.ldr + on0;
      }
      uint4 resv[8];
      auto load_res = [&](int cc) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          resv[ch] = (resid && on0 + cc + ch * 8 < n_out)
                         ? *reinterpret_cast<const uint4*>(rrow + cc + ch * 8)
                         : make_uint4(0u, 0u, 0u, 0u);
      };
      load_res(0);
      if (runs) {
        ++tc;
        if (!mbar_wait(&ss->tfull[buf], use & 1, err, kDevTimeoutMma)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
      }
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * kBN;
#pragma unroll 1
      for (int c = 0; c < ncols; c += 64) {
        float v[64];
        if (!skip && glu) {
#pragma unroll
          for (int h = 0; h < 64; h += 32) {  // value columns c+h.., gate columns 128+c+h..
            uint32_t ar[32], gr[32];
            tmem_ld32(taddr + c + h, ar);
            tmem_ld32(taddr + 128 + c + h, gr);
            tmem_ld_wait();
            float a[32], g[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              a[e] = __uint_as_float(ar[e]);
              g[e] = __uint_as_float(gr[e]);
            }
            if (bias) {
              add_bias32(a, bias, n0 + c + h, N, bias_vec);
              add_bias32(g, bias, n0 + 128 + c + h, N, bias_vec);
            }
#pragma unroll
            for (int e = 0; e < 32; ++e)
              v[h + e] = keep ? a[e] * sigmoid_approx(g[e]) : 0.f;
          }
        } else if (!skip) {
          uint32_t r[64];
          tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          tmem_ld32(taddr + c + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
          {
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 64; ++e) v[e] = __uint_as_float(r[e]);
            if (ep.mode == kEpiRelu) {  // the conv's own rounding, before its bias add
#pragma unroll
              for (int e = 0; e < 64; ++e) v[e] = __bfloat162float(__float2bfloat16_rn(v[e]));
            }
            if (bias) add_bias64(v, bias, n0 + c, N, bias_vec);
            if (ep.mode == kEpiSilu) {
#pragma unroll
              for (int e = 0; e < 64; ++e) v[e] = v[e] * sigmoid_approx(v[e]);
            } else if (ep.mode == kEpiRelu) {
#pragma unroll
              for (int e = 0; e < 64; ++e) v[e] = fmaxf(v[e], 0.f);
            } else if (resid) {
#pragma unroll
              for (int ch = 0; ch < 8; ++ch) {
                const uint4 q = resv[ch];
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f =
                      __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[e]));
                  fma_f32x2v(v[ch * 8 + 2 * e], v[ch * 8 + 2 * e + 1], v[ch * 8 + 2 * e],
                             v[ch * 8 + 2 * e + 1], ep.alpha, f.x, f.y);
                }
              }
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) v[e] = 0.f;
        }
        if (resid && c + 64 < ncols) load_res(c + 64);  // the next slab's residual
        if (absent || on0 + c >= n_out) continue;  // whole slab past N (warp-uniform)
        uint8_t* sb = slab + (nslab & 1) * kSlabBytes;
        // the store issued two slabs ago must have finished reading sb
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) pk[e] = pack_bf16x2(v[ch * 8 + 2 * e], v[ch * 8 + 2 * e + 1]);
          *reinterpret_cast<uint4*>(sb + sw128_offset(lane, ch)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (batched)
            tma_store_3d(&map_y, sb, on0 + c, m0 + quad * 32, bb);
          else
            tma_store_2d(&map_y, sb, on0 + c, m0 + quad * 32);
          bulk_commit();
        }
        ++nslab;
      }
      if (runs) {  // the accumulator may take the next work item (the pair's leader counts 8)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (kPair && rank != 0)
            mbar_arrive_cluster(&ss->tempty[buf], 0);
          else
            mbar_arrive(&ss->tempty[buf]);
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // stores read shared memory until done
  } else if (kQuant) {
    // ------------------------------------------ dequantising W producer
    // 4 threads per W row, 16 bytes (16 weights) each; 32 rows per pass.
    const int t = threadIdx.x - kDeqWarp0 * 32;  // 0..127
    const int sub = t & 3;
    const int row0 = t >> 2;
    const int kgroups = K / 64;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
      int m0, bb;
      if (tile_rows(tile, m0, bb)) continue;
      const int n0 = (tile % tiles_n) * kBN;
      for (int kb = 0; kb < num_kb; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t round = it / kStages;
        if (!mbar_wait(&ss->empty[s], (round & 1) ^ 1, err, kDevTimeoutLoad)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* tileB = sB + s * kBBytes;
#pragma unroll 2
        for (int pass = 0; pass < kBN / 32; ++pass) {
          const int r = row0 + pass * 32;
          const int n = n0 + r;
          uint4 q = make_uint4(0, 0, 0, 0);
          float sc = 0.f, bi = 0.f;
          if (n < N) {
            q = *reinterpret_cast<const uint4*>(wq + static_cast<size_t>(n) * K + kb * kBK +
                                                sub * 16);
            sc = __bfloat162float(qs[static_cast<size_t>(n) * kgroups + kb]);
            bi = __bfloat162float(qb[static_cast<size_t>(n) * kgroups + kb]);
          }
          const uint32_t words[4] = {q.x, q.y, q.z, q.w};
          uint32_t outw[8];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t v = words[w];
            const float f0 = fmaf(sc, static_cast<float>(v & 0xFF), bi);
            const float f1 = fmaf(sc, static_cast<float>((v >> 8) & 0xFF), bi);
            const float f2 = fmaf(sc, static_cast<float>((v >> 16) & 0xFF), bi);
            const float f3 = fmaf(sc, static_cast<float>(v >> 24), bi);
            outw[2 * w] = pack_bf16x2(f0, f1);
            outw[2 * w + 1] = pack_bf16x2(f2, f3);
          }
          // elements [sub*16, sub*16+16) of the row = 16-byte chunks 2*sub, 2*sub+1
          *reinterpret_cast<uint4*>(tileB + sw128_offset(r, 2 * sub)) =
              make_uint4(outw[0], outw[1], outw[2], outw[3]);
          *reinterpret_cast<uint4*>(tileB + sw128_offset(r, 2 * sub + 1)) =
              make_uint4(outw[4], outw[5], outw[6], outw[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ss->full[s]);
      }
    }
  }

  tc_fence_before();
  if (kPair) {
    // neither CTA leaves (or frees the pair's TMEM) while the other may still
    // signal its barriers or feed the leader's MMAs from its shared memory
    cluster_sync();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, 512);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
  }
}

}  // namespace

int gemm_smem_bytes() { return static_cast<int>(smem_bytes<256>()); }

namespace {
bool make_y_map(CUtensorMap* map, __nv_bfloat16* y, int ldy, int M, int N, const RowTiling& rt) {
  if (rt.T > 0) {
    const uint64_t bstride = rt.y_bstride > 0 ? static_cast<uint64_t>(rt.y_bstride)
                                              : static_cast<uint64_t>(ldy) * rt.T;
    return make_tmap_3d(map, y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, rt.T, rt.B,
                        static_cast<uint64_t>(ldy) * 2, bstride * 2, 64, 32, 1, true);
  }
  return make_tmap_2d(map, y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M,
                      static_cast<uint64_t>(ldy) * 2, 64, 32, true);
}
// The residual is read with 16-byte loads; GLU tiles pair 128 value and 128
// gate columns.
bool epilogue_ok(const Epilogue& ep, int N) {
  if (ep.mode == kEpiResidual)
    return ep.res && ep.ldr % 8 == 0 && ep.res_bs % 8 == 0 && N % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(ep.res) & 15) == 0;
  if (ep.mode == kEpiGlu) return N % 256 == 0;
  return ep.mode == kEpiBias || ep.mode == kEpiSilu || ep.mode == kEpiRelu;
}
int tiles_m_of(int M, const RowTiling& rt) {
  return rt.T > 0 ? rt.B * ((rt.T + kBM - 1) / kBM) : (M + kBM - 1) / kBM;
}
// 128-wide tiles when 256-wide ones would not fill one wave of the persistent
// grid (M = 896 rows of a streaming chunk: 84 tiles -> 168).  With more tiles
// the 256-wide tile is faster per FLOP (it reads 1.5x less shared memory per
// MMA), which outweighs the better wave fill (config 1's linear_out: 312
// tiles ran 7% slower as 624).  GLU needs the 256-wide layout.
// The CTA-pair GEMM is on unless NRP_PAIR_GEMM=0 (read once).
bool pair_gemm_enabled() {
  static const int on = [] {
    const char* e = getenv("NRP_PAIR_GEMM");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}
int pick_bn(int M, int N, const RowTiling& rt, const Epilogue& ep, int num_sms) {
  if (ep.mode == kEpiGlu) return 256;
  const int tiles256 = tiles_m_of(M, rt) * ((N + 255) / 256);
  return tiles256 < num_sms ? 128 : 256;
}
int grid_size(int M, int N, int bn, const RowTiling& rt, int num_sms) {
  const int tiles = tiles_m_of(M, rt) * ((N + bn - 1) / bn);
  return tiles < num_sms ? tiles : num_sms;
}

template <bool kQuant, int kBN, bool kPair = false>
cudaError_t launch_tn(const CUtensorMap& map_x, const void* w, const uint8_t* wq,
                      const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                      const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int M, int N, int K,
                      int num_sms, int* err, cudaStream_t stream, const RowTiling& rt,
                      const Epilogue& ep, bool w_early) {
  static std::atomic<uint64_t> attr{0};
  constexpr int kSmem = static_cast<int>(smem_bytes<kBN, kPair>());
  if (cudaError_t e = smem_attr_once(gemm_tn_kernel<kQuant, kBN, kPair>, kSmem, attr)) return e;
  CUtensorMap map_w = map_x;  // unused by the quantised kernel
  // a pair's CTA loads half of the tile's W rows
  if (!kQuant && !make_tmap_2d(&map_w, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N,
                               static_cast<uint64_t>(K) * 2, 64, kPair ? kBN / 2 : kBN, true))
    return cudaErrorInvalidValue;
  CUtensorMap map_y;
  if (!make_y_map(&map_y, y, ldy, M, ep.mode == kEpiGlu ? N / 2 : N, rt))
    return cudaErrorInvalidValue;
  if constexpr (!kPair) {
    const int grid = grid_size(M, N, kBN, rt, num_sms);
    return launch_pdl(gemm_tn_kernel<kQuant, kBN, false>, dim3(grid), dim3(kQuant ? 320 : 192),
                      static_cast<size_t>(kSmem), stream, map_x, map_w, map_y, wq, qs, qb, bias,
                      M, N, K, rt, ep, w_early ? 1 : 0, err);
  } else {
  // clusters of two CTAs, one per work item (a pair of row tiles), at most
  // one per two SMs
  const int tiles_m = tiles_m_of(M, rt), tiles_n = (N + kBN - 1) / kBN;
  const int work = ((tiles_m + 1) / 2) * tiles_n;
  const int pairs = std::min(work, std::max(1, (num_sms > 0 ? num_sms : 148) / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = static_cast<size_t>(kSmem);
  cfg.stream = stream;
  cudaLaunchAttribute la[2];
  la[0].id = cudaLaunchAttributeClusterDimension;
  la[0].val.clusterDim.x = 2;
  la[0].val.clusterDim.y = 1;
  la[0].val.clusterDim.z = 1;
  la[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = la;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemm_tn_kernel<kQuant, kBN, true>, map_x, map_w, map_y, wq,
                            qs, qb, bias, M, N, K, rt, ep, 0, err);
  }
}
}  // namespace

cudaError_t launch_gemm_bf16(const CUtensorMap& map_x, const void* w,
                             const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int M, int N,
                             int K, int num_sms, int* err, cudaStream_t stream, RowTiling rt,
                             const Epilogue& ep, bool w_early) {
  if (rt.T > 0 && (rt.B < 1 || rt.B > kMaxBatch)) return cudaErrorInvalidValue;
  if (!epilogue_ok(ep, N)) return cudaErrorInvalidValue;
  const int bn = pick_bn(M, N, rt, ep, num_sms);
  // 192-wide tiles when 128-wide ones would spill past one wave and
  // 192-wide ones fit it (the Q|K|V projection of a streaming chunk step,
  // M = 896, N = 3072: 168 tiles -> 112, so no SM runs a second tile)
  const int tm = tiles_m_of(M, rt);
  if (bn == 128 && ep.mode != kEpiGlu && N % 192 == 0 && tm * (N / 128) > num_sms &&
      tm * (N / 192) <= num_sms)
    return launch_tn<false, 192>(map_x, w, nullptr, nullptr, nullptr, bias, y, ldy, M, N, K,
                                 num_sms, err, stream, rt, ep, w_early);
  // 64-wide tiles when 128-wide ones fill at most half the SMs (the N = 1024
  // projections of a streaming chunk step, M = 896: 56 tiles -> 112): each
  // CTA streams a quarter less, and twice the SMs pull their operands
  if (bn == 128 && ep.mode != kEpiGlu && N % 64 == 0 && 2 * tm * ((N + 127) / 128) <= num_sms)
    return launch_tn<false, 64>(map_x, w, nullptr, nullptr, nullptr, bias, y, ldy, M, N, K,
                                num_sms, err, stream, rt, ep, w_early);
  if (bn == 128)
    return launch_tn<false, 128>(map_x, w, nullptr, nullptr, nullptr, bias, y, ldy, M, N, K,
                                 num_sms, err, stream, rt, ep, w_early);
  // CTA pairs (256 x 256 tiles shared by two SMs) for tall problems: from
  // 128 row tiles on (same-box A/B: config 3's encoder, 128 row tiles, 21.2 ->
  // 20.3 ms; config 4's windowed layer, 391, 0.595 -> 0.571 ms; config 1's
  // 96 per-utterance row tiles ran 2% slower as pairs)
  if (pair_gemm_enabled() && N % 256 == 0 && tm >= 128 &&
      ((tm + 1) / 2) * (N / 256) >= (num_sms > 0 ? num_sms : 148) / 2)
    return launch_tn<false, 256, true>(map_x, w, nullptr, nullptr, nullptr, bias, y, ldy, M, N,
                                       K, num_sms, err, stream, rt, ep, w_early);
  return launch_tn<false, 256>(map_x, w, nullptr, nullptr, nullptr, bias, y, ldy, M, N, K,
                               num_sms, err, stream, rt, ep, w_early);
}

cudaError_t launch_gemm_q8(const CUtensorMap& map_x, const uint8_t* wq, const __nv_bfloat16* qs,
                           const __nv_bfloat16* qb, const __nv_bfloat16* bias, __nv_bfloat16* y,
                           int ldy, int M, int N, int K, int num_sms, int* err,
                           cudaStream_t stream, RowTiling rt, const Epilogue& ep) {
  if (rt.T > 0 && (rt.B < 1 || rt.B > kMaxBatch)) return cudaErrorInvalidValue;
  if (!epilogue_ok(ep, N)) return cudaErrorInvalidValue;
  if (pick_bn(M, N, rt, ep, num_sms) == 128)
    return launch_tn<true, 128>(map_x, nullptr, wq, qs, qb, bias, y, ldy, M, N, K, num_sms, err,
                                stream, rt, ep, false);
  return launch_tn<true, 256>(map_x, nullptr, wq, qs, qb, bias, y, ldy, M, N, K, num_sms, err,
                              stream, rt, ep, false);
}

}  // namespace nrp
