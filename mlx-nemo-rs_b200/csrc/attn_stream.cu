// attn_stream.cu -- cache-aware streaming rel-pos attention on tensor cores.
//
// RelPositionMultiHeadAttention::forward_with_cache
// (src/asr/modules/encoders/attention.rs:606-816) between the projections:
// a chunk of T query frames attends over Tk = C + T keys, the C cached
// frames (read in place from the ring, slot (head + j) mod C) and the
// chunk's own.  The positional term is rel_shift((q+v) . P^T)[i, j] =
// (q_i+v) . P[T-1-i+j] (attention.rs:832-855) with P = linear_pos of the
// 2Tk-1 positions, projected once per length (749-761).
//
// Shapes are small (config 2: T = 14 queries, Tk = 84 keys per session and
// head) and K, V are read once.  One CTA of 4 warps takes 16 query rows of
// one (session, head):
//   0. before waiting on the projection kernel, the session's ring rows of
//      this head (K and V) are prefetched into L2 (they were written by an
//      earlier launch; the prefetch overlaps the projection GEMM) and the
//      positional biases are loaded;
//   1. after the wait, one thread issues TMA tensor copies (128-byte swizzled
//      boxes of 64 head dims, mbarrier completion, bounded waits): the
//      tile's q rows, then K -- the whole ring of the session in slot order,
//      one box per half, and the chunk's rows -- so a CTA's K arrives in
//      four copies and one round trip; a key's shared row is its ring slot
//      (head + j mod C) or, for the chunk, a row after the ring;
//   2. q+u and q+v are rounded to bf16 into shared memory;
//   3. mma.sync m16n8k16 (bf16 -> f32): W = (q+v) P_win^T over 16-column
//      tiles dealt to the warps, the B operand (the batch-shared, L2-resident
//      positional rows) loaded from global memory as 16-byte rows with a
//      double-buffered register pipeline while K lands; then S = (q+u) K^T
//      from shared memory.  The 128-dim contraction runs in a permuted order
//      (k-step 2s+t, lane column 2c+e <-> head dim 32s+8c+4t+e, and +2 for
//      the upper half), the same for both operands, so one 16-byte load of
//      a row gives a lane its fragments of two k-steps;
//   4. the chunk's new K rows go from shared memory into the ring, and V is
//      copied (as K) into the same buffer;
//   5. softmax, four rows per warp at once (8 lanes a row), while V lands:
//      score(i, j) = (S[i][j] + W[i][15 - i + j]) / sqrt(dh) -- rel_shift is
//      the skewed read of W --, masked by the streaming mask
//      (create_attention_mask, conformer.rs:97-221), bf16 probabilities;
//   6. O = P . V with V rows read from shared memory and transposed by
//      movmatrix (8x8 blocks of (key, dim-pair) words), so each lane ends
//      with 8 contiguous output dims of two rows: one 16-byte store each;
//   7. when the chunk fits one CTA, the new V and x rows (the latter loaded
//      into registers after the wait) are written into the ring for this
//      head's columns -- the sliding window update of 661-684 -- after the
//      CTA's copies of the ring have landed; no other CTA touches these
//      columns.
// Shared memory is ~54 KB per CTA at Tk = 84, so four CTAs share an SM and
// config 2's 512 (session, head) items run as one wave; the kernel is bound
// by HBM (K and V, 22 MB per layer at config 2).
#include <cuda_bf16.h>

#include "gemm.h"
#include "masks.cuh"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kQ = 16;        // query rows per CTA
constexpr int kDh = 128;
constexpr int kLd = kDh + 8;  // shared q row stride in bf16 (272 B: conflict-free 16-byte reads)
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxKeys = 256;
constexpr uint32_t kRowBytes = kDh * 2;  // one head's row of q, K or V

// 2^x with the MUFU approximation (arguments here are <= 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// Transpose of an 8x8 b16 matrix held one 32-bit word (row g, columns
// 2c, 2c+1) per lane.
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(a));
  return d;
}

// 16 bytes from global memory, or zeros when !pred.  The zeros are written
// before a predicated load, so no instruction waits on the load's result
// until its first real use (a select between the two would).
__device__ __forceinline__ uint4 ld16z(const __nv_bfloat16* p, bool pred) {
  uint4 r;
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %5, 0;\n"
      " mov.b32 %0, 0;\n mov.b32 %1, 0;\n mov.b32 %2, 0;\n mov.b32 %3, 0;\n"
      " @q ld.global.v4.b32 {%0, %1, %2, %3}, [%4];\n}\n"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "r"(static_cast<int>(pred)));
  return r;
}

__device__ __forceinline__ uint32_t word(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// d += a . b for one m16n8k16 tile (bf16 inputs, f32 accumulate).
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct StreamSmem {
  int nk, np;     // key rows (Tk rounded up to 16), P window rows
  int c8;         // first row of the chunk's keys in a key half (C rounded up to 8)
  int lds, ldw;   // f32 row strides of S and W (+8: two-wavefront float2 stores)
  int ldpr;       // bf16 row stride of the probabilities
  size_t half;    // bytes of one 64-dim key half (a multiple of 1024)
  size_t off_s, off_w, off_qu, off_qv, off_pr, off_inv, off_bar, bytes;
};

// From a 1024-aligned base: K (then V) as two 64-dim halves of 128-byte rows
// in the TMA's 128-byte swizzle -- ring slots [0, C), the chunk's keys from
// row c8, zero rows up to key nk --, then S (whose first 4 KB stage the
// tile's q rows, also two swizzled halves), W, q+u and q+v [16][kLd], the
// probabilities, 1/row sums and three mbarriers (q, K, V).  `bytes` adds
// 1 KB for aligning the base.
__host__ __device__ inline StreamSmem stream_smem(int C, int T) {
  StreamSmem m;
  const int Tk = C + T;
  m.nk = (Tk + 15) / 16 * 16;
  m.np = (Tk + kQ - 1 + 15) / 16 * 16;
  m.c8 = (C + 7) / 8 * 8;
  m.lds = m.nk + 8;
  m.ldw = m.np + 8;
  m.ldpr = m.nk + 8;
  m.half = (static_cast<size_t>(m.c8 + m.nk - C) * 128 + 1023) / 1024 * 1024;
  size_t o = 2 * m.half;
  m.off_s = o;
  o += static_cast<size_t>(kQ) * m.lds * 4 > 4096 ? static_cast<size_t>(kQ) * m.lds * 4 : 4096;
  m.off_w = o; o += static_cast<size_t>(kQ) * m.ldw * 4;
  m.off_qu = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_qv = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_pr = o; o += static_cast<size_t>(kQ) * m.ldpr * 2;
  m.off_inv = o; o += kQ * 4;
  m.off_bar = o; o += 3 * 8;
  m.bytes = (o + 15) / 16 * 16 + 1024;
  return m;
}

// kKG = ceil(nk / 32): 32-key groups a lane walks in the softmax.
template <int kKG>
__global__ void __launch_bounds__(kThreads, 4)
    stream_attn_kernel(const __grid_constant__ CUtensorMap map_kc,  // ring K [B][C][D], box 64 x C
                       const __grid_constant__ CUtensorMap map_vc,  // ring V
                       const __grid_constant__ CUtensorMap map_q,   // qkv [B][T][3D], box 64 x 16
                       const __grid_constant__ CUtensorMap map_ch,  // qkv, box 64 x T
                       __nv_bfloat16* kc_w, __nv_bfloat16* vc_w, __nv_bfloat16* hc_w,
                       const __nv_bfloat16* __restrict__ x,  // attention input [B][T][D]
                       int C, int head, int n_app, int src0,
                       const __nv_bfloat16* __restrict__ p,  // [2Tk-1][D]
                       const float* __restrict__ pos_u, const float* __restrict__ pos_v,
                       StreamMaskDev sm, __nv_bfloat16* __restrict__ out, int T, int D,
                       int* err) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // the swizzled key halves need a 1024-byte aligned base
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int Tk = C + T;
  const StreamSmem L = stream_smem(C, T);
  uint8_t* sKV = smem;  // half h at h * L.half
  uint8_t* sQs = smem + L.off_s;  // the tile's q rows (two halves of 2 KB), then S
  __nv_bfloat16* sQu = reinterpret_cast<__nv_bfloat16*>(smem + L.off_qu);
  __nv_bfloat16* sQv = reinterpret_cast<__nv_bfloat16*>(smem + L.off_qv);
  float* sS = reinterpret_cast<float*>(smem + L.off_s);
  float* sW = reinterpret_cast<float*>(smem + L.off_w);
  __nv_bfloat16* sPr = reinterpret_cast<__nv_bfloat16*>(smem + L.off_pr);
  float* sInv = reinterpret_cast<float*>(smem + L.off_inv);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);  // q, K, V

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, cq = lane & 3;
  const int i0 = blockIdx.x * kQ, h = blockIdx.y, b = blockIdx.z;
  const int col = h * kDh;

  // shared row of key j: ring slot head + j (mod C) for the cache, c8 + j - C
  // for the chunk's keys and the zero rows after them
  auto krow = [&](int j) -> int {
    if (j < C) {
      const int slot = head + j;
      return slot >= C ? slot - C : slot;
    }
    return L.c8 + j - C;
  };
  // 16 bytes of key row `row`, head dims 8 ch .. 8 ch + 7
  auto kv16 = [&](int row, int ch) -> const uint4* {
    return reinterpret_cast<const uint4*>(sKV + (ch >> 3) * L.half + sw128_offset(row, ch & 7));
  };
  // global row of the ring slot that the r-th appended frame replaces
  auto ring_row = [&](int r) -> int64_t {
    int slot = head + r;
    slot = slot >= C ? slot - C : slot;
    return (static_cast<int64_t>(b) * C + slot) * D + col;
  };

  // ---- 0. barriers; key rows past the chunk zeroed (their probabilities
  // are 0, so their V rows must be finite); the ring's K and V rows of this
  // head into L2 while the projection still runs; the positional biases
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
    for (int hf = 0; hf < 2; ++hf) {
      tma_prefetch_3d(&map_kc, col + 64 * hf, 0, b);
      tma_prefetch_3d(&map_vc, col + 64 * hf, 0, b);
    }
  }
  const int nz = L.nk - Tk;  // zero rows c8 + T ..
  for (int e = tid; e < 2 * nz * 8; e += kThreads) {
    const int hf = e / (nz * 8), r = (e / 8) % nz, ch = e & 7;
    *reinterpret_cast<uint4*>(sKV + hf * L.half + sw128_offset(L.c8 + T + r, ch)) =
        make_uint4(0u, 0u, 0u, 0u);
  }
  const int qrow = tid >> 3, c16 = (tid & 7) * 16;  // phase 2: row tid/8, dims 16 (tid%8) ..
  float4 uu4[4], vv4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uu4[k] = reinterpret_cast<const float4*>(pos_u + col + c16)[k];
    vv4[k] = reinterpret_cast<const float4*>(pos_v + col + c16)[k];
  }
  __syncthreads();  // barriers initialised
  pdl_launch_dependents();
  pdl_wait();

  // ---- 1. TMA: the tile's q rows (rows past T load as zeros), then every
  // key row of K -- the ring in slot order and the chunk -- in two 64-dim
  // halves each
  auto load_keys = [&](uint64_t* bar, const CUtensorMap* ring, int chunk_col) {
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(Tk) * kRowBytes);
    for (int hf = 0; hf < 2; ++hf) {
      tma_load_3d(sKV + hf * L.half, ring, bar, col + 64 * hf, 0, b);
      tma_load_3d(sKV + hf * L.half + L.c8 * 128, &map_ch, bar, chunk_col + 64 * hf, 0, b);
    }
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 2u * kQ * 128u);
    tma_load_3d(sQs, &map_q, &bars[0], col, i0, b);
    tma_load_3d(sQs + 2048, &map_q, &bars[0], col + 64, i0, b);
    load_keys(&bars[1], &map_kc, D + col);
  }

  // the new frames' attention input rows for the h ring (step 7), in
  // registers from here on: 16-byte chunk tid and tid + 128 of n_app x 16
  uint4 xr[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int e = tid + k * kThreads, r = e >> 4;
    xr[k] = ld16z(x + (static_cast<int64_t>(b) * T + src0 + (r < n_app ? r : 0)) * D + col +
                      (e & 15) * 8,
                  r < n_app);
  }

  // ---- 2. q+u and q+v in bf16 (the reference's bf16 adds, attention.rs:740-747);
  // rows past T are zeros
  const int nqr = min(kQ, T - i0);
  bool ok = mbar_wait(&bars[0], 0, err, kDevTimeoutLoad);
  {
    const int row = qrow;
    uint4 q[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    if (row < nqr && ok) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int ch = (c16 >> 3) + k;  // 0..15
        q[k] = *reinterpret_cast<const uint4*>(sQs + (ch >> 3) * 2048 + sw128_offset(row, ch & 7));
      }
    }
    uint32_t ou[8], ov[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 uu = uu4[k], vv = vv4[k];
      const uint32_t w0 = word(q[k >> 1], 2 * (k & 1)), w1 = word(q[k >> 1], 2 * (k & 1) + 1);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w0));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w1));
      ou[2 * k] = pack_bf16x2(a.x + uu.x, a.y + uu.y);
      ou[2 * k + 1] = pack_bf16x2(c.x + uu.z, c.y + uu.w);
      ov[2 * k] = pack_bf16x2(a.x + vv.x, a.y + vv.y);
      ov[2 * k + 1] = pack_bf16x2(c.x + vv.z, c.y + vv.w);
    }
    if (row >= nqr) {
#pragma unroll
      for (int k = 0; k < 8; ++k) ou[k] = ov[k] = 0u;
    }
    uint4* du = reinterpret_cast<uint4*>(sQu + row * kLd + c16);
    uint4* dv = reinterpret_cast<uint4*>(sQv + row * kLd + c16);
    du[0] = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    du[1] = make_uint4(ou[4], ou[5], ou[6], ou[7]);
    dv[0] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
    dv[1] = make_uint4(ov[4], ov[5], ov[6], ov[7]);
  }
  // a copy that never landed: the error is recorded, the CTA leaves
  if (!__syncthreads_and(ok)) return;

  // ---- 3. W = (q+v) P_win^T from global memory (the batch-shared P rows,
  // L2-resident) while K lands, then S = (q+u) K^T from shared memory;
  // 16-column tiles warp, warp + 4, ...
  const int r0 = T - kQ - i0;  // global P row of window row 0
  const int ns = L.nk / 16, nw = L.np / 16;
  // A fragments: 16 bytes of rows g and g + 8 for each 32-dim quarter s
  auto load_a = [&](const __nv_bfloat16* sA, uint4 (&ax)[4], uint4 (&ay)[4]) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      ax[s] = *reinterpret_cast<const uint4*>(sA + g * kLd + 32 * s + 8 * cq);
      ay[s] = *reinterpret_cast<const uint4*>(sA + (g + 8) * kLd + 32 * s + 8 * cq);
    }
  };
  // bb[hf][s]: 16 bytes of B row 16 n16 + 8 hf + g, head dims 32s + 8cq ..
  auto tile = [&](const uint4 (&ax)[4], const uint4 (&ay)[4], const uint4 (&bb)[2][4],
                  float* sOut, int ld, int n16) {
    float acc[2][4] = {};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const uint32_t a[4] = {word(ax[s], 2 * tt), word(ay[s], 2 * tt), word(ax[s], 2 * tt + 1),
                               word(ay[s], 2 * tt + 1)};
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          mma16816(acc[hf], a, word(bb[hf][s], 2 * tt), word(bb[hf][s], 2 * tt + 1));
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int n0 = n16 * 16 + hf * 8 + 2 * cq;
      *reinterpret_cast<float2*>(sOut + g * ld + n0) = make_float2(acc[hf][0], acc[hf][1]);
      *reinterpret_cast<float2*>(sOut + (g + 8) * ld + n0) = make_float2(acc[hf][2], acc[hf][3]);
    }
  };
  auto load_p = [&](int t, uint4 (&bb)[2][4]) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = r0 + t * 16 + hf * 8 + g;
      const bool in = r >= 0 && r < 2 * Tk - 1;
      const __nv_bfloat16* src = in ? p + static_cast<int64_t>(r) * D + col : p;
#pragma unroll
      for (int s = 0; s < 4; ++s) bb[hf][s] = ld16z(src + 32 * s + 8 * cq, in);
    }
  };
  {
    uint4 ax[4], ay[4], bc[2][4], bn[2][4];
    load_a(sQv, ax, ay);
    int t = warp;
    if (t < nw) load_p(t, bc);
    while (t < nw) {
      const int tn = t + kWarps;
      if (tn < nw) load_p(tn, bn);
      tile(ax, ay, bc, sW, L.ldw, t);
      if (tn >= nw) break;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int s = 0; s < 4; ++s) bc[hf][s] = bn[hf][s];
      t = tn;
    }
  }
  ok = mbar_wait(&bars[1], 0, err, kDevTimeoutLoad);
  if (ok) {
    uint4 ax[4], ay[4];
    load_a(sQu, ax, ay);
    for (int t = warp; t < ns; t += kWarps) {
      uint4 bb[2][4];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = krow(t * 16 + hf * 8 + g);
#pragma unroll
        for (int s = 0; s < 4; ++s) bb[hf][s] = *kv16(row, 4 * s + cq);
      }
      tile(ax, ay, bb, sS, L.lds, t);
    }
  }
  if (!__syncthreads_and(ok)) return;

  // ---- 4. the chunk's new K rows (keys C + src0 + r, still in the
  // buffer) into the ring (the chunk fits this CTA), then V into the buffer:
  // every read of K precedes the copies (the barrier above, then a proxy
  // fence)
  for (int e = tid; e < n_app * 16; e += kThreads) {
    const int r = e >> 4, ch = e & 15;
    *reinterpret_cast<uint4*>(kc_w + ring_row(r) + ch * 8) = *kv16(L.c8 + src0 + r, ch);
  }
  __syncthreads();
  if (tid == 0) {
    fence_proxy_async_smem();
    load_keys(&bars[2], &map_vc, 2 * D + col);
  }

  // ---- 5. softmax, the warp's 4 rows at once: row 4w + lane/8, keys
  // lane%8 + 8m, reductions over the row's 8 lanes
  {
    const float scale_log2 = 1.4426950408889634f * rsqrtf(static_cast<float>(kDh));
    const AttnContextDev none{0, -1, -1, 0};
    const int il = warp * (kQ / kWarps) + (lane >> 3), i = i0 + il, sub = lane & 7;
    int lo = 0, hi = 0;
    const bool any = i < T && key_interval(none, sm, i, Tk, lo, hi);
    constexpr int kPer = kKG * 4;  // keys per lane
    float sc[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
      const int j = sub + 8 * m;
      float v = -INFINITY;
      if (any && j >= lo && j < hi)  // hi <= Tk <= nk
        v = (sS[il * L.lds + j] + sW[il * L.ldw + (kQ - 1 - il + j)]) * scale_log2;
      sc[m] = v;
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int m = 0; m < kPer; ++m) {
      const int j = sub + 8 * m;
      const float pr = sc[m] == -INFINITY ? 0.f : fast_exp2(sc[m] - mx);
      sum += pr;
      if (j < L.nk) sPr[il * L.ldpr + j] = __float2bfloat16_rn(pr);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (sub == 0) sInv[il] = sum > 0.f ? 1.f / sum : 0.f;
  }
  ok = mbar_wait(&bars[2], 0, err, kDevTimeoutLoad);
  if (!__syncthreads_and(ok)) return;  // also: the probabilities are complete

  // ---- 6. O = P . V.  B operand of dim block blk (0..3): the 8x8 matrix
  // M[key r][2c + e] = V[key r][32w + 8c + 2blk + e], word blk of lane
  // (r, c); its transpose is the m16n8k16 B fragment, and the accumulator
  // column 2c + e is head dim 32w + 8c + 2blk + e.
  {
    const int nks = L.nk / 16;
    const int vcol = 32 * warp + 8 * cq;
    float acc[4][4] = {};
    // A fragment addresses: row (lane&7) + 8*((lane>>3)&1), column 8*(lane>>4)
    const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_col = (lane >> 4) * 8;
#pragma unroll 4
    for (int ks = 0; ks < nks; ++ks) {
      uint32_t af[4];
      ldsm_x4(sPr + a_row * L.ldpr + ks * 16 + a_col, af);
      const uint4 v0 = *kv16(krow(ks * 16 + g), vcol >> 3);
      const uint4 v1 = *kv16(krow(ks * 16 + 8 + g), vcol >> 3);
#pragma unroll
      for (int blk = 0; blk < 4; ++blk)
        mma16816(acc[blk], af, movm_t(word(v0, blk)), movm_t(word(v1, blk)));
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int il = g + 8 * hf, i = i0 + il;
      if (i >= T) continue;
      const float inv = sInv[il];
      *reinterpret_cast<uint4*>(out + (static_cast<int64_t>(b) * T + i) * D + col + vcol) =
          make_uint4(pack_bf16x2(acc[0][2 * hf] * inv, acc[0][2 * hf + 1] * inv),
                     pack_bf16x2(acc[1][2 * hf] * inv, acc[1][2 * hf + 1] * inv),
                     pack_bf16x2(acc[2][2 * hf] * inv, acc[2][2 * hf + 1] * inv),
                     pack_bf16x2(acc[3][2 * hf] * inv, acc[3][2 * hf + 1] * inv));
    }
  }

  // ---- 7. the new frames' V rows (from the buffer) and attention input
  // rows into the rings; the CTA's copies of the ring have landed
  for (int e = tid; e < n_app * 16; e += kThreads) {
    const int r = e >> 4, ch = e & 15;
    *reinterpret_cast<uint4*>(vc_w + ring_row(r) + ch * 8) = *kv16(L.c8 + src0 + r, ch);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int e = tid + k * kThreads, r = e >> 4;
    if (r < n_app) *reinterpret_cast<uint4*>(hc_w + ring_row(r) + (e & 15) * 8) = xr[k];
  }
}

template <int kKG>
cudaError_t launch_kg(dim3 grid, size_t smem, cudaStream_t stream,
                      const __nv_bfloat16* qkv, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                      __nv_bfloat16* hc, const __nv_bfloat16* x, int C, int head, int n_app,
                      int src0, const __nv_bfloat16* p, const float* u, const float* v,
                      StreamMaskDev sm, __nv_bfloat16* out, int B, int T, int D, int* err) {
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(stream_attn_kernel<kKG>, 227 * 1024, attr)) return e;
  // 128-byte swizzled boxes of 64 head dims: the ring's C rows of a session,
  // the tile's 16 q rows, the chunk's T rows
  CUtensorMap map_kc, map_vc, map_q, map_ch;
  const uint64_t rs = static_cast<uint64_t>(D) * 2, rs3 = 3 * rs;
  if (!make_tmap_3d(&map_kc, kc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, C, B, rs, rs * C, 64, C,
                    1, true) ||
      !make_tmap_3d(&map_vc, vc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, C, B, rs, rs * C, 64, C,
                    1, true) ||
      !make_tmap_3d(&map_q, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3ull * D, T, B, rs3,
                    rs3 * T, 64, kQ, 1, true) ||
      !make_tmap_3d(&map_ch, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3ull * D, T, B, rs3,
                    rs3 * T, 64, T, 1, true))
    return cudaErrorInvalidValue;
  return launch_pdl(stream_attn_kernel<kKG>, grid, dim3(kThreads), smem, stream, map_kc, map_vc,
                    map_q, map_ch, const_cast<__nv_bfloat16*>(kc), const_cast<__nv_bfloat16*>(vc),
                    hc, x, C, head, n_app, src0, p, u, v, sm, out, T, D, err);
}

}  // namespace

bool stream_attn_supported(int C, int T, int D, int H) {
  return D == H * kDh && C + T <= kMaxKeys && C > 0 && T > 0 &&
         stream_smem(C, T).bytes <= 227 * 1024;
}

cudaError_t launch_relpos_attn_stream_mma(const __nv_bfloat16* qkv, const __nv_bfloat16* kc,
                                          const __nv_bfloat16* vc, __nv_bfloat16* hc,
                                          const __nv_bfloat16* x, int C, int head, int n_app,
                                          int src0, const __nv_bfloat16* p, const float* u,
                                          const float* v, StreamMaskDev sm, __nv_bfloat16* out,
                                          int B, int T, int D, int H, int* err,
                                          cudaStream_t stream) {
  if (!stream_attn_supported(C, T, D, H) || B <= 0 || B > 65535) return cudaErrorInvalidValue;
  // tensor maps need 16-byte aligned bases
  if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(kc) |
        reinterpret_cast<uintptr_t>(vc)) & 15) != 0)
    return cudaErrorMisalignedAddress;
  const int nq = (T + kQ - 1) / kQ;
  if (n_app > 0 && (nq != 1 || src0 < 0 || src0 + n_app > T || n_app > C || n_app > kQ))
    return cudaErrorInvalidValue;
  const StreamSmem L = stream_smem(C, T);
  const dim3 grid(nq, H, B);
  switch (L.nk / 32 + (L.nk % 32 != 0)) {
#define NRP_KG(k)                                                                              \
  case k:                                                                                      \
    return launch_kg<k>(grid, L.bytes, stream, qkv, kc, vc, hc, x, C, head, n_app, src0, p, u, \
                        v, sm, out, B, T, D, err);
    NRP_KG(1) NRP_KG(2) NRP_KG(3) NRP_KG(4) NRP_KG(5) NRP_KG(6) NRP_KG(7) NRP_KG(8)
#undef NRP_KG
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace nrp
