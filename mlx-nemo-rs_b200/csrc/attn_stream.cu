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
// head) and K, V are read once, so nothing is staged in shared memory: one
// CTA of 4 warps takes 16 query rows of one (session, head) and every
// operand goes from global memory (HBM or L2) straight into MMA fragments.
//   0. before waiting on the projection kernel, the session's cached K and V
//      rows of this head are prefetched into L2 (they were written by an
//      earlier launch; the prefetch overlaps the projection GEMM) and the
//      positional biases are loaded;
//   1. the new frames' K, V and x rows for the ring update go to shared
//      memory by cp.async; q+u and q+v are rounded to bf16 into shared memory;
//   2. mma.sync m16n8k16 (bf16 -> f32): S = (q+u) K^T and
//      W = (q+v) P_win^T over 16-column tiles dealt to the warps, B operands
//      loaded as 16-byte rows with a double-buffered register pipeline.  The
//      128-dim contraction runs in a permuted order (k-step 2s+t, lane
//      column 2c+e <-> head dim 32s+8c+4t+e, and +2 for the upper half), the
//      same for both operands, so one 16-byte load of a row gives a lane its
//      fragments of two k-steps.  Rows outside the data are predicated
//      loads over zeroed registers, so no instruction waits on a load
//      before its MMA;
//   3. each warp's V rows (32 head dims) are loaded into registers, up to
//      kVDepth k-steps ahead, before the softmax;
//   4. softmax, four rows per warp at once (8 lanes a row):
//      score(i, j) = (S[i][j] + W[i][15 - i + j]) / sqrt(dh) -- rel_shift is
//      the skewed read of W --, masked by the streaming mask
//      (create_attention_mask, conformer.rs:97-221), bf16 probabilities;
//   5. O = P . V with V transposed in registers by movmatrix (8x8 blocks of
//      (key, dim-pair) words), so each lane ends with 8 contiguous output
//      dims of two rows: one 16-byte store each;
//   6. when the chunk fits one CTA, the staged frames are written into the
//      ring for this head's columns -- the sliding window update of 661-684
//      -- after every read of the ring by this CTA; no other CTA touches
//      these columns.
// Shared memory is ~38 KB per CTA (Tk = 84), so four CTAs share an SM and
// config 2's 512 (session, head) items run as one wave; the kernel is bound
// by HBM (K and V, 22 MB per layer at config 2) and load latency.
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
constexpr int kVDepth = 8;    // V k-steps (16 keys each) held in registers ahead of their MMAs

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

// One 256-byte row (two 128-byte lines) into L2.
__device__ __forceinline__ void prefetch_row_l2(const __nv_bfloat16* p) {
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p));
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p + 64));
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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
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
  int lds, ldw;   // f32 row strides of S and W (+8: two-wavefront float2 stores)
  int ldpr;       // bf16 row stride of the probabilities
  size_t off_qu, off_qv, off_s, off_w, off_pr, off_inv, off_app, bytes;
};

__host__ __device__ inline StreamSmem stream_smem(int Tk) {
  StreamSmem m;
  m.nk = (Tk + 15) / 16 * 16;
  m.np = (Tk + kQ - 1 + 15) / 16 * 16;
  m.lds = m.nk + 8;
  m.ldw = m.np + 8;
  m.ldpr = m.nk + 8;
  size_t o = 0;
  m.off_qu = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_qv = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_s = o; o += static_cast<size_t>(kQ) * m.lds * 4;
  m.off_w = o; o += static_cast<size_t>(kQ) * m.ldw * 4;
  m.off_pr = o; o += static_cast<size_t>(kQ) * m.ldpr * 2;
  m.off_inv = o; o += kQ * 4;
  m.off_app = o; o += static_cast<size_t>(3) * kQ * kDh * 2;  // new frames' K, V, x rows
  m.bytes = o;
  return m;
}

// kKG = ceil(nk / 32): 32-key groups a lane walks in the softmax.
template <int kKG>
__global__ void __launch_bounds__(kThreads, 4)
    stream_attn_kernel(const __nv_bfloat16* __restrict__ qkv,  // [B][T][3D]
                       const __nv_bfloat16* kc, const __nv_bfloat16* vc,  // rings [B][C][D]
                       __nv_bfloat16* kc_w, __nv_bfloat16* vc_w, __nv_bfloat16* hc_w,
                       const __nv_bfloat16* __restrict__ x,  // attention input [B][T][D]
                       int C, int head, int n_app, int src0,
                       const __nv_bfloat16* __restrict__ p,  // [2Tk-1][D]
                       const float* __restrict__ pos_u, const float* __restrict__ pos_v,
                       StreamMaskDev sm, __nv_bfloat16* __restrict__ out, int T, int D) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int Tk = C + T;
  const StreamSmem L = stream_smem(Tk);
  __nv_bfloat16* sQu = reinterpret_cast<__nv_bfloat16*>(smem + L.off_qu);
  __nv_bfloat16* sQv = reinterpret_cast<__nv_bfloat16*>(smem + L.off_qv);
  float* sS = reinterpret_cast<float*>(smem + L.off_s);
  float* sW = reinterpret_cast<float*>(smem + L.off_w);
  __nv_bfloat16* sPr = reinterpret_cast<__nv_bfloat16*>(smem + L.off_pr);
  float* sInv = reinterpret_cast<float*>(smem + L.off_inv);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, cq = lane & 3;
  const int i0 = blockIdx.x * kQ, h = blockIdx.y, b = blockIdx.z;
  const int col = h * kDh;
  const int64_t ld3 = 3ll * D;

  // key row j of K (off = D) or V (off = 2D): ring slot head + j (mod C) for
  // the cache, the chunk after it, nothing past Tk
  auto key_src = [&](int j, int off, const __nv_bfloat16* ring) -> const __nv_bfloat16* {
    if (j < C) {
      int slot = head + j;
      slot = slot >= C ? slot - C : slot;
      return ring + (static_cast<int64_t>(b) * C + slot) * D + col;
    }
    if (j < Tk) return qkv + (static_cast<int64_t>(b) * T + (j - C)) * ld3 + off + col;
    return nullptr;
  };

  // ---- 0. cached K and V rows into L2 while the projection still runs;
  // the positional biases (weights) into registers
  for (int r = tid; r < 2 * C; r += kThreads) {
    const int j = r < C ? r : r - C;
    prefetch_row_l2(key_src(j, 0, r < C ? kc : vc));
  }
  const int qrow = tid >> 3, c16 = (tid & 7) * 16;  // phase 1: row tid/8, dims 16 (tid%8) ..
  float4 uu4[4], vv4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uu4[k] = reinterpret_cast<const float4*>(pos_u + col + c16)[k];
    vv4[k] = reinterpret_cast<const float4*>(pos_v + col + c16)[k];
  }
  pdl_launch_dependents();
  pdl_wait();

  // the new frames' K, V and x rows for the ring update (step 6), landing
  // in shared memory while the attention runs
  __nv_bfloat16* sApp = reinterpret_cast<__nv_bfloat16*>(smem + L.off_app);
  for (int e = tid; e < 3 * n_app * 16; e += kThreads) {
    const int a = e / (n_app * 16), r = (e / 16) % n_app, ch = e & 15;
    const int64_t fr = static_cast<int64_t>(b) * T + src0 + r;
    const __nv_bfloat16* src =
        a < 2 ? qkv + fr * ld3 + (a + 1) * D + col + ch * 8 : x + fr * D + col + ch * 8;
    cp_async16(sApp + (a * kQ + r) * kDh + ch * 8, src);
  }

  // ---- 1. q+u and q+v in bf16 (the reference's bf16 adds, attention.rs:740-747)
  {
    const int row = qrow, i = i0 + row;
    const __nv_bfloat16* src =
        qkv + (static_cast<int64_t>(b) * T + (i < T ? i : 0)) * ld3 + col + c16;
    const uint4 q[2] = {ld16z(src, i < T), ld16z(src + 8, i < T)};
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
    uint4* du = reinterpret_cast<uint4*>(sQu + row * kLd + c16);
    uint4* dv = reinterpret_cast<uint4*>(sQv + row * kLd + c16);
    du[0] = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    du[1] = make_uint4(ou[4], ou[5], ou[6], ou[7]);
    dv[0] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
    dv[1] = make_uint4(ov[4], ov[5], ov[6], ov[7]);
  }
  __syncthreads();

  // ---- 2. S = (q+u) K^T (tiles 0..ns-1) and W = (q+v) P_win^T (the rest)
  const int r0 = T - kQ - i0;  // global P row of window row 0
  const int ns = L.nk / 16, ntiles = ns + L.np / 16;
  // B rows n16*16 + 8*hf + g, this lane's 16-byte chunk of each 32-dim
  // quarter s: head dims 32s + 8cq .. +7
  auto load_b = [&](int t, uint4 (&bb)[2][4]) {
    const bool isw = t >= ns;
    const int n16 = isw ? t - ns : t;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int n = n16 * 16 + hf * 8 + g;
      const __nv_bfloat16* src;
      if (isw) {
        const int r = r0 + n;
        src = (r >= 0 && r < 2 * Tk - 1) ? p + static_cast<int64_t>(r) * D + col : nullptr;
      } else {
        src = key_src(n, D, kc);
      }
      const bool ok = src != nullptr;
      if (!ok) src = p;
#pragma unroll
      for (int s = 0; s < 4; ++s) bb[hf][s] = ld16z(src + 32 * s + 8 * cq, ok);
    }
  };
  {
    uint4 bc[2][4], bn[2][4], ax[4], ay[4];
    int have = -1;  // which A operand ax/ay hold: 0 = q+u, 1 = q+v
    int t = warp;
    if (t < ntiles) load_b(t, bc);
    while (t < ntiles) {
      const int tn = t + kWarps;
      if (tn < ntiles) load_b(tn, bn);
      const bool isw = t >= ns;
      if (have != static_cast<int>(isw)) {
        const __nv_bfloat16* sA = isw ? sQv : sQu;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          ax[s] = *reinterpret_cast<const uint4*>(sA + g * kLd + 32 * s + 8 * cq);
          ay[s] = *reinterpret_cast<const uint4*>(sA + (g + 8) * kLd + 32 * s + 8 * cq);
        }
        have = isw;
      }
      float acc[2][4] = {};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
          const uint32_t a[4] = {word(ax[s], 2 * tt), word(ay[s], 2 * tt), word(ax[s], 2 * tt + 1),
                                 word(ay[s], 2 * tt + 1)};
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
            mma16816(acc[hf], a, word(bc[hf][s], 2 * tt), word(bc[hf][s], 2 * tt + 1));
        }
      }
      const int n16 = isw ? t - ns : t;
      float* sOut = isw ? sW : sS;
      const int ld = isw ? L.ldw : L.lds;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int n0 = n16 * 16 + hf * 8 + 2 * cq;
        *reinterpret_cast<float2*>(sOut + g * ld + n0) = make_float2(acc[hf][0], acc[hf][1]);
        *reinterpret_cast<float2*>(sOut + (g + 8) * ld + n0) = make_float2(acc[hf][2], acc[hf][3]);
      }
      if (tn >= ntiles) break;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int s = 0; s < 4; ++s) bc[hf][s] = bn[hf][s];
      t = tn;
    }
  }
  __syncthreads();

  // ---- 3. V rows of this warp's head dims 32w .. 32w+31 (lane: 8 of them),
  // key rows 16ks + 8hf + g, kVDepth k-steps ahead
  const int nks = L.nk / 16;
  const int vcol = 32 * warp + 8 * cq;
  uint4 vb[kVDepth][2];
  auto load_v = [&](int ks, uint4 (&dst)[2]) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const __nv_bfloat16* src = key_src(ks * 16 + hf * 8 + g, 2 * D, vc);
      dst[hf] = ld16z((src ? src : p) + vcol, src != nullptr);
    }
  };
#pragma unroll
  for (int k = 0; k < kVDepth; ++k)
    if (k < nks) load_v(k, vb[k]);

  // ---- 4. softmax, the warp's 4 rows at once: row 4w + lane/8, keys
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
  __syncthreads();

  // ---- 5. O = P . V.  B operand of dim block blk (0..3): the 8x8 matrix
  // M[key r][2c + e] = V[key r][32w + 8c + 2blk + e], word blk of lane
  // (r, c); its transpose is the m16n8k16 B fragment, and the accumulator
  // column 2c + e is head dim 32w + 8c + 2blk + e.
  {
    float acc[4][4] = {};
    // A fragment addresses: row (lane&7) + 8*((lane>>3)&1), column 8*(lane>>4)
    const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_col = (lane >> 4) * 8;
    for (int kb = 0; kb < nks; kb += kVDepth) {
#pragma unroll
      for (int k = 0; k < kVDepth; ++k) {
        const int ks = kb + k;
        if (ks < nks) {
          uint32_t af[4];
          ldsm_x4(sPr + a_row * L.ldpr + ks * 16 + a_col, af);
#pragma unroll
          for (int blk = 0; blk < 4; ++blk)
            mma16816(acc[blk], af, movm_t(word(vb[k][0], blk)), movm_t(word(vb[k][1], blk)));
          if (ks + kVDepth < nks) load_v(ks + kVDepth, vb[k]);
        }
      }
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

  // ---- 6. ring update for this head's columns (the chunk fits this CTA),
  // after every warp's last read of the ring: 16 threads per frame row
  if (n_app > 0) {
    cp_async_wait_all();
    __syncthreads();
    const int ch = tid & 15;
    for (int r = tid >> 4; r < n_app; r += kThreads / 16) {
      int slot = head + r;
      slot = slot >= C ? slot - C : slot;
      const int64_t dst = (static_cast<int64_t>(b) * C + slot) * D + col + ch * 8;
      *reinterpret_cast<uint4*>(kc_w + dst) =
          *reinterpret_cast<const uint4*>(sApp + (0 * kQ + r) * kDh + ch * 8);
      *reinterpret_cast<uint4*>(vc_w + dst) =
          *reinterpret_cast<const uint4*>(sApp + (1 * kQ + r) * kDh + ch * 8);
      *reinterpret_cast<uint4*>(hc_w + dst) =
          *reinterpret_cast<const uint4*>(sApp + (2 * kQ + r) * kDh + ch * 8);
    }
  }
}

template <int kKG>
cudaError_t launch_kg(dim3 grid, size_t smem, cudaStream_t stream,
                      const __nv_bfloat16* qkv, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                      __nv_bfloat16* hc, const __nv_bfloat16* x, int C, int head, int n_app,
                      int src0, const __nv_bfloat16* p, const float* u, const float* v,
                      StreamMaskDev sm, __nv_bfloat16* out, int T, int D) {
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(stream_attn_kernel<kKG>, 227 * 1024, attr)) return e;
  return launch_pdl(stream_attn_kernel<kKG>, grid, dim3(kThreads), smem, stream, qkv, kc, vc,
                    const_cast<__nv_bfloat16*>(kc), const_cast<__nv_bfloat16*>(vc), hc, x, C, head,
                    n_app, src0, p, u, v, sm, out, T, D);
}

}  // namespace

bool stream_attn_supported(int C, int T, int D, int H) {
  return D == H * kDh && C + T <= kMaxKeys && C > 0 && T > 0 &&
         stream_smem(C + T).bytes <= 227 * 1024;
}

cudaError_t launch_relpos_attn_stream_mma(const __nv_bfloat16* qkv, const __nv_bfloat16* kc,
                                          const __nv_bfloat16* vc, __nv_bfloat16* hc,
                                          const __nv_bfloat16* x, int C, int head, int n_app,
                                          int src0, const __nv_bfloat16* p, const float* u,
                                          const float* v, StreamMaskDev sm, __nv_bfloat16* out,
                                          int B, int T, int D, int H, cudaStream_t stream) {
  if (!stream_attn_supported(C, T, D, H) || B <= 0 || B > 65535) return cudaErrorInvalidValue;
  const int nq = (T + kQ - 1) / kQ;
  if (n_app > 0 && (nq != 1 || src0 < 0 || src0 + n_app > T || n_app > C || n_app > kQ))
    return cudaErrorInvalidValue;
  const StreamSmem L = stream_smem(C + T);
  const dim3 grid(nq, H, B);
  switch (L.nk / 32 + (L.nk % 32 != 0)) {
#define NRP_KG(k)                                                                              \
  case k:                                                                                      \
    return launch_kg<k>(grid, L.bytes, stream, qkv, kc, vc, hc, x, C, head, n_app, src0, p, u, \
                        v, sm, out, T, D);
    NRP_KG(1) NRP_KG(2) NRP_KG(3) NRP_KG(4) NRP_KG(5) NRP_KG(6) NRP_KG(7) NRP_KG(8)
#undef NRP_KG
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace nrp
