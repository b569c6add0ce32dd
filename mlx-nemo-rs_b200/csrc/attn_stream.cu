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
// head), so one CTA of 8 warps takes 16 query rows of one (session, head):
//   1. cp.async stages q, K and the 15+Tk-row P window (one group) and V
//      (a second group, still landing while the scores are computed);
//   2. mma.sync m16n8k16 (bf16 -> f32): S = (q+u) K^T and
//      W = (q+v) P_win^T, 16-column tiles dealt to the warps, into shared
//      memory;
//   3. softmax per row: score(i, j) = (S[i][j] + W[i][15 - i + j]) / sqrt(dh)
//      -- rel_shift is the skewed read of W --, masked by the streaming
//      mask (create_attention_mask, conformer.rs:97-221), bf16
//      probabilities back to shared memory;
//   4. mma.sync O = P . V (V through ldmatrix.trans), normalised, stored;
//   5. when the chunk fits one CTA, the chunk's first n_app frames of K, V
//      (from shared memory) and of the attention input x are written into
//      the ring for this head's columns -- the sliding window update of
//      661-684 -- after every read of the ring by this CTA; no other CTA
//      touches these columns.
// The kernel is HBM-bound: it reads K and V once (22 MB per layer at
// config 2) and P from L2.
#include <cuda_bf16.h>

#include "gemm.h"
#include "masks.cuh"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kQ = 16;        // query rows per CTA
constexpr int kDh = 128;
constexpr int kLd = kDh + 8;  // shared row stride in bf16 (272 B: conflict-free ldmatrix)
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxKeys = 256;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

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
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
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
  int nk, np;  // key rows (Tk rounded up to 16), P window rows
  size_t off_qu, off_qv, off_k, off_v, off_p, off_s, off_w, off_pr, off_inv, bytes;
};

__host__ __device__ inline StreamSmem stream_smem(int Tk) {
  StreamSmem m;
  m.nk = (Tk + 15) / 16 * 16;
  m.np = (Tk + kQ - 1 + 15) / 16 * 16;
  size_t o = 0;
  m.off_qu = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_qv = o; o += static_cast<size_t>(kQ) * kLd * 2;
  m.off_k = o; o += static_cast<size_t>(m.nk) * kLd * 2;
  m.off_v = o; o += static_cast<size_t>(m.nk) * kLd * 2;
  m.off_p = o; o += static_cast<size_t>(m.np) * kLd * 2;
  m.off_s = o; o += static_cast<size_t>(kQ) * m.nk * 4;
  m.off_w = o; o += static_cast<size_t>(kQ) * m.np * 4;
  m.off_pr = o; o += static_cast<size_t>(kQ) * (m.nk + 8) * 2;
  m.off_inv = o; o += kQ * 4;
  m.bytes = o;
  return m;
}

__global__ void __launch_bounds__(kThreads)
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
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + L.off_k);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(smem + L.off_v);
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem + L.off_p);
  float* sS = reinterpret_cast<float*>(smem + L.off_s);
  float* sW = reinterpret_cast<float*>(smem + L.off_w);
  __nv_bfloat16* sPr = reinterpret_cast<__nv_bfloat16*>(smem + L.off_pr);
  float* sInv = reinterpret_cast<float*>(smem + L.off_inv);
  const int ldpr = L.nk + 8;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = blockIdx.x * kQ, h = blockIdx.y, b = blockIdx.z;
  pdl_launch_dependents();
  pdl_wait();
  const int col = h * kDh;
  const int64_t ld3 = 3ll * D;
  const int r0 = T - kQ - i0;  // global P row of window row 0

  // ---- 1. stage q, K, P (group 0) and V (group 1), 16-byte chunks, 16
  // threads per row; rows outside the data are zeros
  const int ch = tid & 15;
  auto stage = [&](__nv_bfloat16* dst, const __nv_bfloat16* src) {
    if (src)
      cp_async16(dst + ch * 8, src + ch * 8);
    else
      *reinterpret_cast<uint4*>(dst + ch * 8) = make_uint4(0u, 0u, 0u, 0u);
  };
  // key row j: ring slot head + j (mod C) for the cache, the chunk after it
  auto key_src = [&](int j, int off, const __nv_bfloat16* ring) -> const __nv_bfloat16* {
    if (j < C) {
      int slot = head + j;
      slot = slot >= C ? slot - C : slot;
      return ring + (static_cast<int64_t>(b) * C + slot) * D + col;
    }
    if (j < Tk) return qkv + (static_cast<int64_t>(b) * T + (j - C)) * ld3 + off + col;
    return nullptr;
  };
  for (int row = tid >> 4; row < kQ + L.nk + L.np; row += kThreads / 16) {
    if (row < kQ) {
      const int i = i0 + row;
      stage(sQu + row * kLd, i < T ? qkv + (static_cast<int64_t>(b) * T + i) * ld3 + col : nullptr);
    } else if (row < kQ + L.nk) {
      const int j = row - kQ;
      stage(sK + j * kLd, key_src(j, D, kc));
    } else {
      const int w = row - kQ - L.nk, r = r0 + w;
      stage(sP + w * kLd, (r >= 0 && r < 2 * Tk - 1) ? p + static_cast<int64_t>(r) * D + col
                                                      : nullptr);
    }
  }
  cp_async_commit();
  for (int j = tid >> 4; j < L.nk; j += kThreads / 16) stage(sV + j * kLd, key_src(j, 2 * D, vc));
  cp_async_commit();
  cp_async_wait<1>();  // q, K, P have landed (V may still be in flight)
  __syncthreads();

  // q+u and q+v in bf16 (the reference's bf16 adds, attention.rs:740-747)
  for (int e = tid; e < kQ * kDh / 2; e += kThreads) {
    const int row = e / (kDh / 2), d = (e % (kDh / 2)) * 2;
    const float2 q = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(sQu + row * kLd + d));
    const float2 u2 = *reinterpret_cast<const float2*>(pos_u + col + d);
    const float2 v2 = *reinterpret_cast<const float2*>(pos_v + col + d);
    *reinterpret_cast<uint32_t*>(sQv + row * kLd + d) = pack_bf16x2(q.x + v2.x, q.y + v2.y);
    *reinterpret_cast<uint32_t*>(sQu + row * kLd + d) = pack_bf16x2(q.x + u2.x, q.y + u2.y);
  }
  __syncthreads();

  const int g = lane >> 2, cq = lane & 3;
  // A fragment addresses: row (lane&7) + 8*((lane>>3)&1), column 8*(lane>>4)
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_col = (lane >> 4) * 8;
  // B (non-transposed, [n][k] rows): n = (lane&7) + 8*(lane>>4), k = 8*((lane>>3)&1)
  const int b_row = (lane & 7) + (lane >> 4) * 8, b_col = ((lane >> 3) & 1) * 8;

  // ---- 2. S = (q+u) K^T and W = (q+v) P_win^T: 16-column tiles of both,
  // dealt round-robin to the warps
  {
    const int ns = L.nk / 16, nw = L.np / 16;
    int have = -1;  // which A operand af holds: 0 = q+u, 1 = q+v
    uint32_t af[8][4];
    for (int t = warp; t < ns + nw; t += kWarps) {
      const bool isw = t >= ns;
      const int n16 = isw ? t - ns : t;
      const __nv_bfloat16* sA = isw ? sQv : sQu;
      const __nv_bfloat16* sB = isw ? sP : sK;
      float* sOut = isw ? sW : sS;
      const int nrows = isw ? L.np : L.nk;
      if (have != static_cast<int>(isw)) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) ldsm_x4(sA + a_row * kLd + ks * 16 + a_col, af[ks]);
        have = isw;
      }
      float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t bf[4];
        ldsm_x4(sB + (n16 * 16 + b_row) * kLd + ks * 16 + b_col, bf);
        mma16816(acc0, af[ks], bf[0], bf[1]);
        mma16816(acc1, af[ks], bf[2], bf[3]);
      }
      const int n0 = n16 * 16 + 2 * cq;
      *reinterpret_cast<float2*>(sOut + g * nrows + n0) = make_float2(acc0[0], acc0[1]);
      *reinterpret_cast<float2*>(sOut + (g + 8) * nrows + n0) = make_float2(acc0[2], acc0[3]);
      *reinterpret_cast<float2*>(sOut + g * nrows + n0 + 8) = make_float2(acc1[0], acc1[1]);
      *reinterpret_cast<float2*>(sOut + (g + 8) * nrows + n0 + 8) = make_float2(acc1[2], acc1[3]);
    }
  }
  __syncthreads();

  // ---- 3. softmax per row (warp w: rows 2w, 2w+1)
  const float scale_log2 = 1.4426950408889634f * rsqrtf(static_cast<float>(kDh));
  const AttnContextDev none{0, -1, -1, 0};
  for (int rr = 0; rr < kQ / kWarps; ++rr) {
    const int il = warp * (kQ / kWarps) + rr, i = i0 + il;
    int lo = 0, hi = 0;
    const bool any = i < T && key_interval(none, sm, i, Tk, lo, hi);
    float sc[kMaxKeys / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int m = 0; m < kMaxKeys / 32; ++m) {
      const int j = lane + 32 * m;
      float v = -INFINITY;
      if (j < L.nk && any && j >= lo && j < hi)
        v = (sS[il * L.nk + j] + sW[il * L.np + (kQ - 1 - il + j)]) * scale_log2;
      sc[m] = v;
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxKeys / 32; ++m) {
      const int j = lane + 32 * m;
      const float pr = sc[m] == -INFINITY ? 0.f : fast_exp2(sc[m] - mx);
      sum += pr;
      if (j < L.nk) sPr[il * ldpr + j] = __float2bfloat16_rn(pr);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) sInv[il] = sum > 0.f ? 1.f / sum : 0.f;
  }
  cp_async_wait<0>();  // V
  __syncthreads();

  // ---- 4. O = P . V (warp w: head dims 16w .. 16w+15)
  {
    float acc[2][4] = {};
    // V as the [k=key][n=dim] B operand, transposed by ldmatrix: key row
    // (lane&7) + 8*((lane>>3)&1), dim column 8*(lane>>4)
    const int v_row = (lane & 7) + ((lane >> 3) & 1) * 8, v_col = (lane >> 4) * 8;
    for (int ks = 0; ks < L.nk / 16; ++ks) {
      uint32_t af[4];
      ldsm_x4(sPr + a_row * ldpr + ks * 16 + a_col, af);
      uint32_t bf[4];
      ldsm_x4_t(sV + (ks * 16 + v_row) * kLd + warp * 16 + v_col, bf);
      mma16816(acc[0], af, bf[0], bf[1]);
      mma16816(acc[1], af, bf[2], bf[3]);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int il = g + 8 * half, i = i0 + il;
      if (i >= T) continue;
      const float inv = sInv[il];
      __nv_bfloat16* orow = out + (static_cast<int64_t>(b) * T + i) * D + col + warp * 16;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        *reinterpret_cast<uint32_t*>(orow + nt * 8 + 2 * cq) =
            pack_bf16x2(acc[nt][2 * half] * inv, acc[nt][2 * half + 1] * inv);
    }
  }

  // ---- 5. ring update for this head's columns (the chunk fits this CTA):
  // 16 threads per frame row; K and V from shared memory, h from x
  if (n_app > 0) {
    for (int r = tid >> 4; r < n_app; r += kThreads / 16) {
      int slot = head + r;
      slot = slot >= C ? slot - C : slot;
      const int64_t dst = (static_cast<int64_t>(b) * C + slot) * D + col + ch * 8;
      const int j = C + src0 + r;  // key row of new frame src0 + r
      *reinterpret_cast<uint4*>(kc_w + dst) = *reinterpret_cast<const uint4*>(sK + j * kLd + ch * 8);
      *reinterpret_cast<uint4*>(vc_w + dst) = *reinterpret_cast<const uint4*>(sV + j * kLd + ch * 8);
      *reinterpret_cast<uint4*>(hc_w + dst) = *reinterpret_cast<const uint4*>(
          x + (static_cast<int64_t>(b) * T + src0 + r) * D + col + ch * 8);
    }
  }
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
  if (n_app > 0 && (nq != 1 || src0 < 0 || src0 + n_app > T || n_app > C))
    return cudaErrorInvalidValue;
  const size_t smem = stream_smem(C + T).bytes;
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(stream_attn_kernel, 227 * 1024, attr)) return e;
  const dim3 grid(nq, H, B);
  return launch_pdl(stream_attn_kernel, grid, dim3(kThreads), smem, stream, qkv, kc, vc,
                    const_cast<__nv_bfloat16*>(kc), const_cast<__nv_bfloat16*>(vc), hc, x, C, head,
                    n_app, src0, p, u, v, sm, out, T, D);
}

}  // namespace nrp
