// attn_simt.cu -- relative-position attention on CUDA cores, fp32 math.
//
// Serves modules whose dtype is f32 (the reference's default f32 graph,
// attention.rs:458-573 offline and 606-816 streaming; 1e-4 parity needs
// FFMA, not TF32 tensor cores) and any head_dim <= 128, plus the streaming
// form for bf16 storage.  Offline with head_dim 128, the block-staged kernel
// below (relpos_attn_f32_blocked_kernel) runs.  Otherwise one warp per query
// row: lanes score 32 keys at a
// time ((q+u).k_j + (q+v).p_r with r = Tq-1-i+j, the rel_shift identity of
// attention.rs:1248-1282), keep an online softmax, and accumulate P.V with
// each lane owning dims lane, lane+32, lane+64, lane+96.
//
// Keys j < C come from a ring cache (slot (head + j) mod C) and keys j >= C
// from the chunk's new projections, so the streaming cache never moves.
#include <math.h>

#include "gemm.h"
#include "masks.cuh"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxDh = 128;

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// Four consecutive elements as f32 (one 16- or 8-byte load); p aligned.
template <typename T>
__device__ __forceinline__ void ld4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float (&v)[4]) {
  const float4 f = *reinterpret_cast<const float4*>(p);
  v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
}
template <>
__device__ __forceinline__ void ld4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
}

template <typename T>
__device__ __forceinline__ void st(T* p, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
    relpos_attn_simt_kernel(const T* __restrict__ q, int ldq, const T* __restrict__ knew,
                            int ldk, const T* __restrict__ vnew, int ldv,
                            const T* __restrict__ kc, const T* __restrict__ vc, int C, int head,
                            const T* __restrict__ p, const float* __restrict__ pu,
                            const float* __restrict__ pv, const int32_t* __restrict__ key_len,
                            AttnContextDev ctx, StreamMaskDev sm, T* __restrict__ out, int Tq,
                            int Tk, int D, int H) {
  __shared__ float s_qu[kWarps][kMaxDh];
  __shared__ float s_qv[kWarps][kMaxDh];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int i = blockIdx.x * kWarps + warp;
  const int dh = D / H;
  if (i >= Tq) return;
  const T* qi = q + (static_cast<size_t>(b) * Tq + i) * ldq + h * dh;
  for (int d = lane; d < dh; d += 32) {
    const float x = ld(qi + d);
    s_qu[warp][d] = x + pu[h * dh + d];
    s_qv[warp][d] = x + pv[h * dh + d];
  }
  __syncwarp();
  int kend = Tk;
  if (key_len) kend = min(Tk, max(key_len[b], 1));
  int lo, hi;
  const bool any = key_interval(ctx, sm, i, kend, lo, hi);
  const float scale = rsqrtf(static_cast<float>(dh));
  float m = -INFINITY, l = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  const int Tn = Tk - C;
  if (any) {
    for (int jb = lo; jb < hi; jb += 32) {
      const int j = jb + lane;
      float sc = -INFINITY;
      if (j < hi) {
        const T* kj = j < C ? kc + (static_cast<size_t>(b) * C + (head + j) % C) * D + h * dh
                            : knew + (static_cast<size_t>(b) * Tn + (j - C)) * ldk + h * dh;
        const T* pr = p + static_cast<size_t>(Tq - 1 - i + j) * D + h * dh;
        float a = 0.f, c = 0.f;
        // each lane walks its own key row: 4 elements per load when the rows
        // allow (one L1 request per lane instead of four), the same
        // ascending-d fmaf chain either way
        constexpr uintptr_t kAl = sizeof(T) * 4 - 1;
        if ((dh & 3) == 0 && ((reinterpret_cast<uintptr_t>(kj) | reinterpret_cast<uintptr_t>(pr)) & kAl) == 0) {
          for (int d = 0; d < dh; d += 4) {
            float kv[4], pv4[4];
            ld4(kj + d, kv);
            ld4(pr + d, pv4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              a = fmaf(s_qu[warp][d + e], kv[e], a);
              c = fmaf(s_qv[warp][d + e], pv4[e], c);
            }
          }
        } else {
          for (int d = 0; d < dh; ++d) {
            a = fmaf(s_qu[warp][d], ld(kj + d), a);
            c = fmaf(s_qv[warp][d], ld(pr + d), c);
          }
        }
        sc = (a + c) * scale;
      }
      float cm = sc;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
      const float mn = fmaxf(m, cm);
      const float alpha = (m == -INFINITY) ? 0.f : expf(m - mn);
      const float pj = (sc == -INFINITY) ? 0.f : expf(sc - mn);
      float ps = pj;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l = l * alpha + ps;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] *= alpha;
      const int nk = min(32, hi - jb);
      for (int kk = 0; kk < nk; ++kk) {
        const float w = __shfl_sync(0xffffffffu, pj, kk);
        const int jj = jb + kk;
        const T* vj = jj < C ? vc + (static_cast<size_t>(b) * C + (head + jj) % C) * D + h * dh
                             : vnew + (static_cast<size_t>(b) * Tn + (jj - C)) * ldv + h * dh;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = lane + 32 * e;
          if (d < dh) o[e] = fmaf(w, ld(vj + d), o[e]);
        }
      }
      m = mn;
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* oi = out + (static_cast<size_t>(b) * Tq + i) * D + h * dh;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane + 32 * e;
    if (d < dh) st(oi + d, o[e] * inv);
  }
}


// ---- offline f32 attention, head_dim 128 ----------------------------------
// A CTA takes 4 consecutive query rows of one (utterance, head), one per
// warp, and walks the keys in blocks of 32 that all 128 threads stage in
// shared memory with cp.async (double-buffered: block n+1 lands while block n
// computes): the block's K and V rows and the 35 positional rows its four
// query rows reach (P row T-1-i+j is window row 3 - w + l for warp w's row
// and key jb + l).  Lane l owns head dims 4l .. 4l+3: per key a lane forms
// its share of (q+u).k_j + (q+v).p_r, and a transposed butterfly over the
// warp (31 shuffles for 32 keys) leaves lane l with key jb + l's score, so
// the online softmax and P.V (lane-owned dims, float4 rows) need no
// per-key global loads.  Rows past the data load as zeros (cp.async with a
// zero source size), so masked keys meet finite V rows.
constexpr int kFRows = 4;                     // query rows per CTA
constexpr int kFKeys = 32;                    // keys per block
constexpr int kFPRows = kFKeys + kFRows - 1;  // positional rows per block
constexpr int kFBuf = (2 * kFKeys + kFPRows) * 128;  // floats per staged block

__device__ __forceinline__ void cp_async16z(float* dst, const float* src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src),
               "r"(in ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kFRows * 32)
    relpos_attn_f32_blocked_kernel(const float* __restrict__ q, int ldq,
                                   const float* __restrict__ k, int ldk,
                                   const float* __restrict__ v, int ldv,
                                   const float* __restrict__ p, int p_rows,
                                   const float* __restrict__ pu, const float* __restrict__ pv,
                                   const int32_t* __restrict__ key_len, AttnContextDev ctx,
                                   float* __restrict__ out, int T, int D) {
  extern __shared__ __align__(16) float fsm[];  // [2][kFBuf]
  __shared__ int s_lo[kFRows], s_hi[kFRows];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int i0 = blockIdx.x * kFRows, i = i0 + warp;
  const int col = h * 128 + 4 * lane;  // this lane's head dims
  int kend = T;
  if (key_len) kend = min(T, max(key_len[b], 1));
  int lo = 0, hi = 0;
  const StreamMaskDev none{};
  const bool any = i < T && key_interval(ctx, none, i, kend, lo, hi);
  if (lane == 0) {
    s_lo[warp] = any ? lo : INT32_MAX;
    s_hi[warp] = any ? hi : 0;
  }
  float4 qu = make_float4(0.f, 0.f, 0.f, 0.f), qv = qu;
  if (i < T) {
    const float4 x = *reinterpret_cast<const float4*>(q + (static_cast<int64_t>(b) * T + i) * ldq + col);
    const float4 u4 = *reinterpret_cast<const float4*>(pu + col);
    const float4 v4 = *reinterpret_cast<const float4*>(pv + col);
    qu = make_float4(x.x + u4.x, x.y + u4.y, x.z + u4.z, x.w + u4.w);
    qv = make_float4(x.x + v4.x, x.y + v4.y, x.z + v4.z, x.w + v4.w);
  }
  __syncthreads();
  int jlo = INT32_MAX, jhi = 0;  // the keys any of the CTA's rows sees
#pragma unroll
  for (int w = 0; w < kFRows; ++w) {
    jlo = min(jlo, s_lo[w]);
    jhi = max(jhi, s_hi[w]);
  }
  // block jb -> buffer s: K rows jb.., V rows jb.., positional rows from
  // T-1-(i0+3)+jb; 16 bytes per thread and step
  auto stage = [&](int jb, int s) {
    float* base = fsm + s * kFBuf;
    const int rbase = T - 1 - (i0 + kFRows - 1) + jb;
    for (int e = threadIdx.x; e < (2 * kFKeys + kFPRows) * 32; e += kFRows * 32) {
      const int row = e >> 5, c4 = (e & 31) * 4;
      const float* src;
      bool in;
      if (row < 2 * kFKeys) {
        const int j = jb + (row & (kFKeys - 1));
        in = j < T;
        src = row < kFKeys ? k + (static_cast<int64_t>(b) * T + j) * ldk
                           : v + (static_cast<int64_t>(b) * T + j) * ldv;
      } else {
        const int r = rbase + row - 2 * kFKeys;
        in = r >= 0 && r < p_rows;
        src = p + static_cast<int64_t>(r) * D;
      }
      cp_async16z(base + row * 128 + c4, in ? src + h * 128 + c4 : p, in);
    }
    cp_async_commit();
  };
  const float scale = rsqrtf(128.f);
  float m = -INFINITY, l = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (jlo < jhi) stage(jlo, 0);
  for (int jb = jlo, n = 0; jb < jhi; jb += kFKeys, ++n) {
    if (jb + kFKeys < jhi) {
      stage(jb + kFKeys, (n + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // block n is in shared memory for every thread
    if (any) {
      const float* sK = fsm + (n & 1) * kFBuf;
      const float* sV = sK + kFKeys * 128;
      const float* sP = sV + kFKeys * 128 + (kFRows - 1 - warp) * 128;
      float part[kFKeys];
#pragma unroll
      for (int kk = 0; kk < kFKeys; ++kk) {
        const float4 kv = *reinterpret_cast<const float4*>(sK + kk * 128 + 4 * lane);
        const float4 pr = *reinterpret_cast<const float4*>(sP + kk * 128 + 4 * lane);
        float a = qu.x * kv.x;
        a = fmaf(qu.y, kv.y, a);
        a = fmaf(qu.z, kv.z, a);
        a = fmaf(qu.w, kv.w, a);
        a = fmaf(qv.x, pr.x, a);
        a = fmaf(qv.y, pr.y, a);
        a = fmaf(qv.z, pr.z, a);
        part[kk] = fmaf(qv.w, pr.w, a);
      }
      // transposed butterfly: after the step of width `off`, a lane keeps
      // the keys whose bit matches its own lane bit
#pragma unroll
      for (int off = 16, nk = kFKeys; off >= 1; off >>= 1, nk >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int kk = 0; kk < nk / 2; ++kk) {
          const float send = upper ? part[kk] : part[kk + nk / 2];
          const float keep = upper ? part[kk + nk / 2] : part[kk];
          part[kk] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int j = jb + lane;
      const float sc = (j >= lo && j < hi) ? part[0] * scale : -INFINITY;
      float cm = sc;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
      const float mn = fmaxf(m, cm);
      const float alpha = (m == -INFINITY) ? 0.f : expf(m - mn);
      const float pj = (sc == -INFINITY) ? 0.f : expf(sc - mn);
      float ps = pj;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l = l * alpha + ps;
      o.x *= alpha;
      o.y *= alpha;
      o.z *= alpha;
      o.w *= alpha;
#pragma unroll
      for (int kk = 0; kk < kFKeys; ++kk) {
        const float w = __shfl_sync(0xffffffffu, pj, kk);
        const float4 vv = *reinterpret_cast<const float4*>(sV + kk * 128 + 4 * lane);
        o.x = fmaf(w, vv.x, o.x);
        o.y = fmaf(w, vv.y, o.y);
        o.z = fmaf(w, vv.z, o.z);
        o.w = fmaf(w, vv.w, o.w);
      }
      m = mn;
    }
    __syncthreads();  // buffer n & 1 is restaged for block n + 2
  }
  if (i < T) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    *reinterpret_cast<float4*>(out + (static_cast<int64_t>(b) * T + i) * D + col) =
        make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  }
}

}  // namespace

cudaError_t launch_relpos_attn_f32(const float* q, int ldq, const float* k, int ldk,
                                   const float* v, int ldv, const float* p, const float* u,
                                   const float* vb, const int32_t* key_len, AttnContextDev ctx,
                                   StreamMaskDev sm, float* out, int B, int Tq, int Tk, int D,
                                   int H, cudaStream_t stream) {
  // head_dim 128 with 16-byte aligned rows: the block-staged kernel
  if (D == H * 128 && Tq == Tk && (ldq & 3) == 0 && (ldk & 3) == 0 && (ldv & 3) == 0 &&
      (D & 3) == 0 &&
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(p) |
        reinterpret_cast<uintptr_t>(u) | reinterpret_cast<uintptr_t>(vb) |
        reinterpret_cast<uintptr_t>(out)) & 15) == 0 &&
      !sm.has) {
    constexpr int smem = 2 * kFBuf * 4;
    static std::atomic<uint64_t> attr{0};
    if (cudaError_t e = smem_attr_once(relpos_attn_f32_blocked_kernel, smem, attr)) return e;
    dim3 grid((Tq + kFRows - 1) / kFRows, H, B);
    relpos_attn_f32_blocked_kernel<<<grid, kFRows * 32, smem, stream>>>(
        q, ldq, k, ldk, v, ldv, p, 2 * Tq - 1, u, vb, key_len, ctx, out, Tq, D);
    return cudaGetLastError();
  }
  dim3 grid((Tq + kWarps - 1) / kWarps, H, B);
  relpos_attn_simt_kernel<float><<<grid, kWarps * 32, 0, stream>>>(
      q, ldq, k, ldk, v, ldv, nullptr, nullptr, 0, 0, p, u, vb, key_len, ctx, sm, out, Tq, Tk, D,
      H);
  return cudaGetLastError();
}

// Streaming with ring caches, any storage type (float or bf16).
template <typename T>
cudaError_t launch_relpos_attn_stream_simt(const T* q, int ldq, const T* knew, const T* vnew,
                                           int ldkv, const T* kc, const T* vc, int C, int head,
                                           const T* p, const float* u, const float* vb,
                                           StreamMaskDev sm, T* out, int B, int T_, int D, int H,
                                           cudaStream_t stream) {
  dim3 grid((T_ + kWarps - 1) / kWarps, H, B);
  AttnContextDev none{0, -1, -1, 0};
  relpos_attn_simt_kernel<T><<<grid, kWarps * 32, 0, stream>>>(
      q, ldq, knew, ldkv, vnew, ldkv, kc, vc, C, head, p, u, vb, nullptr, none, sm, out, T_,
      C + T_, D, H);
  return cudaGetLastError();
}

template cudaError_t launch_relpos_attn_stream_simt<float>(
    const float*, int, const float*, const float*, int, const float*, const float*, int, int,
    const float*, const float*, const float*, StreamMaskDev, float*, int, int, int, int,
    cudaStream_t);
template cudaError_t launch_relpos_attn_stream_simt<__nv_bfloat16>(
    const __nv_bfloat16*, int, const __nv_bfloat16*, const __nv_bfloat16*, int,
    const __nv_bfloat16*, const __nv_bfloat16*, int, int, const __nv_bfloat16*, const float*,
    const float*, StreamMaskDev, __nv_bfloat16*, int, int, int, int, cudaStream_t);

}  // namespace nrp
