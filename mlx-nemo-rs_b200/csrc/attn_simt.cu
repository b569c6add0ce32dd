// attn_simt.cu -- relative-position attention on CUDA cores, fp32 math.
//
// Serves modules whose dtype is f32 (the reference's default f32 graph,
// attention.rs:458-573 offline and 606-816 streaming; 1e-4 parity needs
// FFMA, not TF32 tensor cores) and any head_dim <= 128, plus the streaming
// form for bf16 storage.  One warp per query row: lanes score 32 keys at a
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

}  // namespace

cudaError_t launch_relpos_attn_f32(const float* q, int ldq, const float* k, int ldk,
                                   const float* v, int ldv, const float* p, const float* u,
                                   const float* vb, const int32_t* key_len, AttnContextDev ctx,
                                   StreamMaskDev sm, float* out, int B, int Tq, int Tk, int D,
                                   int H, cudaStream_t stream) {
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
