// kernels_misc.cu -- the small kernels around the hot path:
//  * fp32 CUDA-core GEMM for modules whose dtype is f32 (LinearLayer's
//    Standard arm, src/core/quantization.rs:128-135, at f32 parity);
//  * the small-M MLX-affine 8-bit GEMV (quantized_matmul for streaming-size
//    M, quantization.rs:137-160), HBM-bound on the packed weights;
//  * dtype conversions and the ring-buffer row append of the streaming cache;
//  * TMA descriptor construction (driver entry point via the runtime).
#include <cudaTypedefs.h>
#include <math.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {

// -------------------------------------------------------------- TMA maps
namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}
}  // namespace

bool make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                  uint32_t box_outer, bool swizzle128) {
  auto enc = get_encode();
  if (!enc) return false;
  (void)elem_bytes;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                  uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                  bool swizzle128) {
  auto enc = get_encode();
  if (!enc) return false;
  (void)elem_bytes;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------ fp32 SIMT GEMM
// kTM x 64 output tile per CTA, 4 x 4 outputs per thread: 256 threads for
// 64 rows, or 128 threads for 32 rows when the 64-row grid would not give
// every SM two CTAs.  64-wide k tiles.  The next k tile is loaded into
// registers (float4 rows when K and the pointers allow) while the current
// one is multiplied from shared memory, so each step's load latency hides
// under the previous step's FMAs.  Each output sums its products in
// ascending k with fmaf, as a plain loop does.
namespace {
constexpr int kFN = 64, kFK = 64;

template <bool kVec, int kTM>
__global__ void __launch_bounds__(kTM * 4)
    gemm_f32_kernel(const float* __restrict__ x, int M, int K, const float* __restrict__ w, int N,
                    const float* __restrict__ bias, float* __restrict__ y, int ldy) {
  constexpr int kThreads = kTM * 4;
  constexpr int kTY = kThreads / 16;  // thread rows (4 output rows each)
  __shared__ __align__(16) float sx[kFK][kTM + 4];
  __shared__ __align__(16) float sw[kFK][kFN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kFN;
  // loader: rows lr + kTY*h of the x (h < 4) and w (h < 64 / kTY) tiles,
  // k columns lc .. lc+3
  constexpr int kWH = kFN / kTY;
  const int lr = threadIdx.x >> 4, lc = (threadIdx.x & 15) * 4;
  float px[4][4], pw[kWH][4];
  auto load_row = [&](const float* src, int row, int rows, int k, float (&v)[4]) {
    if (kVec) {
      const float4 a = (row < rows && k < K)
                           ? *reinterpret_cast<const float4*>(src + static_cast<size_t>(row) * K + k)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = (row < rows && k + j < K) ? src[static_cast<size_t>(row) * K + k + j] : 0.f;
    }
  };
  auto load = [&](int k0) {
#pragma unroll
    for (int h = 0; h < 4; ++h) load_row(x, m0 + lr + kTY * h, M, k0 + lc, px[h]);
#pragma unroll
    for (int h = 0; h < kWH; ++h) load_row(w, n0 + lr + kTY * h, N, k0 + lc, pw[h]);
  };
  float acc[4][4] = {};
  load(0);
  for (int k0 = 0; k0 < K; k0 += kFK) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 4; ++h) sx[lc + j][lr + kTY * h] = px[h][j];
#pragma unroll
      for (int h = 0; h < kWH; ++h) sw[lc + j][lr + kTY * h] = pw[h][j];
    }
    __syncthreads();
    if (k0 + kFK < K) load(k0 + kFK);  // in flight under the FMAs below
#pragma unroll
    for (int c = 0; c < kFK; ++c) {
      const float4 a = *reinterpret_cast<const float4*>(&sx[c][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&sw[c][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int m = m0 + ty * 4 + u;
    if (m >= M) continue;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int n = n0 + tx * 4 + v;
      if (n < N) y[static_cast<size_t>(m) * ldy + n] = acc[u][v] + (bias ? bias[n] : 0.f);
    }
  }
}

template <int kTM>
void launch_f32(bool vec, const float* x, int M, int K, const float* w, int N, const float* bias,
                float* y, int ldy, cudaStream_t stream) {
  const dim3 grid((N + kFN - 1) / kFN, (M + kTM - 1) / kTM);
  if (vec)
    gemm_f32_kernel<true, kTM><<<grid, kTM * 4, 0, stream>>>(x, M, K, w, N, bias, y, ldy);
  else
    gemm_f32_kernel<false, kTM><<<grid, kTM * 4, 0, stream>>>(x, M, K, w, N, bias, y, ldy);
}
}  // namespace

cudaError_t launch_gemm_f32(const float* x, int M, int K, const float* w, int N,
                            const float* bias, float* y, int ldy, int num_sms,
                            cudaStream_t stream) {
  const bool vec = K % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  // 32-row tiles when 64-row ones would give fewer than two CTAs per SM
  const long tiles64 = static_cast<long>((M + 63) / 64) * ((N + kFN - 1) / kFN);
  if (tiles64 < 2L * (num_sms > 0 ? num_sms : 148))
    launch_f32<32>(vec, x, M, K, w, N, bias, y, ldy, stream);
  else
    launch_f32<64>(vec, x, M, K, w, N, bias, y, ldy, stream);
  return cudaGetLastError();
}

// ------------------------------------------------- small-M quantised GEMV
// One warp per output column n.  Lane l reads 16 packed weights at a time
// (a 16-byte load; 32 lanes cover 512 contiguous bytes of the row), all in
// one group of 64, and FMAs them against every input row staged in shared
// memory as f32.  K is processed in slices of kQK columns.
namespace {
constexpr int kQMaxM = 16;
constexpr int kQK = 1024;
constexpr int kQWarps = 8;

__global__ void __launch_bounds__(kQWarps * 32)
    qgemv_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                 const uint8_t* __restrict__ wq, const __nv_bfloat16* __restrict__ qs,
                 const __nv_bfloat16* __restrict__ qb, const __nv_bfloat16* __restrict__ bias,
                 __nv_bfloat16* __restrict__ y, int ldy, int N) {
  extern __shared__ float sxq[];  // [M][kQK]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kQWarps + warp;
  const int kg = K / 64;
  float acc[kQMaxM];
#pragma unroll
  for (int m = 0; m < kQMaxM; ++m) acc[m] = 0.f;
  for (int k0 = 0; k0 < K; k0 += kQK) {
    const int kw = min(kQK, K - k0);
    __syncthreads();
    for (int e = threadIdx.x; e < M * kw; e += blockDim.x) {
      const int m = e / kw, c = e % kw;
      sxq[m * kQK + c] = __bfloat162float(x[static_cast<size_t>(m) * K + k0 + c]);
    }
    __syncthreads();
    if (n < N) {
      for (int c = lane * 16; c < kw; c += 32 * 16) {
        const int k = k0 + c;
        const uint4 q = *reinterpret_cast<const uint4*>(wq + static_cast<size_t>(n) * K + k);
        const float s = __bfloat162float(qs[static_cast<size_t>(n) * kg + k / 64]);
        const float bz = __bfloat162float(qb[static_cast<size_t>(n) * kg + k / 64]);
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
        float wv[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            wv[4 * u + e] = fmaf(s, static_cast<float>((words[u] >> (8 * e)) & 0xFFu), bz);
        }
#pragma unroll
        for (int m = 0; m < kQMaxM; ++m) {
          if (m < M) {
            const float4* xr = reinterpret_cast<const float4*>(sxq + m * kQK + c);
            float a = acc[m];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const float4 xv = xr[v];
              a = fmaf(xv.x, wv[4 * v], a);
              a = fmaf(xv.y, wv[4 * v + 1], a);
              a = fmaf(xv.z, wv[4 * v + 2], a);
              a = fmaf(xv.w, wv[4 * v + 3], a);
            }
            acc[m] = a;
          }
        }
      }
    }
  }
  if (n >= N) return;
#pragma unroll
  for (int m = 0; m < kQMaxM; ++m) {
    if (m >= M) break;
    float a = acc[m];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if (lane == 0) {
      if (bias) a += __bfloat162float(bias[n]);
      y[static_cast<size_t>(m) * ldy + n] = __float2bfloat16_rn(a);
    }
  }
}
}  // namespace

namespace {
// MLX affine dequantisation of 8-bit weights (quantization.rs:4-8, group
// 64): w[n, k] = scale[n, k/64] * q[n, k] + bias[n, k/64], computed in f32
// and rounded once to bf16 -- the values the in-register GEMM producer
// writes into its B tiles.  One thread per 16 weights (a 16-byte load, two
// 16-byte stores); HBM-bound.
// Dequantises one or more 8-bit weights (w = scale * q + bias per 64-wide
// group, MLX affine) into bf16 in one launch: the jobs' 16-weight units are
// numbered consecutively and the grid strides over all of them.
__global__ void dequant_q8_kernel(const __grid_constant__ DeqBatch jobs) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = jobs.begin16[jobs.n];
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int j = 0;
    while (i >= jobs.begin16[j + 1]) ++j;
    const DeqJob& jb = jobs.job[j];
    const int64_t u = i - jobs.begin16[j];
    const int64_t e0 = u * 16;
    const int64_t n = e0 / jb.K;
    const int k = static_cast<int>(e0 - n * jb.K);
    const int groups = jb.K / 64;
    const float sc = __bfloat162float(jb.qs[n * groups + k / 64]);
    const float bi = __bfloat162float(jb.qb[n * groups + k / 64]);
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(jb.wq) + u);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t v = words[t];
      o[2 * t] = pack_bf16x2(fmaf(sc, static_cast<float>(v & 0xFF), bi),
                             fmaf(sc, static_cast<float>((v >> 8) & 0xFF), bi));
      o[2 * t + 1] = pack_bf16x2(fmaf(sc, static_cast<float>((v >> 16) & 0xFF), bi),
                                 fmaf(sc, static_cast<float>(v >> 24), bi));
    }
    uint4* dst = reinterpret_cast<uint4*>(jb.w + e0);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}
}  // namespace

cudaError_t launch_dequant_q8_batch(const DeqJob* jobs, int n, int num_sms, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (n > kMaxDeqJobs) return cudaErrorInvalidValue;
  DeqBatch b{};
  b.n = n;
  b.begin16[0] = 0;
  for (int j = 0; j < n; ++j) {
    if (jobs[j].K % 64 != 0 || jobs[j].N <= 0) return cudaErrorInvalidValue;
    b.job[j] = jobs[j];
    b.begin16[j + 1] = b.begin16[j] + static_cast<int64_t>(jobs[j].N) * jobs[j].K / 16;
  }
  const int64_t want = (b.begin16[n] + 255) / 256;
  const int grid = static_cast<int>(want < num_sms * 8 ? want : num_sms * 8);
  return launch_pdl(dequant_q8_kernel, dim3(grid), dim3(256), 0, stream, b);
}

cudaError_t launch_dequant_q8(const uint8_t* wq, const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                              __nv_bfloat16* w, int N, int K, int num_sms, cudaStream_t stream) {
  const DeqJob j{wq, qs, qb, w, N, K};
  return launch_dequant_q8_batch(&j, 1, num_sms, stream);
}

cudaError_t launch_qgemv(const __nv_bfloat16* x, int M, int K, const uint8_t* wq,
                         const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                         const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int N,
                         cudaStream_t stream) {
  if (M > kQMaxM || K % 512 != 0) return cudaErrorInvalidValue;
  const int smem = kQMaxM * kQK * 4;
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(qgemv_kernel, smem, attr))
    return e;
  qgemv_kernel<<<(N + kQWarps - 1) / kQWarps, kQWarps * 32, smem, stream>>>(x, M, K, wq, qs, qb,
                                                                           bias, y, ldy, N);
  return cudaGetLastError();
}

// ------------------------------------------------------------ conversions
namespace {
__global__ void f32_to_bf16_kernel(const float* __restrict__ s, __nv_bfloat16* __restrict__ d,
                                   int64_t n) {
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d[e] = __float2bfloat16_rn(s[e]);
}
__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ s, float* __restrict__ d,
                                   int64_t n) {
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d[e] = __bfloat162float(s[e]);
}
int grid_for(int64_t n) {
  int64_t g = (n + 255) / 256;
  return static_cast<int>(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}

// dst[b, (head + i) % C, :] = src[b, i, :]; one block per (i, b), 16-byte
// vectors when the row allows it.
__global__ void ring_append_kernel(const uint8_t* __restrict__ src, int64_t sb, int64_t sr,
                                   uint8_t* __restrict__ dst, int64_t db, int C, int head,
                                   int row_bytes) {
  const int i = blockIdx.x, b = blockIdx.y;
  const uint8_t* s = src + b * sb + i * sr;
  uint8_t* d = dst + b * db + static_cast<int64_t>((head + i) % C) * row_bytes;
  if ((row_bytes & 15) == 0 && (reinterpret_cast<uintptr_t>(s) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
    for (int e = threadIdx.x; e < row_bytes / 16; e += blockDim.x)
      reinterpret_cast<uint4*>(d)[e] = reinterpret_cast<const uint4*>(s)[e];
  } else {
    for (int e = threadIdx.x; e < row_bytes; e += blockDim.x) d[e] = s[e];
  }
}
}  // namespace

cudaError_t launch_f32_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n,
                               cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  f32_to_bf16_kernel<<<grid_for(n), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_bf16_to_f32(const __nv_bfloat16* src, float* dst, int64_t n,
                               cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  bf16_to_f32_kernel<<<grid_for(n), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_ring_append(const void* src, int64_t src_bstride, int64_t src_rstride,
                               void* dst, int64_t dst_bstride, int C, int head, int n, int B,
                               int cols, int elem_bytes, cudaStream_t stream) {
  if (n <= 0 || B <= 0) return cudaSuccess;
  dim3 grid(n, B);
  ring_append_kernel<<<grid, 128, 0, stream>>>(
      static_cast<const uint8_t*>(src), src_bstride * elem_bytes, src_rstride * elem_bytes,
      static_cast<uint8_t*>(dst), dst_bstride * elem_bytes, C, head, cols * elem_bytes);
  return cudaGetLastError();
}

}  // namespace nrp
