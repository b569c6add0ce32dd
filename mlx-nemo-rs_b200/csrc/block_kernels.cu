// block_kernels.cu -- the HBM-bound kernels of the Conformer block
// (src/asr/modules/encoders/conformer.rs:1693-1870, 2120-2330) that are not
// fused into a GEMM epilogue: LayerNorm, the depthwise convolution with the
// inference BatchNorm and SiLU, the input scaling of forward_from_embeddings
// and the final [B, T, D] -> [B, D, T] transpose.  All bf16 in HBM, f32 in
// registers, one rounding per output.
#include <cuda_bf16.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

__device__ __forceinline__ void unpack8(const uint4& q, float* f) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

__device__ __forceinline__ float silu(float v) { return v * sigmoid_approx(v); }

// nn::LayerNorm (eps 1e-5, affine): one warp per row of D = 256 * kChunks,
// the row held in registers (each lane 8 consecutive values per chunk);
// mean first, then the variance about it.  y may alias x.
template <int kChunks>
__global__ void __launch_bounds__(256) layernorm_kernel(const __nv_bfloat16* x,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta,
                                                        __nv_bfloat16* y, int64_t rows, float eps,
                                                        int act_silu) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  pdl_launch_dependents();
  if (row >= rows) return;
  pdl_wait();
  constexpr int D = 256 * kChunks;
  const __nv_bfloat16* xr = x + row * D;
  float v[kChunks][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    unpack8(*reinterpret_cast<const uint4*>(xr + c * 256 + lane * 8), v[c]);
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[c][e];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s * (1.f / D);
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = v[c][e] - mean;
      q += d * d;
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float inv = rsqrtf(q * (1.f / D) + eps);
  __nv_bfloat16* yr = y + row * D;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = c * 256 + lane * 8;
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(beta + col);
    const float4 b1 = *reinterpret_cast<const float4*>(beta + col + 4);
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float t = (v[c][e] - mean) * inv * gg[e] + bb[e];
      o[e] = act_silu ? silu(t) : t;
    }
    *reinterpret_cast<uint4*>(yr + col) = pack8(o);
  }
}

// Depthwise Conv1d over time (groups = D, kernel K, zero padding `pad_left`
// frames before and K-1-pad_left after: (K-1)/2 each side offline, K-1 on the
// left when causal), + bias, then optionally the inference BatchNorm folded
// to a per-channel affine and SiLU.  Taps are taps-major, wt[k * D + c].
//
// dwconv_rows_kernel (kernel size fixed at compile time, D % 128 == 0): no
// shared memory.  A lane owns 4 channels (8-byte loads, a warp covers 128
// channels of a row), a warp kDwF consecutive output frames: it loads the
// kDwF + kK - 1 input rows those need straight into registers, all in flight
// together, and accumulates with packed f32x2 FMAs, taps in registers.  The
// halo rows a neighbouring warp also loads come from L1/L2, so HBM sees each
// input row about once.  Accumulation runs over the taps in order k = 0..K-1.
constexpr int kDwF = 8;      // output frames per warp
constexpr int kDwWarps = 8;  // warps per CTA: kDwF * kDwWarps frames x 128 channels
template <int kK>
__global__ void __launch_bounds__(kDwWarps * 32, 2)
    dwconv_rows_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wt,
                       const float* __restrict__ bias, const float* __restrict__ bn_scale,
                       const float* __restrict__ bn_shift, __nv_bfloat16* __restrict__ y, int T,
                       int D, int pad_left, int act_silu) {
  constexpr int kRows = kDwF + kK - 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.y * 128 + lane * 4;
  const int t0 = (blockIdx.x * kDwWarps + warp) * kDwF;
  pdl_launch_dependents();
  if (t0 >= T) return;  // warp-uniform
  pdl_wait();
  const int64_t boff = static_cast<int64_t>(blockIdx.z) * T * D + c0;
  const __nv_bfloat16* xb = x + boff;
  uint2 raw[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int t = t0 - pad_left + r;
    raw[r] = (t >= 0 && t < T) ? __ldg(reinterpret_cast<const uint2*>(xb + static_cast<int64_t>(t) * D))
                               : make_uint2(0u, 0u);
  }
  float wr[kK][4];
#pragma unroll
  for (int k = 0; k < kK; ++k) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(wt + k * D + c0));
    wr[k][0] = q.x;
    wr[k][1] = q.y;
    wr[k][2] = q.z;
    wr[k][3] = q.w;
  }
  float acc[kDwF][4];
#pragma unroll
  for (int o = 0; o < kDwF; ++o)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[o][e] = 0.f;
  // output o takes input row o + k with tap k; rows ascend, so for each
  // output the taps arrive in order k = 0..K-1
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const float2 f01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[r].x));
    const float2 f23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[r].y));
#pragma unroll
    for (int o = 0; o < kDwF; ++o) {
      const int k = r - o;
      if (k < 0 || k >= kK) continue;
      fma2_acc(acc[o][0], acc[o][1], wr[k][0], wr[k][1], f01.x, f01.y);
      fma2_acc(acc[o][2], acc[o][3], wr[k][2], wr[k][3], f23.x, f23.y);
    }
  }
  float bi[4] = {0.f, 0.f, 0.f, 0.f}, sc[4] = {1.f, 1.f, 1.f, 1.f}, sh[4] = {0.f, 0.f, 0.f, 0.f};
  if (bias) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(bias + c0));
    bi[0] = q.x, bi[1] = q.y, bi[2] = q.z, bi[3] = q.w;
  }
  if (bn_scale) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(bn_scale + c0));
    sc[0] = q.x, sc[1] = q.y, sc[2] = q.z, sc[3] = q.w;
  }
  if (bn_shift) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(bn_shift + c0));
    sh[0] = q.x, sh[1] = q.y, sh[2] = q.z, sh[3] = q.w;
  }
  __nv_bfloat16* yb = y + boff;
#pragma unroll
  for (int o = 0; o < kDwF; ++o) {
    if (t0 + o >= T) break;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float t = (acc[o][e] + bi[e]) * sc[e] + sh[e];
      v[e] = act_silu ? silu(t) : t;
    }
    *reinterpret_cast<uint2*>(yb + static_cast<int64_t>(t0 + o) * D) =
        make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
}

// Any kernel size: a CTA covers kTT output frames of one utterance; its
// input rows (kTT + K - 1) are staged in shared memory with cp.async and the
// taps read from shared memory; each thread owns 8 channels.
constexpr int kTT = 32;
__global__ void __launch_bounds__(256) dwconv_smem_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const float* __restrict__ wt,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ bn_scale,
                                                          const float* __restrict__ bn_shift,
                                                          __nv_bfloat16* __restrict__ y, int T,
                                                          int D, int K, int pad_left,
                                                          int act_silu) {
  extern __shared__ __align__(16) uint8_t dw_smem[];
  __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(dw_smem);  // [kTT + K - 1][D]
  float* wsm = reinterpret_cast<float*>(dw_smem + static_cast<size_t>(kTT + K - 1) * D * 2);
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * kTT;
  const int rows = kTT + K - 1;
  const int vecs = D / 8;
  pdl_launch_dependents();
  pdl_wait();
  const __nv_bfloat16* xb = x + static_cast<int64_t>(b) * T * D;
  for (int i = threadIdx.x; i < rows * vecs; i += blockDim.x) {
    const int r = i / vecs, cv = i - r * vecs;
    const int t = t0 - pad_left + r;
    __nv_bfloat16* dst = tile + r * D + cv * 8;
    if (t >= 0 && t < T) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)),
                   "l"(xb + static_cast<int64_t>(t) * D + cv * 8)
                   : "memory");
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  for (int i = threadIdx.x; i < K * D; i += blockDim.x) wsm[i] = wt[i];
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();
  __nv_bfloat16* yb = y + static_cast<int64_t>(b) * T * D;
  for (int cv = threadIdx.x; cv < vecs; cv += blockDim.x) {
    const int c0 = cv * 8;
    float sc[8], sh[8], bi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      bi[e] = bias ? bias[c0 + e] : 0.f;
      sc[e] = bn_scale ? bn_scale[c0 + e] : 1.f;
      sh[e] = bn_shift ? bn_shift[c0 + e] : 0.f;
    }
    const int tn = min(kTT, T - t0);
    for (int tt = 0; tt < tn; ++tt) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int k = 0; k < K; ++k) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(tile + (tt + k) * D + c0), f);
        const float4 w0 = *reinterpret_cast<const float4*>(wsm + k * D + c0);
        const float4 w1 = *reinterpret_cast<const float4*>(wsm + k * D + c0 + 4);
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(ww[e], f[e], acc[e]);
      }
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float t = (acc[e] + bi[e]) * sc[e] + sh[e];
        o[e] = act_silu ? silu(t) : t;
      }
      *reinterpret_cast<uint4*>(yb + static_cast<int64_t>(t0 + tt) * D + c0) = pack8(o);
    }
  }
}

__global__ void scale_kernel(__nv_bfloat16* x, int64_t n8, float s) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float f[8];
    unpack8(reinterpret_cast<const uint4*>(x)[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] *= s;
    reinterpret_cast<uint4*>(x)[i] = pack8(f);
  }
}

// [B, T, D] -> [B, D, T], 32 x 32 tiles through shared memory.
__global__ void transpose_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                 int T, int D) {
  __shared__ __nv_bfloat16 tile[32][33];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const __nv_bfloat16* xb = x + static_cast<int64_t>(b) * T * D;
  __nv_bfloat16* yb = y + static_cast<int64_t>(b) * T * D;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int t = t0 + r, d = d0 + threadIdx.x;
    if (t < T && d < D) tile[r][threadIdx.x] = xb[static_cast<int64_t>(t) * D + d];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int d = d0 + r, t = t0 + threadIdx.x;
    if (t < T && d < D) yb[static_cast<int64_t>(d) * T + t] = tile[threadIdx.x][r];
  }
}

}  // namespace

cudaError_t launch_layernorm(const __nv_bfloat16* x, const float* gamma, const float* beta,
                             __nv_bfloat16* y, int64_t rows, int D, float eps, bool act_silu,
                             cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  switch (D) {
    case 256:
      return launch_pdl(layernorm_kernel<1>, grid, dim3(256), 0, stream, x, gamma, beta, y, rows,
                        eps, act_silu);
    case 512:
      return launch_pdl(layernorm_kernel<2>, grid, dim3(256), 0, stream, x, gamma, beta, y, rows,
                        eps, act_silu);
    case 1024:
      return launch_pdl(layernorm_kernel<4>, grid, dim3(256), 0, stream, x, gamma, beta, y, rows,
                        eps, act_silu);
    case 2048:
      return launch_pdl(layernorm_kernel<8>, grid, dim3(256), 0, stream, x, gamma, beta, y, rows,
                        eps, act_silu);
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_dwconv(const __nv_bfloat16* x, const float* wt, const float* bias,
                          const float* bn_scale, const float* bn_shift, __nv_bfloat16* y, int B,
                          int T, int D, int K, bool causal, bool act_silu, cudaStream_t stream) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 8 != 0 || K < 1 || B > 65535) return cudaErrorInvalidValue;
  const int pad = causal ? K - 1 : (K - 1) / 2;
  if (K == 9 && D % 128 == 0) {  // FastConformer's kernel size
    const int frames = kDwF * kDwWarps;
    const dim3 grid((T + frames - 1) / frames, D / 128, B);
    return launch_pdl(dwconv_rows_kernel<9>, grid, dim3(kDwWarps * 32), 0, stream, x, wt, bias,
                      bn_scale, bn_shift, y, T, D, pad, static_cast<int>(act_silu));
  }
  const size_t smem = static_cast<size_t>(kTT + K - 1) * D * 2 + static_cast<size_t>(K) * D * 4;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr{0};
  if (smem > 48 * 1024)
    if (cudaError_t e = smem_attr_once(dwconv_smem_kernel, 227 * 1024, attr)) return e;
  const dim3 grid((T + kTT - 1) / kTT, B);
  const int threads = D / 8 < 256 ? D / 8 : 256;
  return launch_pdl(dwconv_smem_kernel, grid, dim3(threads), smem, stream, x, wt, bias, bn_scale,
                    bn_shift, y, T, D, K, pad, static_cast<int>(act_silu));
  return cudaGetLastError();
}

cudaError_t launch_scale(__nv_bfloat16* x, int64_t n, float s, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (n % 8 != 0) return cudaErrorInvalidValue;
  return launch_pdl(scale_kernel, dim3(592), dim3(256), 0, stream, x, n / 8, s);
  return cudaGetLastError();
}

namespace {
__global__ void fill_i32_kernel(int32_t* p, int v, int n) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}
}  // namespace

cudaError_t launch_fill_i32(int32_t* p, int v, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  return launch_pdl(fill_i32_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, p, v, n);
}

cudaError_t launch_transpose_btd(const __nv_bfloat16* x, __nv_bfloat16* y, int B, int T, int D,
                                 cudaStream_t stream) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (B > 65535) return cudaErrorInvalidValue;
  const dim3 grid((T + 31) / 32, (D + 31) / 32, B);
  return launch_pdl(transpose_kernel, grid, dim3(32, 8), 0, stream, x, y, T, D);
  return cudaGetLastError();
}

}  // namespace nrp
