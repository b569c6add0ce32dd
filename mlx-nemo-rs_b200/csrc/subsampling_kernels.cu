// subsampling_kernels.cu -- the convolutions of the dw_striding subsampling
// (src/asr/modules/encoders/conformer.rs:1413-1555) that are not GEMMs.
//
//   conv0_dw_kernel  mel -> conv.0 (1 -> C, 3x3, stride 2) + ReLU, and with
//                    kFuse the first depthwise 3x3 stride-2 conv (+ bias) on
//                    top, the conv.0 activations kept in shared memory (they
//                    are the largest tensor of the stack: 4x the depthwise
//                    output).  The mel frames are read in either layout
//                    ([B, F, T] as the encoder gets them, or [B, T, F]),
//                    masked past each length and rounded to bf16 on the way.
//   dw_s2_kernel     a further depthwise 3x3 stride-2 conv (+ bias), NHWC.
// Activations are NHWC bf16 [B, T, F, C] (channels innermost, so the 1x1
// pointwise convs are plain [rows, C] x [C, C] GEMMs).  Each conv output is
// rounded to bf16, then the bias add is rounded again, then the ReLU, as the
// reference's bf16 graph does (nn::Conv2d::forward adds its bias as a
// separate op).  Weights are f32 holding bf16-rounded values, [C][9] taps.
#include <cuda_bf16.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kSubThreads = 256;
constexpr int kSubCb = 32;  // channels per CTA (4 threads x 8)
constexpr int kSubR2 = 8;   // depthwise output rows per CTA (fused)
constexpr int kSubR1 = 16;  // conv.0 output rows per CTA (conv.0 alone)

__device__ __forceinline__ float bf16r(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ void unpack8s(const uint4& q, float* f) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8s(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// Eight channels' 3x3 taps (w [C][9], c0 a multiple of 8: 16-byte aligned).
__device__ __forceinline__ void load_taps8(const float* __restrict__ w, int c0, float (&t)[8][9]) {
  const float4* p = reinterpret_cast<const float4*>(w + c0 * 9);
  float f[72];
#pragma unroll
  for (int i = 0; i < 18; ++i) {
    const float4 v = __ldg(p + i);
    f[4 * i] = v.x;
    f[4 * i + 1] = v.y;
    f[4 * i + 2] = v.z;
    f[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int k = 0; k < 9; ++k) t[e][k] = f[e * 9 + k];
}

// conv output -> round, + bias -> round (+ ReLU)
__device__ __forceinline__ void finish8(float* acc, const float* b, bool relu) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float v = bf16r(bf16r(acc[e]) + b[e]);
    acc[e] = relu ? fmaxf(v, 0.f) : v;
  }
}

// grid (row tiles, C / 32, B).  Row tile: kSubR2 depthwise rows (kFuse) or
// kSubR1 conv.0 rows.  Shared memory: the mel rows the tile reads as f32
// [rows][2 F1 + 1] (column j is frequency j - pad), then with kFuse the
// conv.0 rows [2 kSubR2 + 1][F1][32] bf16.
template <bool kFuse>
__global__ void __launch_bounds__(kSubThreads, 2) conv0_dw_kernel(const SubConvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * kSubCb;
  const int q = tid & 3;  // this thread's 8 channels: c0 + 8q ..
  const int R1 = kFuse ? 2 * kSubR2 + 1 : kSubR1;
  const int t2_0 = blockIdx.x * kSubR2;
  const int t1_0 = kFuse ? 2 * t2_0 - a.pad : blockIdx.x * kSubR1;  // first conv.0 row
  const int nm = 2 * R1 + 1;                                         // mel rows
  const int fm = 2 * a.F1 + 1;                                       // mel columns
  const int tm0 = 2 * t1_0 - a.pad;                                  // first mel row
  float* mel = reinterpret_cast<float*>(smem);
  __nv_bfloat16* c0t = reinterpret_cast<__nv_bfloat16*>(
      smem + ((static_cast<uint32_t>(nm) * fm * 4 + 15) & ~15u));
  pdl_wait();
  const int lenb = a.len ? a.len[b] : a.T;

  // 1. mel rows (zero outside the input and past the length), rounded to
  // bf16; walk the layout's contiguous axis with consecutive threads
  const float* src = a.mel + static_cast<int64_t>(b) * a.mel_bs;
  const int lim = min(a.T, lenb);
  const int n = nm * fm;
  if (a.mel_ts == 1) {
    for (int idx = tid; idx < n; idx += kSubThreads) {
      const int i = idx % nm, j = idx / nm;
      const int t = tm0 + i, f = j - a.pad;
      float v = 0.f;
      if (t >= 0 && t < lim && f >= 0 && f < a.F)
        v = bf16r(__ldg(src + static_cast<int64_t>(t) + static_cast<int64_t>(f) * a.mel_fs));
      mel[i * fm + j] = v;
    }
  } else {
    for (int idx = tid; idx < n; idx += kSubThreads) {
      const int i = idx / fm, j = idx % fm;
      const int t = tm0 + i, f = j - a.pad;
      float v = 0.f;
      if (t >= 0 && t < lim && f >= 0 && f < a.F)
        v = bf16r(__ldg(src + static_cast<int64_t>(t) * a.mel_ts + static_cast<int64_t>(f) * a.mel_fs));
      mel[i * fm + j] = v;
    }
  }
  __syncthreads();

  // 2. conv.0 + bias + ReLU: item = (row, f1, q)
  {
    float w[8][9], bias[8];
    load_taps8(a.w0, c0 + 8 * q, w);
#pragma unroll
    for (int e = 0; e < 8; ++e) bias[e] = __ldg(a.b0 + c0 + 8 * q + e);
    const int items = R1 * a.F1 * 4;
    for (int idx = tid; idx < items; idx += kSubThreads) {
      const int pos = idx >> 2;
      const int r = pos / a.F1, f1 = pos - r * a.F1;
      const int t1 = t1_0 + r;
      const bool live = t1 >= 0 && t1 < a.T1;
      if (!kFuse && !live) continue;
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      if (live) {
        const float* m = mel + (2 * r) * fm + 2 * f1;
#pragma unroll
        for (int kt = 0; kt < 3; ++kt)
#pragma unroll
          for (int kf = 0; kf < 3; ++kf) {
            const float x = m[kt * fm + kf];
#pragma unroll
            for (int e = 0; e < 8; e += 2)
              fma_f32x2v(acc[e], acc[e + 1], w[e][kt * 3 + kf], w[e + 1][kt * 3 + kf], x,
                         acc[e], acc[e + 1]);
          }
        finish8(acc, bias, true);
      }
      const uint4 o = pack8s(acc);  // padding rows of the depthwise input: zeros
      if (kFuse)
        *reinterpret_cast<uint4*>(c0t + (static_cast<int64_t>(pos) * kSubCb + 8 * q)) = o;
      else
        *reinterpret_cast<uint4*>(
            a.out + ((static_cast<int64_t>(b) * a.T1 + t1) * a.F1 + f1) * a.C + c0 + 8 * q) = o;
    }
  }
  if (!kFuse) return;
  __syncthreads();

  // 3. depthwise 3x3 stride 2 + bias over the conv.0 rows: item = (row, f2, q)
  float w[8][9], bias[8];
  load_taps8(a.w1, c0 + 8 * q, w);
#pragma unroll
  for (int e = 0; e < 8; ++e) bias[e] = __ldg(a.b1 + c0 + 8 * q + e);
  const int items = kSubR2 * a.F2 * 4;
  for (int idx = tid; idx < items; idx += kSubThreads) {
    const int pos = idx >> 2;
    const int r2 = pos / a.F2, f2 = pos - r2 * a.F2;
    const int t2 = t2_0 + r2;
    if (t2 >= a.T2) continue;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int kt = 0; kt < 3; ++kt)
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) {
        const int f1 = 2 * f2 + kf - a.pad;
        if (f1 < 0 || f1 >= a.F1) continue;
        float x[8];
        unpack8s(*reinterpret_cast<const uint4*>(
                     c0t + ((static_cast<int64_t>(2 * r2 + kt) * a.F1 + f1) * kSubCb + 8 * q)),
                 x);
#pragma unroll
        for (int e = 0; e < 8; e += 2)
          fma2_acc(acc[e], acc[e + 1], x[e], x[e + 1], w[e][kt * 3 + kf], w[e + 1][kt * 3 + kf]);
      }
    finish8(acc, bias, false);
    *reinterpret_cast<uint4*>(a.out + ((static_cast<int64_t>(b) * a.T2 + t2) * a.F2 + f2) * a.C +
                              c0 + 8 * q) = pack8s(acc);
  }
}

// y [B][To][Fo][C] = depthwise 3x3 stride 2 (+ bias) of x [B][Ti][Fi][C];
// input (2 to + kt - pad, 2 fo + kf - pad), zero outside.  Each thread keeps
// one 8-channel group (256 % (C / 8) == 0) and its taps, and strides over
// output positions.
__global__ void __launch_bounds__(kSubThreads) dw_s2_kernel(const __nv_bfloat16* __restrict__ x,
                                                            int Ti, int Fi, int C, int pad,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bvec,
                                                            __nv_bfloat16* __restrict__ y, int To,
                                                            int Fo, int64_t positions) {
  pdl_launch_dependents();
  const int groups = C >> 3;
  const int64_t start = static_cast<int64_t>(blockIdx.x) * kSubThreads + threadIdx.x;
  const int g = static_cast<int>(start % groups);
  const int64_t step = static_cast<int64_t>(gridDim.x) * kSubThreads / groups;
  float taps[8][9], bias[8];
  load_taps8(w, 8 * g, taps);
#pragma unroll
  for (int e = 0; e < 8; ++e) bias[e] = __ldg(bvec + 8 * g + e);
  pdl_wait();
  for (int64_t p = start / groups; p < positions; p += step) {
    const int fo = static_cast<int>(p % Fo);
    const int64_t bt = p / Fo;  // b * To + to
    const int to = static_cast<int>(bt % To);
    const int64_t b = bt / To;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int kt = 0; kt < 3; ++kt) {
      const int ti = 2 * to + kt - pad;
      if (ti < 0 || ti >= Ti) continue;
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) {
        const int fi = 2 * fo + kf - pad;
        if (fi < 0 || fi >= Fi) continue;
        float v[8];
        unpack8s(__ldg(reinterpret_cast<const uint4*>(
                     x + ((b * Ti + ti) * Fi + fi) * C + 8 * g)),
                 v);
#pragma unroll
        for (int e = 0; e < 8; e += 2)
          fma2_acc(acc[e], acc[e + 1], v[e], v[e + 1], taps[e][kt * 3 + kf],
                   taps[e + 1][kt * 3 + kf]);
      }
    }
    finish8(acc, bias, false);
    *reinterpret_cast<uint4*>(y + p * C + 8 * g) = pack8s(acc);
  }
}

}  // namespace

constexpr int kSubMaxSmem = 227 * 1024;

size_t subsample_conv0_smem(int F1, bool fuse) {
  const int R1 = fuse ? 2 * kSubR2 + 1 : kSubR1;
  const size_t mel = (static_cast<size_t>(2 * R1 + 1) * (2 * F1 + 1) * 4 + 15) & ~size_t(15);
  return mel + (fuse ? static_cast<size_t>(R1) * F1 * kSubCb * 2 : 0);
}

cudaError_t launch_subsample_conv0(const SubConvArgs& a, int B, bool fuse, cudaStream_t stream) {
  if (a.C % kSubCb != 0) return cudaErrorInvalidValue;
  const size_t smem = subsample_conv0_smem(a.F1, fuse);
  if (smem > static_cast<size_t>(kSubMaxSmem)) return cudaErrorInvalidValue;
  const int tiles = fuse ? (a.T2 + kSubR2 - 1) / kSubR2 : (a.T1 + kSubR1 - 1) / kSubR1;
  const dim3 grid(tiles, a.C / kSubCb, B);
  if (fuse) {
    static std::atomic<uint64_t> done{0};
    cudaError_t e = smem_attr_once(conv0_dw_kernel<true>, kSubMaxSmem, done);
    if (e != cudaSuccess) return e;
    return launch_pdl(conv0_dw_kernel<true>, grid, dim3(kSubThreads), smem, stream, a);
  }
  static std::atomic<uint64_t> done{0};
  cudaError_t e = smem_attr_once(conv0_dw_kernel<false>, kSubMaxSmem, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(conv0_dw_kernel<false>, grid, dim3(kSubThreads), smem, stream, a);
}

cudaError_t launch_subsample_dw(const __nv_bfloat16* x, int B, int Ti, int Fi, int C, int pad,
                                const float* w, const float* b, __nv_bfloat16* y, int To, int Fo,
                                int num_sms, cudaStream_t stream) {
  if (C % 8 != 0 || kSubThreads % (C / 8) != 0) return cudaErrorInvalidValue;
  const int64_t positions = static_cast<int64_t>(B) * To * Fo;
  const int64_t threads = positions * (C / 8);
  const int64_t want = (threads + kSubThreads - 1) / kSubThreads;
  const int grid = static_cast<int>(want < 8LL * num_sms ? want : 8LL * num_sms);
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(dw_s2_kernel, dim3(grid), dim3(kSubThreads), 0, stream, x, Ti, Fi, C, pad, w,
                    b, y, To, Fo, positions);
}

}  // namespace nrp
