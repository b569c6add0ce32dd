// kernels_misc.cu -- the small kernels around the hot path:
//  * fp32 CUDA-core GEMM for modules whose dtype is f32 (LinearLayer's
//    Standard arm, src/core/quantization.rs:128-135, at f32 parity);
//  * the small-M MLX-affine 8-bit GEMM (quantized_matmul for streaming-size
//    M, quantization.rs:137-160): weights dequantised in registers into
//    bf16 MMA fragments, HBM-bound on the packed weights;
//  * dtype conversions, the ring-buffer row append of the streaming cache,
//    and the packed <-> padded frame moves around a host upload/download;
//  * TMA descriptor construction (driver entry point via the runtime).
#include <cudaTypedefs.h>
#include <algorithm>
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
                            const float* bias, float* y, int ldy, int num_sms, int* err,
                            cudaStream_t stream) {
  if (gemm_tf32_supported(M, K, N, x, w) && ldy >= N)
    return launch_gemm_tf32x3(x, M, K, w, N, bias, y, ldy, num_sms, err, stream);
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

// ------------------------------------------- small-M quantised GEMM
// y[M, N] = x[M, K] . W^T (+ bias, epilogue) for M <= 256 rows and MLX-affine
// 8-bit W (quantization.rs:137-160; w = scale * q + bias per 64-wide group,
// computed in f32 and rounded once to bf16, as the other 8-bit paths do).
// At these row counts the work is streaming the codes (1 byte per weight):
// the kernel is HBM-bound when every SM keeps enough code bytes in flight.
//
// A work unit is NG groups of 8 output columns and up to 64 rows; a CTA's 8
// warps split K (whole 64-wide groups) and reduce their partial sums through
// shared memory.  A unit's code rows come into shared memory by one bulk
// asynchronous copy per row; the CTA is persistent and double-buffers them
// (the first two units' copies are issued before the PDL wait, so they
// stream while the previous kernel finishes).  Per 64-wide block a lane (g = lane / 4:
// column g of a group, c = lane % 4) reads 16 code bytes of its column,
// dequantises them in registers, and feeds four m16n8k16 bf16 MMAs whose k
// order is permuted identically for both operands: k-step t, fragment
// columns 2c, 2c+1 / 2c+8, 2c+9 <-> k = 16c + 4t + {0, 1} / {2, 3}.  So the
// lane's 16 bytes are exactly its B fragments of the four k-steps, and its A
// fragments are 16 consecutive bf16 of rows g and g + 8 (two 16-byte loads
// per row, the next block's issued before the current one's MMAs).
namespace {
constexpr int kQsWarps = 8;

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// the 16 codes of a 16-byte load as floats: each byte placed in the low
// mantissa bits of 2^23 (one byte permute), then 2^23 subtracted (exact)
__device__ __forceinline__ void codes16(const uint4 q, float s, float z, float (&w)[16]) {
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[4 * u + e] =
          fmaf(s, __uint_as_float(__byte_perm(words[u], 0x4B000000u, 0x7540u | e)) - 8388608.f,
               z);
}

// Shared memory: two stages of code rows (row stride K + 64 bytes: the 8
// rows a quarter-warp reads fall in distinct banks), their mbarriers, two
// stages of (scale, zero point) bf16 pairs [column][group], then the partial
// sums [warp][MT * 16 rows][NG * 8 columns].
constexpr int kQsStages = 2;
__host__ __device__ constexpr int qs_code_stride(int K) { return K + 64; }
template <int NG>
__host__ __device__ constexpr int qs_bar_offset(int K) {
  return kQsStages * NG * 8 * qs_code_stride(K);
}
template <int NG>
__host__ __device__ constexpr int qs_scale_offset(int K) {
  return qs_bar_offset<NG>(K) + 16;
}
template <int MT, int NG>
__host__ __device__ constexpr int qs_red_offset(int K) {
  return qs_scale_offset<NG>(K) + kQsStages * NG * 8 * (K / 64) * 4;
}
template <int MT, int NG>
__host__ __device__ constexpr int qs_smem_bytes(int K) {
  return qs_red_offset<MT, NG>(K) + kQsWarps * MT * 16 * NG * 8 * 4;
}

// Persistent: CTA b works units b, b + G, b + 2G, ... (G = gridDim.x); unit
// u = (column slab u / chunks, 64-row chunk u % chunks).  While a unit
// computes, the unit two ahead has its code rows in flight into the other
// stage and its scale pairs in registers.
template <int MT, int NG>
__global__ void __launch_bounds__(kQsWarps * 32)
    qgemm_small_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                       const uint8_t* __restrict__ wq, const __nv_bfloat16* __restrict__ qs,
                       const __nv_bfloat16* __restrict__ qb, const __nv_bfloat16* __restrict__ bias,
                       __nv_bfloat16* y, int ldy, int N, Epilogue ep, int* err) {
  extern __shared__ __align__(128) uint8_t qsm[];
  constexpr int NC = NG * 8, ROWS = MT * 16;
  constexpr int kMaxPairs = NC * (kQSmallMaxK / 64) / (kQsWarps * 32);  // per thread
  const int stride = qs_code_stride(K);
  const int kblocks = K >> 6;
  uint8_t* codes = qsm;
  uint64_t* full = reinterpret_cast<uint64_t*>(qsm + qs_bar_offset<NG>(K));
  uint32_t* szs = reinterpret_cast<uint32_t*>(qsm + qs_scale_offset<NG>(K));
  float* red = reinterpret_cast<float*>(qsm + qs_red_offset<MT, NG>(K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int slabs = (N + NC - 1) / NC, chunks = (M + 63) / 64, units = slabs * chunks;
  const int per = (kblocks + kQsWarps - 1) / kQsWarps;
  const int kb0 = min(kblocks, warp * per), kb1 = min(kblocks, kb0 + per);

  // the code rows of unit u into stage s (warp 0)
  auto issue_codes = [&](int u, int s) {
    if (warp != 0) return;
    const int n0 = (u / chunks) * NC, ncols = min(NC, N - n0);
    if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ncols) * K);
    __syncwarp();
    if (lane < ncols)
      bulk_g2s(codes + (s * NC + lane) * stride, wq + static_cast<size_t>(n0 + lane) * K,
               static_cast<uint32_t>(K), &full[s]);
  };
  // the scale pairs of unit u: loaded into registers, stored into a stage
  uint32_t pend[kMaxPairs];
  auto load_scales = [&](int u) {
    const int n0 = (u / chunks) * NC, ncols = min(NC, N - n0);
#pragma unroll
    for (int p = 0; p < kMaxPairs; ++p) {
      const int e = threadIdx.x + p * kQsWarps * 32;
      if (e < ncols * kblocks) {
        const size_t gi = static_cast<size_t>(n0) * kblocks + e;
        pend[p] = static_cast<uint32_t>(__bfloat16_as_ushort(qs[gi])) |
                  (static_cast<uint32_t>(__bfloat16_as_ushort(qb[gi])) << 16);
      }
    }
  };
  auto store_scales = [&](int u, int s) {
    const int n0 = (u / chunks) * NC, ncols = min(NC, N - n0);
#pragma unroll
    for (int p = 0; p < kMaxPairs; ++p) {
      const int e = threadIdx.x + p * kQsWarps * 32;
      if (e < ncols * kblocks) szs[s * NC * kblocks + e] = pend[p];
    }
  };

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the first two units' weights, before waiting on the previous kernel:
  // the weights never depend on it
  for (int s = 0; s < kQsStages; ++s) {
    const int u = blockIdx.x + s * gridDim.x;
    if (u < units) {
      issue_codes(u, s);
      load_scales(u);
      store_scales(u, s);
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  __syncthreads();  // the stored scale pairs

  int i = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
    const int s = i & 1;
    const int n0 = (u / chunks) * NC, ncols = min(NC, N - n0);
    const int row0 = (u % chunks) * 64, mrows = min(64, M - row0);
    const __nv_bfloat16* xr = x + static_cast<size_t>(row0) * K;
    const int un = u + kQsStages * gridDim.x;
    if (un < units) load_scales(un);  // in flight under this unit
    float acc[MT][NG][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int q = 0; q < NG; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][q][e] = 0.f;
    // x: 16 bf16 of rows g and g + 8 of every m tile for one 64-wide block
    auto load_x = [&](int kb, uint4 (&xa)[MT][2][2]) {
      const int k = kb * 64 + 16 * c;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = 16 * m + g + 8 * r;
          xa[m][r][0] = xa[m][r][1] = make_uint4(0u, 0u, 0u, 0u);
          if (row < mrows) {
            const uint4* src =
                reinterpret_cast<const uint4*>(xr + static_cast<size_t>(row) * K + k);
            xa[m][r][0] = src[0];
            xa[m][r][1] = src[1];
          }
        }
    };
    uint4 xa[2][MT][2][2];
    if (kb0 < kb1) load_x(kb0, xa[0]);
    const bool landed =
        __all_sync(0xffffffffu, mbar_wait(&full[s], (i >> 1) & 1, err, kDevTimeoutLoad));
    const uint8_t* cs = codes + s * NC * stride;
    const uint32_t* ss = szs + s * NC * kblocks;
    // dequantise one block's codes for column group q into B fragments
    auto b_frags = [&](int kb, int q, uint32_t (&b)[8]) {
      const int nl = q * 8 + g;
      uint4 code = make_uint4(0u, 0u, 0u, 0u);
      float sc = 0.f, zp = 0.f;
      if (nl < ncols) {
        code = *reinterpret_cast<const uint4*>(cs + nl * stride + kb * 64 + 16 * c);
        const uint32_t sz = ss[nl * kblocks + kb];
        sc = __uint_as_float(sz << 16);
        zp = __uint_as_float(sz & 0xFFFF0000u);
      }
      float w[16];
      codes16(code, sc, zp, w);
#pragma unroll
      for (int t = 0; t < 8; ++t) b[t] = pack_bf16x2(w[2 * t], w[2 * t + 1]);
    };
    if (landed) {
      for (int kb = kb0; kb < kb1; kb += 2) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (kb + h >= kb1) break;
          if (kb + h + 1 < kb1) load_x(kb + h + 1, xa[h ^ 1]);
#pragma unroll
          for (int q = 0; q < NG; ++q) {
            uint32_t b[8];
            b_frags(kb + h, q, b);
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                // word 2t / 2t + 1 of a row's 16 bf16: columns 4t, 4t+1 / 4t+2, 4t+3
                const uint32_t* r0 = reinterpret_cast<const uint32_t*>(&xa[h][m][0][0]);
                const uint32_t* r1 = reinterpret_cast<const uint32_t*>(&xa[h][m][1][0]);
                mma_bf16_16816(acc[m][q], r0[2 * t], r1[2 * t], r0[2 * t + 1], r1[2 * t + 1],
                               b[2 * t], b[2 * t + 1]);
              }
          }
        }
      }
    }
    // partial sums of this warp's k range -> shared memory
    float* mine = red + warp * ROWS * NC;
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int q = 0; q < NG; ++q) {
        const int col = q * 8 + 2 * c;
        *reinterpret_cast<float2*>(mine + (16 * m + g) * NC + col) =
            make_float2(acc[m][q][0], acc[m][q][1]);
        *reinterpret_cast<float2*>(mine + (16 * m + g + 8) * NC + col) =
            make_float2(acc[m][q][2], acc[m][q][3]);
      }
    if (!__syncthreads_and(landed)) return;  // a copy never landed: error recorded
    for (int idx = threadIdx.x; idx < mrows * NC; idx += kQsWarps * 32) {
      const int row = idx / NC, col = idx - row * NC, n = n0 + col;
      if (col >= ncols) continue;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kQsWarps; ++w) v += red[(w * ROWS + row) * NC + col];
      if (ep.mode == kEpiRelu) v = __bfloat162float(__float2bfloat16_rn(v));
      if (bias) v += __bfloat162float(bias[n]);
      if (ep.mode == kEpiSilu) {
        v = v * sigmoid_approx(v);
      } else if (ep.mode == kEpiRelu) {
        v = fmaxf(v, 0.f);
      } else if (ep.mode == kEpiResidual) {
        v = fmaf(ep.alpha, v,
                 __bfloat162float(ep.res[static_cast<size_t>(row0 + row) * ep.ldr + n]));
      }
      y[static_cast<size_t>(row0 + row) * ldy + n] = __float2bfloat16_rn(v);
    }
    __syncthreads();  // stage s and the partial sums are free again
    if (un < units) {
      issue_codes(un, s);
      store_scales(un, s);
    }
  }
}

template <int MT, int NG>
cudaError_t launch_qs(const __nv_bfloat16* x, int M, int K, const uint8_t* wq,
                      const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                      const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int N,
                      int num_sms, const Epilogue& ep, int* err, cudaStream_t stream) {
  const int smem = qs_smem_bytes<MT, NG>(K);
  if (smem > kQSmallMaxSmem) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(qgemm_small_kernel<MT, NG>, kQSmallMaxSmem, attr))
    return e;
  // persistent: as many CTAs per SM as registers and shared memory allow (at
  // most 4), asked of the runtime once per shared-memory size
  static std::atomic<uint64_t> occ{0};  // (smem << 8) | CTAs per SM
  uint64_t o = occ.load(std::memory_order_relaxed);
  int per_sm = static_cast<int>(o & 0xFF);
  if ((o >> 8) != static_cast<uint64_t>(smem) || per_sm == 0) {
    if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, qgemm_small_kernel<MT, NG>, kQsWarps * 32, smem))
      return e;
    per_sm = std::max(1, std::min(4, per_sm));
    occ.store((static_cast<uint64_t>(smem) << 8) | static_cast<uint64_t>(per_sm),
              std::memory_order_relaxed);
  }
  const int units = ((N + NG * 8 - 1) / (NG * 8)) * ((M + 63) / 64);
  const int grid = std::min(units, per_sm * (num_sms > 0 ? num_sms : 148));
  return launch_pdl(qgemm_small_kernel<MT, NG>, dim3(grid), dim3(kQsWarps * 32), smem,
                    stream,
                    x, M, K, wq, qs, qb, bias, y, ldy, N, ep, err);
}

template <int MT>
cudaError_t launch_qs_ng(int ng, const __nv_bfloat16* x, int M, int K, const uint8_t* wq,
                         const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                         const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int N,
                         int num_sms, const Epilogue& ep, int* err, cudaStream_t stream) {
  if (ng == 2)
    return launch_qs<MT, 2>(x, M, K, wq, qs, qb, bias, y, ldy, N, num_sms, ep, err,
                                   stream);
  return launch_qs<MT, 1>(x, M, K, wq, qs, qb, bias, y, ldy, N, num_sms, ep, err, stream);
}
}  // namespace

bool qgemm_small_supported(int M, int K, const void* x, const void* wq, const Epilogue& ep) {
  return M >= 1 && M <= kQSmallMaxM && K % 64 == 0 && K <= kQSmallMaxK && ep.mode != kEpiGlu &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(wq) & 15) == 0;
}

cudaError_t launch_qgemm_small(const __nv_bfloat16* x, int M, int K, const uint8_t* wq,
                               const __nv_bfloat16* qs, const __nv_bfloat16* qb,
                               const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy, int N,
                               int num_sms, int* err, cudaStream_t stream, const Epilogue& ep) {
  if (!qgemm_small_supported(M, K, x, wq, ep) || N <= 0) return cudaErrorInvalidValue;
  // 16-column slabs (x read once for twice the columns) where two CTAs of
  // them still fit an SM; 8-column slabs otherwise
  const int mr = std::min(M, 64);
  const int ng = (mr <= 16 ? qs_smem_bytes<1, 2>(K)
                           : mr <= 32 ? qs_smem_bytes<2, 2>(K) : qs_smem_bytes<4, 2>(K)) <=
                         113 * 1024
                     ? 2
                     : 1;
  if (mr <= 16)
    return launch_qs_ng<1>(ng, x, M, K, wq, qs, qb, bias, y, ldy, N, num_sms, ep, err, stream);
  if (mr <= 32)
    return launch_qs_ng<2>(ng, x, M, K, wq, qs, qb, bias, y, ldy, N, num_sms, ep, err, stream);
  return launch_qs_ng<4>(ng, x, M, K, wq, qs, qb, bias, y, ldy, N, num_sms, ep, err, stream);
}

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

// Packed <-> padded frames of up to kMaxFrameUtts utterances: utterance u's
// rows are packed rows [off[u], off[u] + len[u]) and padded rows b0 + u,
// [0, len[u]).  Each block copies 16-byte vectors (V = uint4) or bytes
// (V = uint8_t) of one utterance (blockIdx.y), strided over blockIdx.x.
template <typename V>
__global__ void frames_kernel(uint8_t* __restrict__ padded, uint8_t* __restrict__ packed,
                              FramesPlan plan, bool to_padded, int32_t* __restrict__ dev_len) {
  const int u = blockIdx.y;
  const int64_t nv = plan.row_bytes / static_cast<int64_t>(sizeof(V));
  const int64_t n = static_cast<int64_t>(plan.len[u]) * nv;
  V* pd = reinterpret_cast<V*>(padded + (plan.b0 + u) * plan.bstride);
  V* pk = reinterpret_cast<V*>(packed + plan.off[u] * plan.row_bytes);
  if (dev_len && blockIdx.x == 0 && threadIdx.x == 0) dev_len[plan.b0 + u] = plan.len[u];
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (to_padded)
      pd[e] = pk[e];
    else
      pk[e] = pd[e];
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

namespace {

__global__ void wait_expiry_kernel(int* err, uint64_t budget_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x != 0) return;
  // nothing arrives on `bar`: the wait ends by its deadline
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(&bar, 0)) {
    if (globaltimer_ns() - t0 > budget_ns) {
      atomicCAS(err, 0, kDevTimeoutSelftest);
      return;
    }
  }
}

}  // namespace

cudaError_t launch_wait_expiry(int* err, uint64_t budget_ns, cudaStream_t stream) {
  if (!err || budget_ns == 0 || budget_ns > kWaitBudgetNs) return cudaErrorInvalidValue;
  wait_expiry_kernel<<<1, 32, 0, stream>>>(err, budget_ns);
  return cudaGetLastError();
}

cudaError_t launch_frames(void* padded, void* packed, const FramesPlan& plan, int n_utts,
                          bool to_padded, int32_t* dev_lengths, cudaStream_t stream) {
  if (n_utts <= 0) return cudaSuccess;
  if (n_utts > kMaxFrameUtts || plan.row_bytes <= 0) return cudaErrorInvalidValue;
  int max_len = 0;
  for (int u = 0; u < n_utts; ++u) max_len = std::max(max_len, plan.len[u]);
  const bool vec = (plan.row_bytes & 15) == 0 && (plan.bstride & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(padded) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(packed) & 15) == 0;
  const int64_t per_utt = static_cast<int64_t>(max_len) * (vec ? plan.row_bytes / 16
                                                                 : plan.row_bytes);
  // about four elements per thread; every utterance gets at least one block
  // (dev_lengths is written by block 0 of each)
  const int64_t gx = std::min<int64_t>(std::max<int64_t>((per_utt + 1023) / 1024, 1), 4096);
  dim3 grid(static_cast<unsigned>(gx), n_utts);
  uint8_t* pd = static_cast<uint8_t*>(padded);
  uint8_t* pk = static_cast<uint8_t*>(packed);
  if (vec)
    frames_kernel<uint4><<<grid, 256, 0, stream>>>(pd, pk, plan, to_padded, dev_lengths);
  else
    frames_kernel<uint8_t><<<grid, 256, 0, stream>>>(pd, pk, plan, to_padded, dev_lengths);
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
