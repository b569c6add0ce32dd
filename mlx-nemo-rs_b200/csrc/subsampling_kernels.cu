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
//                    conv.0 runs on the tensor cores as an implicit GEMM:
//                    16 output positions x 16 taps (9 used) x 8 channels per
//                    warp-level bf16 MMA, the im2col rows read straight from
//                    the shared mel tile; K = 9 makes tensor throughput
//                    irrelevant, the MMA only replaces 72 FMAs per position
//                    and channel octet with a fraction of an instruction.
//   dw_s2_kernel     a further depthwise 3x3 stride-2 conv (+ bias): the
//                    input rows of a tile of output rows staged in shared
//                    memory, then the same depthwise step.
// Activations are NHWC bf16 [B, T, F, C] (channels innermost, so the 1x1
// pointwise convs are plain [rows, C] x [C, C] GEMMs).  Each conv output is
// rounded to bf16, then the bias add is rounded again, then the ReLU, as the
// reference's bf16 graph does (nn::Conv2d::forward adds its bias as a
// separate op): the bias add runs as add.rn.bf16x2 on the rounded conv
// output, which equals rounding the f32 sum of the two bf16 values.
// Weights come as MMA B fragments built on the host (subsampling.cpp).
#include <cuda_bf16.h>

#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kSubThreads = 256;
constexpr int kSubWarps = kSubThreads / 32;
constexpr int kSubCb = 32;       // channels per CTA (4 threads x 8)
constexpr int kSubR2 = 8;        // depthwise output rows per CTA
constexpr int kSubR1 = 16;       // conv.0 output rows per CTA (conv.0 alone)
constexpr int kPosStride = 80;   // bytes per position of a shared NHWC tile:
                                 // 64 B of channels + 16 B, so that the eight
                                 // positions of a warp's stores hit distinct banks
constexpr int kSubMaxSmem = 227 * 1024;

__device__ __forceinline__ uint32_t max0_bf16x2(uint32_t a) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(0u));
  return d;
}

// Asynchronous copies into shared memory; src_bytes 0 writes zeros (src is
// then not read but must still be a valid address).
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// d += a . b, one 16x8x16 bf16 MMA with f32 accumulators (row-major A
// fragment, column-major B).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four 8x8 b16 matrices from shared memory: lanes 8i .. 8i+7 give the row
// addresses (16 bytes each) of matrix i; register i receives matrix i in the
// MMA fragment layout (row lane / 4, elements 2 (lane % 4), +1).
__device__ __forceinline__ void ldmatrix_x4(uint32_t row, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(row));
}

// MMA B fragments in the order the host lays them out (subsampling.cpp,
// kSubFragWords words per lane and n-tile group): this lane's 12 words.
__device__ __forceinline__ void load_frag12(const uint32_t* __restrict__ f, int lane,
                                            uint32_t (&w)[12]) {
  const uint4* p = reinterpret_cast<const uint4*>(f) + lane * 3;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const uint4 v = __ldg(p + i);
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}

// Shared NHWC tiles of the depthwise convs.  A tile row holds the input
// columns c = col + pad in [0, W) (col in [-pad, W - pad); the padding
// columns hold zeros), even c in slots 0 .. E - 1 and odd c in slots E ..:
// the stride-2 taps of 8 consecutive output positions then read 8
// consecutive slots (80 bytes apart: distinct banks), and E = 4 (mod 8)
// puts the odd half 16 banks away from the even one, so the 8 consecutive
// columns a warp's conv.0 stores cover are distinct banks too.
struct TileRow {
  int E, slots;  // even slots, slots per row
};
__host__ __device__ __forceinline__ TileRow tile_row(int W) {
  const int e = (W + 1) / 2;
  const int E = e + (12 - e % 8) % 8;
  return {E, E + W / 2};
}
__host__ __device__ __forceinline__ int tile_slot(int c, int E) {
  return (c & 1) ? E + (c >> 1) : (c >> 1);
}

// Depthwise 3x3 stride 2 + bias, on the tensor cores, of an NHWC tile in
// shared memory in the layout above (W = Wt columns, tr = tile_row(Wt)),
// 32 channels bf16 per slot; tile row 0 = input row 2 t0 - pad; `zero`
// 64 zero bytes.  Output rows t0 .. t0 + kSubR2 - 1 (< To), Fo positions
// wide, into y (NHWC [B][To][Fo][C], the tile's channels from c0).  Each
// warp takes blocks of 16 output positions of one row; per block and
// n-tile, five 16x8x16 MMAs whose A rows (one position's 8 channels for one
// tap) come by ldmatrix straight from the tile.
__device__ __forceinline__ void dw_tile_mma(const uint8_t* tile, TileRow tr, int Fo, int To, int t0,
                                            const uint32_t* __restrict__ frag,
                                            const uint8_t* zero, __nv_bfloat16* y, int64_t b,
                                            int C, int c0, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int rows = min(kSubR2, To - t0);
  const int nb = (Fo + 15) >> 4;  // blocks per row
  // byte offset of tap 2j + (mi >> 1) from the slot of column 2f (even,
  // row 2 r2) of output position f: tap (kt, kf) reads row 2 r2 + kt,
  // column 2f + kf (-1: tap 9)
  int toff[5];
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int tap = 2 * j + (mi >> 1), kt = tap / 3, kf = tap % 3;
    toff[j] = tap < 9 ? (kt * tr.slots + (kf == 1 ? tr.E : kf >> 1)) * kPosStride : -1;
  }
  const uint32_t tile_s = smem_u32(tile), zero_s = smem_u32(zero);
  // fragments of n-tile nt: words 2j, 2j+1 = k-step j, word 10 = bias pair
  uint32_t nxt[12];
  load_frag12(frag + (c0 / 8) * 32 * kSubFragWords, lane, nxt);
#pragma unroll 1
  for (int nt = 0; nt < kSubCb / 8; ++nt) {
    uint32_t fw[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) fw[i] = nxt[i];
    if (nt + 1 < kSubCb / 8)  // in flight while this n-tile runs
      load_frag12(frag + (c0 / 8 + nt + 1) * 32 * kSubFragWords, lane, nxt);
    // two position blocks at a time: independent accumulator chains
    for (int blk = warp; blk < rows * nb; blk += 2 * kSubWarps) {
      const int nbk = blk + kSubWarps < rows * nb ? 2 : 1;  // (warp-uniform)
      uint32_t base[2];
      bool lv[2];
      int r2[2], f0[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int bk = blk + h * kSubWarps;
        r2[h] = bk / nb;
        f0[h] = (bk - r2[h] * nb) * 16;
        const int fl = f0[h] + rr + 8 * (mi & 1);  // this lane's ldmatrix row (position)
        lv[h] = h < nbk && fl < Fo;
        // row 2 r2, column c = 2 f (even: slot f)
        base[h] = tile_s + (2 * r2[h] * tr.slots + fl) * kPosStride + nt * 16;
      }
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int j = 0; j < 5; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t row = (lv[h] && toff[j] >= 0) ? base[h] + toff[j] : zero_s + nt * 16;
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(row, a0, a1, a2, a3);
          mma_16816(d[h], a0, a1, a2, a3, fw[2 * j], fw[2 * j + 1]);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h >= nbk) break;
        // the positions of this lane's accumulators: f0 + g, f0 + g + 8
        __nv_bfloat16* yr =
            y + ((b * To + t0 + r2[h]) * Fo + f0[h] + g) * C + c0 + 8 * nt + 2 * t;
        if (f0[h] + g < Fo)
          *reinterpret_cast<uint32_t*>(yr) = add_bf16x2(pack_bf16x2(d[h][0], d[h][1]), fw[10]);
        if (f0[h] + g + 8 < Fo)
          *reinterpret_cast<uint32_t*>(yr + 8 * static_cast<int64_t>(C)) =
              add_bf16x2(pack_bf16x2(d[h][2], d[h][3]), fw[10]);
      }
    }
  }
}

// Bytes of an NHWC tile of R rows of W columns with padding columns
// (dw_tile_mma's layout), then 64 zero bytes.
__host__ __device__ __forceinline__ int tile_bytes(int R, int W, int pad) {
  return R * tile_row(W + pad + 1).slots * kPosStride + 64;
}

// conv.0 position blocks (16 positions of one conv.0 row) a warp keeps the
// im2col fragments of in registers: R1 * ceil(F1 / 16) blocks over 8 warps,
// so F1 <= 80 (feat_in <= 158).
constexpr int kMaxBlk = 11;

// grid (row tiles, 1, B).  Row tile: kSubR2 depthwise rows (kFuse) or
// kSubR1 conv.0 rows, every channel, kSubCb at a time.  Shared memory: the
// mel rows the tile reads as f32 [nm][2 F1 + 1] (column j is frequency
// j - pad), then one channel block's conv.0 rows in dw_tile_mma's layout
// (F1 columns and the padding columns).  The mel tile and the im2col
// fragments built from it serve all C / kSubCb channel blocks.
template <bool kFuse>
__global__ void __launch_bounds__(kSubThreads, 2) conv0_dw_kernel(const SubConvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z;
  constexpr int R1 = kFuse ? 2 * kSubR2 + 1 : kSubR1;
  const int t2_0 = blockIdx.x * kSubR2;
  const int t1_0 = kFuse ? 2 * t2_0 - a.pad : blockIdx.x * kSubR1;  // first conv.0 row
  constexpr int nm = 2 * R1 + 1;                                     // mel rows
  const int fm = 2 * a.F1 + 1;                                       // mel columns
  const int tm0 = 2 * t1_0 - a.pad;                                  // first mel row
  float* mel = reinterpret_cast<float*>(smem);
  uint8_t* ctile = smem + ((static_cast<uint32_t>(nm) * fm * 4 + 15) & ~15u);
  const int Wt = a.F1 + a.pad + 1;  // conv.0 tile columns per row
  const TileRow tr = tile_row(Wt);
  uint8_t* zero = ctile + R1 * tr.slots * kPosStride;
  const int g = lane >> 2, t = lane & 3;
  pdl_wait();
  const int lenb = a.len ? a.len[b] - a.len_off : a.T;

  // 1. mel rows (zero outside the input and past the length), copied
  // asynchronously; lanes walk the layout's contiguous axis.  (The bf16
  // rounding of the input happens when the values are packed for the MMA.)
  {
    const float* src = a.mel + static_cast<int64_t>(b) * a.mel_bs;
    const int lim = min(a.T, lenb);
    if (a.mel_ts == 1) {
      for (int j = warp; j < fm; j += kSubWarps) {
        const int f = j - a.pad;
        const bool fok = f >= 0 && f < a.F;
        const float* col = src + static_cast<int64_t>(fok ? f : 0) * a.mel_fs;
        for (int i = lane; i < nm; i += 32) {
          const int tt = tm0 + i;
          const bool ok = fok && tt >= 0 && tt < lim;
          cp_async4(mel + i * fm + j, ok ? col + tt : a.mel, ok ? 4 : 0);
        }
      }
    } else {
      for (int i = warp; i < nm; i += kSubWarps) {
        const int tt = tm0 + i;
        const bool tok = tt >= 0 && tt < lim;
        const float* row = src + static_cast<int64_t>(tok ? tt : 0) * a.mel_ts;
        for (int j = lane; j < fm; j += 32) {
          const int f = j - a.pad;
          const bool ok = tok && f >= 0 && f < a.F;
          cp_async4(mel + i * fm + j, ok ? row + static_cast<int64_t>(f) * a.mel_fs : a.mel,
                    ok ? 4 : 0);
        }
      }
    }
    cp_async_wait_all();
    // the padding columns of the conv.0 tile and the zero row (never
    // written again)
    for (int idx = tid; idx < R1 * (a.pad + 1) * 4 + 4; idx += kSubThreads) {
      const int s = idx >> 2, q = idx & 3;
      const int r = s / (a.pad + 1), k = s - r * (a.pad + 1);
      uint8_t* dst =
          r < R1 ? ctile + (r * tr.slots + tile_slot(k < a.pad ? k : Wt - 1, tr.E)) * kPosStride
                 : zero;
      *reinterpret_cast<uint4*>(dst + 16 * q) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();

  // 2a. im2col fragments of this warp's blocks: block i = conv.0 row r,
  // positions f0 .. f0 + 15; this lane's rows f0 + g and f0 + g + 8, taps
  // 2t, 2t+1 (and tap 8 for t = 0, the only nonzero halves of the A
  // registers 2 and 3, kept as one word).  soff: the lane's store offset in the
  // conv.0 tile with bit 31 = row f0 + g valid, 30 = row f0 + g + 8 valid,
  // 29 = a conv.0 output row (else the depthwise conv's zero padding).
  const int nb1 = (a.F1 + 15) >> 4;
  const int nblk = R1 * nb1;
  uint32_t af[kMaxBlk][3], soff[kMaxBlk];
  {
    const int off0 = ((2 * t) / 3) * fm + (2 * t) % 3;
    const int off1 = ((2 * t + 1) / 3) * fm + (2 * t + 1) % 3;
    const int off8 = 2 * fm + 2;
#pragma unroll
    for (int i = 0; i < kMaxBlk; ++i) {
      const int blk = warp + kSubWarps * i;
      af[i][0] = af[i][1] = af[i][2] = 0u;
      soff[i] = 0u;
      if (blk < nblk) {
        const int r = blk / nb1;
        const int fa = (blk - r * nb1) * 16 + g, fb = fa + 8;
        const bool va = fa < a.F1, vb = fb < a.F1;
        const float* m = mel + 2 * r * fm;
        const float m8a = va ? m[2 * fa + off8] : 0.f, m8b = vb ? m[2 * fb + off8] : 0.f;
        if (va) af[i][0] = pack_bf16x2(m[2 * fa + off0], m[2 * fa + off1]);
        if (vb) af[i][1] = pack_bf16x2(m[2 * fb + off0], m[2 * fb + off1]);
        af[i][2] = t == 0 ? pack_bf16x2(m8a, m8b) : 0u;
        const bool live = t1_0 + r >= 0 && t1_0 + r < a.T1;
        soff[i] = static_cast<uint32_t>((r * tr.slots + tile_slot(fa + a.pad, tr.E)) * kPosStride +
                                        4 * t) |
                  (va ? 1u << 31 : 0u) | (vb ? 1u << 30 : 0u) | (live ? 1u << 29 : 0u);
      }
    }
  }

  for (int c0 = 0; c0 < a.C; c0 += kSubCb) {
    // 2b. conv.0 + bias + ReLU of channels c0 .. c0 + 31 on the tensor cores
    {
      // B fragments of n-tile nt (channels c0 + 8 nt + g; k = 2t, 2t+1 |
      // 2t+8): words 3 nt, 3 nt + 1; word 3 nt + 2 = the bias pair
      uint32_t fw[12];
      load_frag12(a.f0 + (c0 / kSubCb) * 32 * kSubFragWords, lane, fw);
#pragma unroll
      for (int i = 0; i < kMaxBlk; ++i) {
        if (warp + kSubWarps * i >= nblk) break;  // (warp-uniform)
        const uint32_t so = soff[i];
        const bool va = so >> 31, vb = (so >> 30) & 1u, live = (so >> 29) & 1u;
        uint8_t* sa = ctile + (so & 0x1fffffffu);
#pragma unroll
        for (int nt = 0; nt < kSubCb / 8; ++nt) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(d, af[i][0], af[i][1], af[i][2] & 0xffffu, af[i][2] >> 16, fw[3 * nt],
                    fw[3 * nt + 1]);
          const uint32_t oa =
              live ? max0_bf16x2(add_bf16x2(pack_bf16x2(d[0], d[1]), fw[3 * nt + 2])) : 0u;
          const uint32_t ob =
              live ? max0_bf16x2(add_bf16x2(pack_bf16x2(d[2], d[3]), fw[3 * nt + 2])) : 0u;
          if (va) *reinterpret_cast<uint32_t*>(sa + nt * 16) = oa;
          if (vb) *reinterpret_cast<uint32_t*>(sa + 4 * kPosStride + nt * 16) = ob;  // column + 8
        }
      }
    }
    __syncthreads();
    if (!kFuse) {
      // 3'. the conv.0 rows of these channels out, 16 bytes per thread
      for (int idx = tid; idx < R1 * a.F1 * 4; idx += kSubThreads) {
        const int pos = idx >> 2, q = idx & 3;
        const int r = pos / a.F1, f1 = pos - r * a.F1;
        if (t1_0 + r >= a.T1) break;
        *reinterpret_cast<uint4*>(
            a.out + ((static_cast<int64_t>(b) * a.T1 + t1_0 + r) * a.F1 + f1) * a.C + c0 + 8 * q) =
            *reinterpret_cast<const uint4*>(
                ctile + (r * tr.slots + tile_slot(f1 + a.pad, tr.E)) * kPosStride + 16 * q);
      }
    } else {
      // 3. depthwise 3x3 stride 2 + bias over the conv.0 rows
      dw_tile_mma(ctile, tr, a.F2, a.T2, t2_0, a.f1, zero, a.out, b, a.C, c0, warp, lane);
    }
    __syncthreads();  // the conv.0 tile is rewritten for the next channels
  }
}

// grid (row tiles, C / 32, B): output rows t0 .. t0 + kSubR2 - 1 of
// y [B][To][Fo][C] = depthwise 3x3 stride 2 (+ bias) of x [B][Ti][Fi][C];
// input rows 2 t0 - pad .. 2 t0 + 2 kSubR2 - pad staged in shared memory
// (zeros outside the input).
__global__ void __launch_bounds__(kSubThreads, 3) dw_s2_kernel(const __nv_bfloat16* __restrict__ x,
                                                               int Ti, int Fi, int C, int pad,
                                                               const uint32_t* __restrict__ frag,
                                                               __nv_bfloat16* __restrict__ y,
                                                               int To, int Fo) {
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.z;
  const int c0 = blockIdx.y * kSubCb;
  const int t0 = blockIdx.x * kSubR2;
  const int ti0 = 2 * t0 - pad;
  constexpr int R1 = 2 * kSubR2 + 1;
  const int Wt = Fi + pad + 1;
  const TileRow tr = tile_row(Wt);
  uint8_t* zero = smem + R1 * tr.slots * kPosStride;
  pdl_wait();
  // slots (row, column - pad) for columns [0, Wt) and the zero row, 16
  // bytes per copy, zero-filled outside the input
  const int items = (R1 * Wt + 1) * 4;
  {
    const int q = tid & 3;
    int slot = tid >> 2;
    int r = slot / Wt, cs = slot - r * Wt;
    for (int idx = tid; idx < items; idx += kSubThreads) {
      const int tt = ti0 + r, fi = cs - pad;
      const bool ok = r < R1 && tt >= 0 && tt < Ti && fi >= 0 && fi < Fi;
      cp_async16(smem + (r < R1 ? r * tr.slots + tile_slot(cs, tr.E) : R1 * tr.slots) * kPosStride +
                     16 * q,
                 ok ? x + ((b * Ti + tt) * Fi + fi) * C + c0 + 8 * q : x, ok ? 16 : 0);
      cs += kSubThreads / 4;
      while (cs >= Wt) {
        cs -= Wt;
        ++r;
      }
    }
    cp_async_wait_all();
  }
  __syncthreads();
  dw_tile_mma(smem, tr, Fo, To, t0, frag, zero, y, b, C, c0, warp, lane);
}

size_t dw_s2_smem(int Fi, int pad) { return tile_bytes(2 * kSubR2 + 1, Fi, pad); }

}  // namespace

size_t subsample_conv0_smem(int F1, bool fuse) {
  const int R1 = fuse ? 2 * kSubR2 + 1 : kSubR1;
  const size_t mel = (static_cast<size_t>(2 * R1 + 1) * (2 * F1 + 1) * 4 + 15) & ~size_t(15);
  return mel + tile_bytes(R1, F1, 2);
}

cudaError_t launch_subsample_conv0(const SubConvArgs& a, int B, bool fuse, cudaStream_t stream) {
  if (a.C % kSubCb != 0) return cudaErrorInvalidValue;
  const size_t smem = subsample_conv0_smem(a.F1, fuse);
  if (smem > static_cast<size_t>(kSubMaxSmem)) return cudaErrorInvalidValue;
  if (a.F1 > 16 * ((kMaxBlk * kSubWarps) / (fuse ? 2 * kSubR2 + 1 : kSubR1)))
    return cudaErrorInvalidValue;  // more conv.0 blocks than a warp keeps
  const int tiles = fuse ? (a.T2 + kSubR2 - 1) / kSubR2 : (a.T1 + kSubR1 - 1) / kSubR1;
  const dim3 grid(tiles, 1, B);
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
                                const uint32_t* frag, __nv_bfloat16* y, int To, int Fo,
                                int num_sms, cudaStream_t stream) {
  (void)num_sms;
  if (C % kSubCb != 0) return cudaErrorInvalidValue;
  const size_t smem = dw_s2_smem(Fi, pad);
  if (smem > static_cast<size_t>(kSubMaxSmem)) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> done{0};
  cudaError_t e = smem_attr_once(dw_s2_kernel, kSubMaxSmem, done);
  if (e != cudaSuccess) return e;
  const dim3 grid((To + kSubR2 - 1) / kSubR2, C / kSubCb, B);
  return launch_pdl(dw_s2_kernel, grid, dim3(kSubThreads), smem, stream, x, Ti, Fi, C, pad, frag,
                    y, To, Fo);
}

}  // namespace nrp
