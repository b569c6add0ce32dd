// gemm_tf32.cu -- Y[M,N] = X[M,K] . W[N,K]^T (+ bias[N]) in f32 on tcgen05.
//
// Serves LinearLayer::forward's Standard arm (reference:
// src/core/quantization.rs:128-135) for modules whose dtype is f32, at f32
// accuracy: each operand is split into a TF32 part and the rest,
// a = a_hi + a_lo with a_hi = a with its low 13 mantissa bits cleared (exact
// in TF32) and a_lo = a - a_hi (exact in f32; its TF32 rounding loses at
// most 2^-21 |a|), and the product is x_hi.w_hi + x_hi.w_lo + x_lo.w_hi --
// three kind::tf32 MMAs per K step accumulating in f32 in TMEM (the dropped
// x_lo.w_lo term is below 2^-20 |x w|).  Relative error per output is then
// about 1e-6 of the dot product's magnitude, inside the f32 modules' 1e-4
// parity bound, where one TF32 product alone (2^-11) is not.
//
// Tiling: one 128 x kBN output tile per CTA (kBN = 64, or 32 when 64-wide
// tiles would leave most SMs idle: config 0's projections have a single
// 128-row tile), K in 32-element stages (one 128-byte swizzle row of f32).
// A stage holds X and W as loaded, 5 (kBN = 64) or 7 (kBN = 32) deep; the
// lo parts go to four slots used in turn, each free again once the commit
// of its last K block's MMAs arrives.  That commit's latency, not the MMAs
// or the split, paced the pipeline when only two slots alternated.
//
// Warp roles (6 warps):
//   warp 0      TMA producer for X and W
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2-5   split each landed stage (hi in place, lo beside it; the
//               swizzle is elementwise so the layout carries over), then the
//               epilogue: TMEM -> registers -> + bias -> f32 rows.
#include "gemm.h"
#include "sm100.cuh"

namespace nrp {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 32;  // f32 elements per stage row: 128 bytes
constexpr int kMaxStages = 7;
constexpr int kLoSlots = 4;  // lo parts of the last 4 K blocks
constexpr int kThreads = 192;
constexpr int kSplitWarp0 = 2;
constexpr uint32_t kABytes = kBM * kBK * 4;  // 16 KB
template <int kBN>
struct Tf32Cfg {
  static constexpr uint32_t kBBytes = kBN * kBK * 4;  // 4 / 8 KB
  // a stage holds X and W as loaded (hi after the split, in place); the lo
  // parts go to one of two slots, free again once that stage's MMAs are done
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kBN == 64 ? 5 : 7;
  static constexpr size_t kSmem = 1024 + (kStages + kLoSlots) * kStageBytes + 256;
};
static_assert(Tf32Cfg<64>::kSmem <= 232448 && Tf32Cfg<32>::kSmem <= 232448,
              "shared memory budget");

struct Tf32Bars {
  uint64_t full[kMaxStages], split[kMaxStages], empty[kMaxStages], lofree[kLoSlots], done;
  uint32_t tmem_base;
  int abort;
};

// Bounded wait that polls (mbarrier.test_wait) instead of suspending: the
// stages hand over every few hundred nanoseconds, and a thread suspended in
// try_wait resumed too late for that (about 0.5 us per stage in a probe).
// After kWaitBudgetNs it records `code` in *err and returns false.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, int* err, int code) {
  auto test = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (test()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (test()) return true;
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Bounded polling wait whose outcome is the same for every lane of the warp.
__device__ __forceinline__ bool warp_all_wait(uint64_t* bar, uint32_t parity, int* err,
                                              int code) {
  return __all_sync(0xffffffffu, mbar_poll(bar, parity, err, code));
}

// a -> (a with the low 13 mantissa bits cleared, a minus that), elementwise
__device__ __forceinline__ void split4(uint4& hi, uint4& lo) {
  const uint32_t m = 0xFFFFE000u;
  const uint4 h = make_uint4(hi.x & m, hi.y & m, hi.z & m, hi.w & m);
  lo = make_uint4(__float_as_uint(__uint_as_float(hi.x) - __uint_as_float(h.x)),
                  __float_as_uint(__uint_as_float(hi.y) - __uint_as_float(h.y)),
                  __float_as_uint(__uint_as_float(hi.z) - __uint_as_float(h.z)),
                  __float_as_uint(__uint_as_float(hi.w) - __uint_as_float(h.w)));
  hi = h;
}

template <int kBN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_x,  // [M, K] f32, box (32, 128)
                       const __grid_constant__ CUtensorMap map_w,  // [N, K] f32, box (32, kBN)
                       const float* __restrict__ bias, float* __restrict__ y, int ldy, int M,
                       int N, int K, int* err) {
  using Cfg = Tf32Cfg<kBN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  Tf32Bars* bars = reinterpret_cast<Tf32Bars*>(base + (kStages + kLoSlots) * Cfg::kStageBytes);
  // stage s: X at sx(s), W at sw(s); lo slot q: X lo at sx(kStages + q), W lo at sw(...)
  auto sx = [&](int s) { return base + s * Cfg::kStageBytes; };
  auto sw = [&](int s) { return base + s * Cfg::kStageBytes + kABytes; };

  const int warp = warp_id(), lane = lane_id();
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int num_kb = K / kBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->split[s], 4);
      mbar_init(&bars->empty[s], 1);
    }
    for (int q = 0; q < kLoSlots; ++q) mbar_init(&bars->lofree[q], 1);
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&map_x);
      prefetch_tensormap(&map_w);
      for (int kb = 0; kb < num_kb && !*abort_flag; ++kb) {
        const int s = kb % kStages;
        const uint32_t round = kb / kStages;
        if (kb >= kStages && !mbar_wait(&bars->empty[s], (round & 1) ^ 1, err, kDevTimeoutLoad)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&bars->full[s], kABytes + Cfg::kBBytes);
        tma_load_2d(sx(s), &map_x, &bars->full[s], kb * kBK, m0);
        tma_load_2d(sw(s), &map_w, &bars->full[s], kb * kBK, n0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32_f32(kBM, kBN);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % kStages;
        const uint32_t round = kb / kStages;
        if (*abort_flag || !mbar_poll(&bars->split[s], round & 1, err, kDevTimeoutLoad)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t xh = smem_u32(sx(s)), xl = smem_u32(sx(kStages + kb % kLoSlots));
        const uint32_t wh = smem_u32(sw(s)), wl = smem_u32(sw(kStages + kb % kLoSlots));
#pragma unroll
        for (int k = 0; k < kBK / 8; ++k) {  // 8 TF32 (32 bytes) per MMA
          const uint32_t o = k * 32;
          umma_tf32_ss(tmem, sdesc_sw128(xl + o, 16, 1024), sdesc_sw128(wh + o, 16, 1024),
                       idesc, (kb | k) != 0);
          umma_tf32_ss(tmem, sdesc_sw128(xh + o, 16, 1024), sdesc_sw128(wl + o, 16, 1024),
                       idesc, 1);
          umma_tf32_ss(tmem, sdesc_sw128(xh + o, 16, 1024), sdesc_sw128(wh + o, 16, 1024),
                       idesc, 1);
        }
        umma_commit(&bars->empty[s]);
        umma_commit(&bars->lofree[kb % kLoSlots]);
      }
      if (ok) umma_commit(&bars->done);
    }
  } else {
    // ---------------------------------------- split, then the epilogue
    const int t = threadIdx.x - kSplitWarp0 * 32;  // 0..127
    constexpr int kVec = (kABytes + Cfg::kBBytes) / 16;
    bool ok = true;
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % kStages;
      const uint32_t round = kb / kStages;
      const int q = kb % kLoSlots;  // lo slot, last read by the MMAs of block kb - kLoSlots
      ok = warp_all_wait(&bars->full[s], round & 1, err, kDevTimeoutLoad) &&
           (kb < kLoSlots || warp_all_wait(&bars->lofree[q], (kb / kLoSlots - 1) & 1, err,
                                           kDevTimeoutMma)) &&
           !*abort_flag;
      if (!ok) break;
      // X: vectors [0, kVecA) of the stage, then W; the same offsets in the
      // slot.  A fixed trip count, so the loads of a thread go out together.
      static_assert(kVec % 128 == 0, "split: whole rounds of 128 threads");
      uint4 hv[kVec / 128], lv[kVec / 128];
#pragma unroll
      for (int r = 0; r < kVec / 128; ++r)
        hv[r] = *reinterpret_cast<const uint4*>(sx(s) + (t + 128 * r) * 16);
#pragma unroll
      for (int r = 0; r < kVec / 128; ++r) split4(hv[r], lv[r]);
#pragma unroll
      for (int r = 0; r < kVec / 128; ++r) {
        *reinterpret_cast<uint4*>(sx(s) + (t + 128 * r) * 16) = hv[r];
        *reinterpret_cast<uint4*>(sx(kStages + q) + (t + 128 * r) * 16) = lv[r];
      }
      fence_proxy_async_smem();  // the MMAs read what this thread wrote
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->split[s]);
    }
    if (!ok) *abort_flag = 1;
    // epilogue: warp (2..5) reads TMEM lane quadrant warp & 3
    if (ok && warp_all_wait(&bars->done, 0, err, kDevTimeoutMma)) {
      tc_fence_after();
      const int quad = warp & 3;
      const int row = m0 + quad * 32 + lane;
      float* yr = y + static_cast<int64_t>(row) * ldy;
      const bool vec = (ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c, r);
        tmem_ld_wait();
        const int n = n0 + c;
        if (row >= M || n >= N) continue;
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          v[e] = __uint_as_float(r[e]) + (bias && n + e < N ? bias[n + e] : 0.f);
        if (vec && n + 32 <= N) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(yr + n + 4 * q) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (n + e < N) yr[n + e] = v[e];
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBN);
  }
}

template <int kBN>
cudaError_t launch_bn(const float* x, int M, int K, const float* w, int N, const float* bias,
                      float* y, int ldy, int* err, cudaStream_t stream) {
  static std::atomic<uint64_t> attr{0};
  if (cudaError_t e = smem_attr_once(gemm_tf32x3_kernel<kBN>,
                                     static_cast<int>(Tf32Cfg<kBN>::kSmem), attr))
    return e;
  CUtensorMap map_x, map_w;
  if (!make_tmap_2d(&map_x, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, M,
                    static_cast<uint64_t>(K) * 4, kBK, kBM, true) ||
      !make_tmap_2d(&map_w, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K, N,
                    static_cast<uint64_t>(K) * 4, kBK, kBN, true))
    return cudaErrorInvalidValue;
  const dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
  return launch_pdl(gemm_tf32x3_kernel<kBN>, grid, dim3(kThreads), Tf32Cfg<kBN>::kSmem, stream,
                    map_x, map_w, bias, y, ldy, M, N, K, err);
}

}  // namespace

bool gemm_tf32_supported(int M, int K, int N, const void* x, const void* w) {
  return M > 0 && N > 0 && K >= kBK && K % kBK == 0 && M <= 65535 * kBM &&
         ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
}

cudaError_t launch_gemm_tf32x3(const float* x, int M, int K, const float* w, int N,
                               const float* bias, float* y, int ldy, int num_sms, int* err,
                               cudaStream_t stream) {
  if (!gemm_tf32_supported(M, K, N, x, w) || ldy < N) return cudaErrorInvalidValue;
  // 64-wide tiles when they fill the SMs, else 32-wide (twice the CTAs)
  const long tiles64 = static_cast<long>((M + kBM - 1) / kBM) * ((N + 63) / 64);
  if (tiles64 >= (num_sms > 0 ? num_sms : 148))
    return launch_bn<64>(x, M, K, w, N, bias, y, ldy, err, stream);
  return launch_bn<32>(x, M, K, w, N, bias, y, ldy, err, stream);
}

}  // namespace nrp
