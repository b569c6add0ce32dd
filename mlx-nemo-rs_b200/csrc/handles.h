// handles.h -- definitions of the C ABI's opaque handles and the small
// host-side types they hold (internal to the library).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/nemo_relpos.h"

namespace nrp {

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  cudaError_t ensure(size_t n) {
    if (n <= bytes && p) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, n ? n : 16);
    if (e == cudaSuccess) bytes = n;
    return e;
  }
  template <typename T>
  T* as() const { return static_cast<T*>(p); }
};

struct Linear {
  bool loaded = false;
  bool quant = false;
  int bits = 8, group = 64;
  std::vector<float> w;        // f32 master [N, K] (standard)
  std::vector<uint32_t> wq;    // packed [N, K*bits/32] (quantised)
  std::vector<float> qs, qb;   // [N, K/group]
  std::vector<float> bias;     // [N] or empty
};

// Optional per-launch timing: CUDA events recorded on the launching stream
// around each kernel the library launches, summed per kernel kind.
struct ProfRec {
  int kind;
  cudaEvent_t start, stop;
};

// Sets this thread's nrp_last_error() message and returns `code`.
int report_error(int code, const char* msg);

// Looks up, on `device` (the current device), the device address of the
// static array nrp_attn_forward_noalloc keeps its intermediates in
// (noalloc.cu).  The array lives in a module of its own, which the CUDA
// runtime loads -- committing the array's device memory -- on this first
// use; nrp_context_create calls it so that no noalloc call ever does.
int noalloc_scratch_prepare(int device);

}  // namespace nrp

// d_err[0]: the sticky device error code; then kSchedSlots pairs of ints,
// the item counters of persistent kernels (each left zero by its launch;
// consecutive launches take consecutive pairs).
constexpr int kSchedSlots = 32;
constexpr int kCtxInts = 2 + 2 * kSchedSlots;

struct nrp_context {
  int device = 0;
  int num_sms = 148;
  int* d_err = nullptr;
  uint32_t sched_seq = 0;
  bool prof = false;
  std::vector<nrp::ProfRec> recs;
  std::vector<cudaEvent_t> pool;
  double prof_ms[NRP_KERNEL_KINDS] = {};
  int64_t prof_n[NRP_KERNEL_KINDS] = {};
  std::vector<std::pair<int, float>> prof_log;  // (kind, ms) per launch, issue order
  // bf16 copy of one quantised weight for the large-M quantised GEMM
  // (stream-ordered: reused by every such call on the context)
  nrp::DevBuf wscratch;
  nrp::DevBuf wscratch_side;  // the same for work on `side`
  // bf16 copies of quantised weights made ahead of time (the encoder
  // dequantises the next layer while the current one runs): a quantised
  // linear whose code pointer is listed uses the copy.  Set and cleared by
  // the caller around the launches it covers, which must be stream-ordered
  // after the copies were written.
  std::vector<std::pair<const void*, const void*>> predeq;
  // bf16 copies of quantised weights kept for the weights' lifetime, keyed
  // by the device address of their codes: a quantised linear with many rows
  // uses its copy instead of dequantising the whole weight again every
  // call.  A module drops its entries when it re-uploads or frees the codes
  // (deq_forget), so a reused address never matches a stale copy.
  bool deq_cache_on = true;
  std::unordered_map<const void*, std::unique_ptr<nrp::DevBuf>> deq_cache;
  // expires with the context: modules destroyed after it leave its table alone
  std::shared_ptr<bool> alive = std::make_shared<bool>(true);
  // a second stream for work that overlaps the caller's (forked and joined
  // with events, so the caller's stream order is kept)
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

struct nrp_attn {
  nrp_context* ctx = nullptr;
  int device = 0;  // ctx->device, kept for teardown
  std::weak_ptr<bool> ctx_alive;
  int D = 0, H = 0, dh = 0;
  int use_bias = 1;
  int dtype = NRP_DTYPE_F32;
  int cache_drop = 0;
  nrp::Linear lin[5];
  std::vector<float> u, v;
  std::vector<uint32_t> uv_packed;  // [H][128] bf16 pairs of the rounded u, v (AttnUV)
  bool dirty = true;
  // device parameters in the module dtype
  bool qkv_quant = false;
  nrp::DevBuf w_qkv, s_qkv, z_qkv, b_qkv;  // weights (or u8 codes), scales, zero-points, bias
  bool has_b_qkv = false;
  nrp::DevBuf w_out, s_out, z_out, b_out;
  bool out_quant = false, has_b_out = false;
  nrp::DevBuf w_pos, s_pos, z_pos;
  bool pos_quant = false;
  nrp::DevBuf u_dev, v_dev;
  // workspace
  nrp::DevBuf qkv, cbuf, pbuf;
  // projected streaming positions, reused while pos_len is unchanged
  int spos_len = -1;
  nrp::DevBuf spos;
};

struct nrp_cache {
  nrp_attn* attn = nullptr;
  int device = 0;  // attn's device, kept for teardown
  int B = 0, C = 0, D = 0, dtype = 0;
  int head = 0;  // ring slot of the oldest frame
  nrp::DevBuf kc, vc, hc;
  nrp::DevBuf tmp;
};

// Sequence-split communicator (halo.cpp).  `comm` is the ncclComm_t; the
// exchange runs on its own high-priority stream so that it overlaps the
// attention of the query tiles that need no halo.
struct nrp_halo {
  nrp_context* ctx = nullptr;
  void* comm = nullptr;
  int rank = 0, nranks = 1;
  int timeout_ms = 10000;
  bool dead = false;  // aborted after a timeout or an NCCL error
  cudaStream_t stream = nullptr;
  cudaEvent_t ready = nullptr, done = nullptr;
  nrp::DevBuf buf;  // time-major q|k|v [halo + len + halo][batch][3 d_model]
};

namespace nrp {
// The counter pair of the next persistent-kernel launch on this context.
inline int* sched_slot(nrp_context* c) {
  return c->d_err + 2 + 2 * static_cast<int>(c->sched_seq++ % kSchedSlots);
}

// Queues on halo->stream, after the work queued so far on `st`: for side s
// (0: rank - 1, 1: rank + 1; skipped when that rank does not exist or both
// byte counts are 0) send send_bytes[s] bytes from buf + send_off[s] and
// receive recv_bytes[s] bytes into buf + recv_off[s] (one NCCL group); then
// records halo->done.  Offsets in bytes into halo->buf.
int halo_exchange(nrp_halo* halo, const size_t send_off[2], const size_t send_bytes[2],
                  const size_t recv_off[2], const size_t recv_bytes[2], cudaStream_t st);
}  // namespace nrp
