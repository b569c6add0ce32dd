// halo.cpp -- the NCCL side of the sequence-split forward
// (nrp_attn_forward_seq_sharded): the communicator and the halo exchange.
//
// A windowed attention over a sequence cut into one contiguous segment per
// GPU needs, on each rank, the keys and values of the frames its window
// reaches on the neighbouring segments.  The ranks exchange those rows with
// one grouped ncclSend/ncclRecv per step (NVLink peer-to-peer); the rows
// travel as whole time-major q|k|v rows, so each side is one contiguous block
// for every utterance of the batch.
//
// NCCL is loaded with dlopen on first use (libnccl.so.2 -- in a process that
// already runs torch this is the copy torch loaded), so the library itself
// loads on machines without NCCL.  The communicator is non-blocking: every
// host-side wait (joining, queueing a group, a step's completion in
// nrp_halo_comm_check) is bounded by the communicator's timeout, after which
// it is aborted (ncclCommAbort also ends its kernels) and reports
// NRP_ERR_DEVICE.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>

#include "handles.h"

namespace {

using Clock = std::chrono::steady_clock;

int report(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return nrp::report_error(code, buf);
}

struct Nccl {
  bool loaded = false;
  std::string why;
  int version = 0;
  decltype(&ncclGetVersion) GetVersion = nullptr;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&ncclCommFinalize) CommFinalize = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  decltype(&ncclSend) Send = nullptr;
  decltype(&ncclRecv) Recv = nullptr;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!so) so = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!so) {
      const char* e = dlerror();
      n.why = e ? e : "libnccl.so.2 not found";
      return;
    }
#define NRP_NCCL_SYM(field, name)                                        \
  n.field = reinterpret_cast<decltype(n.field)>(dlsym(so, name));        \
  if (!n.field) {                                                        \
    n.why = "libnccl has no " name;                                      \
    return;                                                              \
  }
    NRP_NCCL_SYM(GetVersion, "ncclGetVersion")
    NRP_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
    NRP_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
    NRP_NCCL_SYM(CommFinalize, "ncclCommFinalize")
    NRP_NCCL_SYM(CommDestroy, "ncclCommDestroy")
    NRP_NCCL_SYM(CommAbort, "ncclCommAbort")
    NRP_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
    NRP_NCCL_SYM(GetErrorString, "ncclGetErrorString")
    NRP_NCCL_SYM(GroupStart, "ncclGroupStart")
    NRP_NCCL_SYM(GroupEnd, "ncclGroupEnd")
    NRP_NCCL_SYM(Send, "ncclSend")
    NRP_NCCL_SYM(Recv, "ncclRecv")
#undef NRP_NCCL_SYM
    if (n.GetVersion(&n.version) != ncclSuccess) {
      n.why = "ncclGetVersion failed";
      return;
    }
    n.loaded = true;
  });
  return n;
}

int need_nccl(Nccl** out) {
  Nccl& n = nccl();
  if (!n.loaded) return report(NRP_ERR_UNSUPPORTED, "NCCL is not available: %s", n.why.c_str());
  *out = &n;
  return NRP_OK;
}

// Polls the communicator until it leaves ncclInProgress or `deadline`
// passes (then *late = true and ncclInProgress is returned).
ncclResult_t settle(Nccl& n, ncclComm_t c, Clock::time_point deadline, bool* late) {
  *late = false;
  for (;;) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t r = n.CommGetAsyncError(c, &st);
    if (r != ncclSuccess) return r;
    if (st != ncclInProgress) return st;
    if (Clock::now() > deadline) {
      *late = true;
      return ncclInProgress;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

Clock::time_point deadline_of(const nrp_halo* h) {
  return Clock::now() + std::chrono::milliseconds(h->timeout_ms);
}

// Aborts the communicator (ending its kernels) and marks the handle dead.
void abort_comm(nrp_halo* h) {
  if (h->comm && !h->dead) {
    Nccl& n = nccl();
    n.CommAbort(static_cast<ncclComm_t>(h->comm));
  }
  h->comm = nullptr;
  h->dead = true;
}

}  // namespace

namespace nrp {

int halo_exchange(nrp_halo* h, const size_t send_off[2], const size_t send_bytes[2],
                  const size_t recv_off[2], const size_t recv_bytes[2], cudaStream_t st) {
  if (h->dead) return report(NRP_ERR_DEVICE, "the halo communicator was aborted");
  Nccl* n = nullptr;
  if (int rc = need_nccl(&n)) return rc;
  const size_t cap = h->buf.bytes;
  for (int s = 0; s < 2; ++s)
    if (send_off[s] + send_bytes[s] > cap || recv_off[s] + recv_bytes[s] > cap)
      return report(NRP_ERR_INVALID, "halo rows outside the buffer");
  cudaError_t e = cudaEventRecord(h->ready, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(h->stream, h->ready, 0);
  if (e != cudaSuccess) return report(NRP_ERR_CUDA, "halo stream order: %s", cudaGetErrorString(e));
  ncclComm_t c = static_cast<ncclComm_t>(h->comm);
  uint8_t* buf = static_cast<uint8_t*>(h->buf.p);
  ncclResult_t r = n->GroupStart();
  for (int s = 0; s < 2 && r == ncclSuccess; ++s) {
    const int peer = s == 0 ? h->rank - 1 : h->rank + 1;
    if (peer < 0 || peer >= h->nranks) continue;
    if (send_bytes[s] && r == ncclSuccess)
      r = n->Send(buf + send_off[s], send_bytes[s], ncclUint8, peer, c, h->stream);
    if (recv_bytes[s] && r == ncclSuccess)
      r = n->Recv(buf + recv_off[s], recv_bytes[s], ncclUint8, peer, c, h->stream);
  }
  const ncclResult_t r_end = n->GroupEnd();
  if (r == ncclSuccess) r = r_end;
  bool late = false;
  if (r == ncclInProgress) r = settle(*n, c, deadline_of(h), &late);
  if (late) {
    abort_comm(h);
    return report(NRP_ERR_DEVICE, "rank %d: queueing the halo exchange took more than %d ms; "
                  "communicator aborted", h->rank, h->timeout_ms);
  }
  if (r != ncclSuccess) {
    const char* why = n->GetErrorString(r);
    abort_comm(h);
    return report(NRP_ERR_DEVICE, "rank %d: halo exchange failed: %s", h->rank, why);
  }
  e = cudaEventRecord(h->done, h->stream);
  if (e != cudaSuccess) return report(NRP_ERR_CUDA, "halo event: %s", cudaGetErrorString(e));
  return NRP_OK;
}

}  // namespace nrp

extern "C" {

int nrp_halo_unique_id(unsigned char id[NRP_HALO_ID_BYTES]) {
  if (!id) return report(NRP_ERR_INVALID, "null id");
  Nccl* n = nullptr;
  if (int rc = need_nccl(&n)) return rc;
  ncclUniqueId u;
  const ncclResult_t r = n->GetUniqueId(&u);
  if (r != ncclSuccess)
    return report(NRP_ERR_CUDA, "ncclGetUniqueId: %s", n->GetErrorString(r));
  static_assert(sizeof(u.internal) == NRP_HALO_ID_BYTES, "NCCL unique id size");
  memcpy(id, u.internal, NRP_HALO_ID_BYTES);
  return NRP_OK;
}

int nrp_halo_comm_create(nrp_context* ctx, const unsigned char id[NRP_HALO_ID_BYTES], int rank,
                         int nranks, int timeout_ms, nrp_halo** out) {
  if (!ctx || !id || !out) return report(NRP_ERR_INVALID, "null argument");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return report(NRP_ERR_INVALID, "rank %d of %d", rank, nranks);
  if (timeout_ms <= 0) return report(NRP_ERR_INVALID, "timeout_ms must be positive");
  Nccl* n = nullptr;
  if (int rc = need_nccl(&n)) return rc;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return report(NRP_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  auto* h = new nrp_halo;
  h->ctx = ctx;
  h->rank = rank;
  h->nranks = nranks;
  h->timeout_ms = timeout_ms;
  ncclUniqueId u;
  memcpy(u.internal, id, NRP_HALO_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  ncclResult_t r = n->CommInitRankConfig(&c, nranks, u, rank, &cfg);
  bool late = false;
  if ((r == ncclSuccess || r == ncclInProgress) && c) {
    h->comm = c;
    r = settle(*n, c, deadline_of(h), &late);
  }
  if (late || r != ncclSuccess || !c) {
    const char* why = late ? "not every rank joined in time" : n->GetErrorString(r);
    abort_comm(h);
    delete h;
    return report(NRP_ERR_DEVICE, "rank %d of %d: communicator not formed within %d ms: %s",
                  rank, nranks, timeout_ms, why);
  }
  int least = 0, greatest = 0;
  e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
  if (e == cudaSuccess)
    e = cudaStreamCreateWithPriority(&h->stream, cudaStreamNonBlocking, greatest);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->done, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    nrp_halo_comm_destroy(h);
    return report(NRP_ERR_CUDA, "halo stream/events: %s", cudaGetErrorString(e));
  }
  *out = h;
  return NRP_OK;
}

int nrp_halo_comm_check(nrp_halo* h, void* stream) {
  if (!h) return report(NRP_ERR_INVALID, "null halo");
  if (h->dead) return report(NRP_ERR_DEVICE, "the halo communicator was aborted");
  Nccl* n = nullptr;
  if (int rc = need_nccl(&n)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ncclComm_t c = static_cast<ncclComm_t>(h->comm);
  const Clock::time_point deadline = deadline_of(h);
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return NRP_OK;
    if (e != cudaErrorNotReady) return report(NRP_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
    ncclResult_t as = ncclSuccess;
    if (n->CommGetAsyncError(c, &as) == ncclSuccess && as != ncclSuccess && as != ncclInProgress) {
      const char* why = n->GetErrorString(as);
      abort_comm(h);
      return report(NRP_ERR_DEVICE, "rank %d: NCCL error %s; communicator aborted", h->rank, why);
    }
    if (Clock::now() > deadline) {
      abort_comm(h);
      return report(NRP_ERR_DEVICE, "rank %d: step not finished within %d ms (a peer did not "
                    "send its halo); communicator aborted", h->rank, h->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

int nrp_halo_comm_destroy(nrp_halo* h) {
  if (!h) return NRP_OK;
  int rc = NRP_OK;
  if (h->comm && !h->dead) {
    Nccl& n = nccl();
    ncclComm_t c = static_cast<ncclComm_t>(h->comm);
    ncclResult_t r = n.CommFinalize(c);
    bool late = false;
    if (r == ncclSuccess || r == ncclInProgress) r = settle(n, c, deadline_of(h), &late);
    if (late || r != ncclSuccess) {
      abort_comm(h);
      rc = report(NRP_ERR_DEVICE, "rank %d: communicator did not finalize; aborted", h->rank);
    } else {
      n.CommDestroy(c);
      h->comm = nullptr;
    }
  }
  if (h->stream) cudaStreamDestroy(h->stream);
  if (h->ready) cudaEventDestroy(h->ready);
  if (h->done) cudaEventDestroy(h->done);
  delete h;
  return rc;
}

}  // extern "C"
