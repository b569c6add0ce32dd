// masks.cuh -- the visible key interval of one query row, shared by the
// CUDA-core and tensor-core streaming kernels.
#pragma once

#include "gemm.h"

namespace nrp {

// Visible key interval [lo, hi) of query row i: the AttentionContext window
// (attention.rs:232-272 / conformer.rs:97-221 on absolute positions), the
// key padding bound (attention.rs:280-294) and the unfilled-cache offset
// (conformer.rs:153-181).  Returns false when the row sees no key.
__device__ __forceinline__ bool key_interval(const AttnContextDev& ctx, const StreamMaskDev& sm,
                                             int i, int kend, int& lo, int& hi) {
  lo = 0;
  hi = kend;
  int ia = i;
  int has = ctx.has, left = ctx.left, right = ctx.right, chunked = ctx.chunked;
  if (sm.has) {
    if (i >= sm.valid) return false;
    ia = sm.cache_len + i;
    lo = max(lo, sm.cache_len - sm.filled);
    has = sm.ctx_has;
    left = sm.left;
    right = sm.right;
    chunked = sm.chunked;
  }
  if (has) {
    if (chunked && right >= 0) {
      const int chunk = right + 1;
      const int lc = left >= 0 ? left / chunk : 10000;
      const int ci = ia / chunk;
      lo = max(lo, (ci - lc) * chunk);
      hi = min(hi, (ci + 1) * chunk);
    } else {
      if (left >= 0) lo = max(lo, ia - left);
      if (!chunked && right >= 0) hi = min(hi, ia + right + 1);
    }
  }
  return hi > lo;
}

}  // namespace nrp
