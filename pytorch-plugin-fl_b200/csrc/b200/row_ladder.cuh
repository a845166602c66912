// Row geometry ladder shared by the kernels that keep a whole row in
// registers between two passes over it (RMSNorm, softmax).
//
// A row of `nvec` 16-byte packs is owned by TPR consecutive threads, each
// holding VPT packs in registers, so a row costs one HBM read and one HBM
// write.  Rows of up to 4 packs use 4 threads; the ladder then widens the
// per-thread depth to 16 packs (256 bytes in flight per thread) before it
// adds threads, and stops at 64 KB rows.  Longer
// rows go to the looped kernels, which re-read the row from L2.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace flb200 {

template <int TPR>
constexpr int ladder_block() {
  return TPR >= 256 ? TPR : 256;
}

// At least two 256-thread CTAs per SM (<= 128 registers per thread): a row
// of 16 packs then lives in 64 registers and the rest fits beside it.
template <int BLOCK>
constexpr int ladder_min_blocks() {
  return BLOCK <= 256 ? 2 : 1;
}

// Calls f(integral_constant<TPR>, integral_constant<VPT>) for the smallest
// ladder rung that holds nvec packs with at most MAX_VPT packs per thread;
// returns -1 when the row is too long for the ladder.
template <int MAX_VPT = 16, typename F>
int row_ladder(int64_t nvec, F&& f) {
  using std::integral_constant;
  static_assert(MAX_VPT == 8 || MAX_VPT == 16, "ladder depth is 8 or 16 packs");
  if (nvec <= 4) return f(integral_constant<int, 4>{}, integral_constant<int, 1>{});
  if (nvec <= 8) return f(integral_constant<int, 8>{}, integral_constant<int, 1>{});
  if (nvec <= 16) return f(integral_constant<int, 16>{}, integral_constant<int, 1>{});
  if (nvec <= 32) return f(integral_constant<int, 32>{}, integral_constant<int, 1>{});
  if (nvec <= 64) return f(integral_constant<int, 32>{}, integral_constant<int, 2>{});
  if (nvec <= 128) return f(integral_constant<int, 32>{}, integral_constant<int, 4>{});
  if (nvec <= 256) return f(integral_constant<int, 32>{}, integral_constant<int, 8>{});
  if constexpr (MAX_VPT == 16) {
    if (nvec <= 512) return f(integral_constant<int, 32>{}, integral_constant<int, 16>{});
    if (nvec <= 1024) return f(integral_constant<int, 64>{}, integral_constant<int, 16>{});
    if (nvec <= 2048) return f(integral_constant<int, 128>{}, integral_constant<int, 16>{});
    if (nvec <= 4096) return f(integral_constant<int, 256>{}, integral_constant<int, 16>{});
  } else {
    if (nvec <= 512) return f(integral_constant<int, 64>{}, integral_constant<int, 8>{});
    if (nvec <= 1024) return f(integral_constant<int, 128>{}, integral_constant<int, 8>{});
    if (nvec <= 2048) return f(integral_constant<int, 256>{}, integral_constant<int, 8>{});
    if (nvec <= 4096) return f(integral_constant<int, 512>{}, integral_constant<int, 8>{});
  }
  return -1;
}

}  // namespace flb200
