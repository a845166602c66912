// Row geometry ladder shared by the kernels that keep a whole row in
// registers between two passes over it (RMSNorm, softmax).
//
// A row of `nvec` 16-byte packs is owned by TPR consecutive threads, each
// holding VPT packs in registers, so a row costs one HBM read and one HBM
// write.  Rows of up to 32 packs use one pack per thread (4..32 threads);
// the ladder then deepens each thread up to MAX_VPT packs, then adds
// threads (up to 1024 per row).  Longer rows go to the looped kernels,
// which re-read the row from L2.
//
// The kernels are launched with one CTA per group of rows (a full grid, not
// a persistent one): measured on B200 at 131072 x 4096 bf16 rows, a full
// grid of (64 threads x 8 packs) rows streams RMSNorm at 6.8 TB/s and a full
// grid of (256 x 2) rows streams the two-input add+RMSNorm at 6.9 TB/s,
// against 6.0 and 5.0 TB/s for persistent grids.  MAX_VPT picks that depth
// per kernel (fewer packs per thread when a row has two input streams).
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
// rung that holds nvec packs with at most MAX_VPT packs per thread; returns
// -1 when the row is too long for the ladder.
template <int MAX_VPT, typename F>
int row_ladder(int64_t nvec, F&& f) {
  using std::integral_constant;
  static_assert(MAX_VPT == 2 || MAX_VPT == 4 || MAX_VPT == 8 || MAX_VPT == 16,
                "ladder depth is 2, 4, 8 or 16 packs");
  constexpr int V = MAX_VPT;
  if (nvec <= 4) return f(integral_constant<int, 4>{}, integral_constant<int, 1>{});
  if (nvec <= 8) return f(integral_constant<int, 8>{}, integral_constant<int, 1>{});
  if (nvec <= 16) return f(integral_constant<int, 16>{}, integral_constant<int, 1>{});
  if (nvec <= 32) return f(integral_constant<int, 32>{}, integral_constant<int, 1>{});
  if (nvec <= 64) return f(integral_constant<int, 32>{}, integral_constant<int, 2>{});
  if constexpr (V >= 4)
    if (nvec <= 128) return f(integral_constant<int, 32>{}, integral_constant<int, 4>{});
  if constexpr (V >= 8)
    if (nvec <= 256) return f(integral_constant<int, 32>{}, integral_constant<int, 8>{});
  if constexpr (V >= 16)
    if (nvec <= 512) return f(integral_constant<int, 32>{}, integral_constant<int, 16>{});
  if (nvec <= 64 * V) return f(integral_constant<int, 64>{}, integral_constant<int, V>{});
  if (nvec <= 128 * V) return f(integral_constant<int, 128>{}, integral_constant<int, V>{});
  if (nvec <= 256 * V) return f(integral_constant<int, 256>{}, integral_constant<int, V>{});
  if (nvec <= 512 * V) return f(integral_constant<int, 512>{}, integral_constant<int, V>{});
  if constexpr (V <= 4)
    if (nvec <= 1024 * V) return f(integral_constant<int, 1024>{}, integral_constant<int, V>{});
  return -1;
}

}  // namespace flb200
