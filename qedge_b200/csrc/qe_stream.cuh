// qe_stream.cuh — data layout of the streaming sampler (qe_sample_stream.cu).
//
// The sampler runs as two launches.  The summary kernel streams every row of
// logits from HBM once, one warp per task of `tpw` tiles of 1024 ids inside a
// canonical slice, and reduces each 32-id group (the canonical layout of
// qe_common.cuh) to a GroupSum.  The row kernel (one CTA per row) works from
// those summaries: row max, softmax normaliser, the exponential race, the
// kept-set test and the exact fallback, re-reading from global memory only
// the groups that can matter.
#pragma once
#include <cstddef>
#include <cstdint>

#include "qe_common.cuh"

namespace qe {
namespace st {

constexpr int kSumThreads = 256;              // summary kernel: threads per CTA (8 warp tasks)
constexpr int kRowThreads = 256;              // row kernel: threads per CTA (one row)
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kTC = 4;                        // race candidates tested for kept-set membership
constexpr int kSmallK = 64;                   // top-k rows up to this k take the direct top-k path
constexpr int kGrpCap = 1024;                 // direct top-k: groups collected
constexpr int kSelCap = 4096;                 // direct top-k: elements collected
constexpr int kSortCap = 512;                 // direct top-k: elements sorted
constexpr int kHashCap = 8192;                // history ids hashed per row (repetition penalty)

enum RowKind : int { kKindGreedy = 0, kKindArgmax = 1, kKindRace = 2, kKindSmallK = 3 };

// Summary of one 32-id group.  aux is the group-relative sum
// fsum = sum_j 2^(x_j c1 - RN(gmax c1)) of a row that samples, or, for rows
// that only need the position of the max (greedy and top_k = 1 rows) and for
// groups whose max is NaN or +inf, the member index (0..31, stored as an int)
// of the group's first element equal to gmax (the first NaN for NaN).
struct alignas(8) GroupSum {
  float gmax;   // NaN-propagating max of the (penalised) logits; -inf for a group with no ids
  float aux;
};

// Launch-wide words, zeroed by the row kernel.
struct alignas(128) Ctl {
  unsigned int err;          // 4: a race found no candidate (cannot happen on finite rows)
  unsigned int pad[31];
};

// Workspace layout (offsets in bytes from the workspace base).
struct Layout {
  int64_t G;                 // groups per row
  size_t summ, emin, total;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

inline int64_t stream_groups_per_row(int64_t V) {
  int64_t n = 0;
  for (int s = 0; s < kNumSlices; ++s) n += slice_groups(slice_start(s + 1, V) - slice_start(s, V));
  return n;
}

inline Layout make_layout(int64_t B, int64_t V) {
  Layout L;
  L.G = stream_groups_per_row(V);
  const size_t n0 = align256(sizeof(Ctl));
  L.summ = n0;
  L.emin = align256(L.summ + size_t(B) * size_t(L.G) * sizeof(GroupSum));
  L.total = align256(L.emin + size_t(B) * size_t(L.G) * sizeof(float));
  return L;
}

}  // namespace st
}  // namespace qe
