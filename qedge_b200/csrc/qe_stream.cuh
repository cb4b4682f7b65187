// qe_stream.cuh — data layout of the streaming sampler (qe_sample_stream.cu).
//
// The sampler runs as six launches (scan, decide, count, retry, count,
// finish).  The scan kernel streams every row of
// logits from HBM once, one warp per task of `tpw` tiles of 1024 ids inside a
// canonical slice.  It reduces each 32-id group (the canonical layout of
// qe_common.cuh) to a GroupSum and each task to a TaskRec.  The decide kernel
// (one CTA per row) works from the task records: row max, softmax
// normaliser, the exponential race over the few groups whose noise bound can
// win, and the kept-set test of the race candidates.  Rows whose test the
// records cannot settle are counted exactly by the count kernel (all SMs over
// the (row, tile) pairs of those rows); rows whose counted candidates all lie
// outside the kept set race again in the retry kernel; rows that need the
// full kept set (small top-k, out_kept asked for, the rare rest) are finished
// by the finish kernel.
#pragma once
#include <cstddef>
#include <cstdint>

#include "qe_common.cuh"

namespace qe {
namespace st {

constexpr int kSumThreads = 256;              // scan / count kernels: threads per CTA (8 warp tasks)
constexpr int kRowThreads = 256;              // decide / finish kernels: threads per CTA (one row)
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kTC = 4;                        // race candidates tested for kept-set membership
constexpr int kSmallK = 64;                   // top-k rows up to this k take the direct top-k path
constexpr int kSelCap = 4096;                 // direct top-k: elements collected
constexpr int kSortCap = 512;                 // direct top-k: elements sorted
constexpr int kHashCap = 8192;                // history ids hashed per row (repetition penalty)
constexpr int kMaxTasksPerSlice = 64;         // tpw grows with the slice so a row has <= 1024 tasks
constexpr int kMaxTasks = kNumSlices * kMaxTasksPerSlice;
constexpr int kGList = 2048;                  // decide kernel: race groups expanded per round
constexpr int kRescanCap = 256;               // decide kernel: tasks whose groups are re-bounded

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

// Summary of one scan task (tpw tiles of one slice).  Bound keys are
// RN(gmax c1) - log2(lower bound of the group's noise minimum): a group's best
// race ratio is at most 2^(bk - RN(xmax c1)) / S.  Sampled rows only.
struct alignas(16) TaskRec {
  float tmax;     // NaN-propagating max of the task's (penalised) logits
  float bk0, bk1; // the two largest group bound keys (-inf: none)
  float bceil;    // the third largest: a ceiling for every other group of the task
  double tsum;    // sum of the task's group sums scaled to RN(tmax c1)
  int bg0, bg1;   // global group ids of bk0 and bk1 (-1: none)
};

// Race candidate: ratio r = RN(RN(e/S)/E), penalised logit x, noise E, id.
struct Cand {
  float r, x, E;
  int id;
};

// Per-row state handed from the decide kernel to the count, retry and
// finish kernels.
struct alignas(16) RowState {
  float xmax, u, Sf, thr_m;   // row max, RN(xmax c1), float(S), min-p threshold on p
  double S;                   // softmax normaliser relative to 2^u
  int ncand;                  // candidates still to test (count kernel)
  unsigned int done;          // tasks counted so far (count kernel)
  float rx;                   // retry race: only ids strictly ahead of (rx, rid) in the order
  int rid;
  Cand cand[kTC];
  unsigned long long cmass[kTC];   // mass ahead of each candidate, fixed point 2^-40
  unsigned long long ccnt[kTC];    // ids ahead of each candidate
};

// Launch-wide words, zeroed by the scan kernel.
struct alignas(128) Ctl {
  unsigned int err;          // 4: a race found no candidate (cannot happen on finite rows)
  unsigned int n_pend[2];    // rows queued for the count kernel (first and retry round)
  unsigned int n_retry;      // rows queued for the retry round (all candidates outside the kept set)
  unsigned int n_fin;        // rows queued for the finish kernel
  unsigned int pad[27];
};

// Finish-list entries: row | kind << 28.
constexpr unsigned kFinExact = 0u, kFinSmallK = 1u;

// Workspace layout (offsets in bytes from the workspace base).
struct Layout {
  int64_t G;                 // groups per row
  int tasks;                 // scan tasks per row
  int tpw;                   // tiles per task
  size_t summ, trec, emin, rstate, plist, rlist, flist, total;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

inline int64_t stream_groups_per_row(int64_t V) {
  int64_t n = 0;
  for (int s = 0; s < kNumSlices; ++s) n += slice_groups(slice_start(s + 1, V) - slice_start(s, V));
  return n;
}

// Tiles per scan task: 4 for 16-bit rows and 1 for fp32 rows, doubled until
// no slice has more than kMaxTasksPerSlice tasks.
inline int stream_tpw(int64_t V, int esize) {
  int64_t maxt = 0;
  for (int s = 0; s < kNumSlices; ++s) {
    const int64_t t = (slice_start(s + 1, V) - slice_start(s, V) + kTile - 1) / kTile;
    maxt = t > maxt ? t : maxt;
  }
  int tpw = esize == 4 ? 1 : 4;
  while ((maxt + tpw - 1) / tpw > kMaxTasksPerSlice) tpw *= 2;
  return tpw;
}

inline int stream_tasks_per_row(int64_t V, int tpw) {
  int n = 0;
  for (int s = 0; s < kNumSlices; ++s) {
    const int64_t t = (slice_start(s + 1, V) - slice_start(s, V) + kTile - 1) / kTile;
    n += int((t + tpw - 1) / tpw);
  }
  return n;
}

inline Layout make_layout(int64_t B, int64_t V, int esize) {
  Layout L;
  L.G = stream_groups_per_row(V);
  L.tpw = stream_tpw(V, esize);
  L.tasks = stream_tasks_per_row(V, L.tpw);
  const size_t b = size_t(B);
  L.summ = align256(sizeof(Ctl));
  L.trec = align256(L.summ + b * size_t(L.G) * sizeof(GroupSum));
  L.emin = align256(L.trec + b * size_t(L.tasks) * sizeof(TaskRec));
  L.rstate = align256(L.emin + b * size_t(L.G) * sizeof(float));
  L.plist = align256(L.rstate + b * sizeof(RowState));
  L.rlist = align256(L.plist + 2 * b * sizeof(int));
  L.flist = align256(L.rlist + b * sizeof(int));
  L.total = align256(L.flist + b * sizeof(int));
  return L;
}

}  // namespace st
}  // namespace qe
