// qe_stream.cuh — data structures of the streaming sampler (qe_sample_stream.cu):
// work items, per-chunk records, per-row rounds and the workspace layout.
//
// A row of V ids is split into chunks: canonical slice s (16 per row, ids
// [slice_start(s), slice_start(s+1))) is cut into `cps` chunks of `tpc` tiles
// of 1024 ids.  A chunk is the unit of work: one CTA streams it from HBM into
// shared memory with a bulk copy and reduces it to a fixed-size record.  The
// CTA that files the last record of a row merges the records and either
// writes the row's token or publishes a follow-up round over the row's chunks
// (re-read from L2), whose last partial decides again.
#pragma once
#include <cstddef>
#include <cstdint>

#include "qe_common.cuh"

namespace qe {
namespace st {

constexpr int kThreads = 256;                 // compute threads per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kCtaThreads = kThreads + 32;    // + one producer warp
constexpr int kNumBuf = 2;                    // chunk buffers per CTA
constexpr int kBufBytes = 32768;              // bytes per chunk buffer
constexpr int kMaxTiles = 16;                 // tiles per chunk (16-bit types; 8 for fp32)
constexpr int kMaxGroups = kMaxTiles * 32;
constexpr int kR = 3;                         // race candidates per chunk record (filtered rows)
constexpr int kBins = 64;                     // mass histogram bins (half a log2 unit each)
constexpr int kSmallK = 64;                   // top-k rows up to this k gather their head
constexpr int kGCap = 256;                    // gathered (x, id) pairs per chunk
constexpr int kTopM = 16;                     // group maxima per warp behind the small top-k bound
constexpr int kTC = 4;                        // candidates per test round
constexpr int kMaxRounds = 8;                 // follow-up rounds a row can publish
constexpr int kQ2Cap = 256;                   // groups expanded per chunk (overflow: conservative)
constexpr int kQ3Cap = 1024;                  // tokens noised per chunk (overflow: conservative)
constexpr int kSortCap = 512;                 // gathered keys the small top-k merge sorts
constexpr int kTargetItems = 592;             // chunks per launch below which chunks are split
constexpr uint32_t kDefaultPolls = 1u << 20;  // bound on every device-side wait

enum RowKind : int { kKindGreedy = 0, kKindArgmax = 1, kKindRace = 2, kKindSmallK = 3 };
enum RoundType : int { kRoundTest = 1, kRoundHist = 2, kRoundTies = 3, kRoundRace = 4 };
// What the producer warp hands the compute warps in a buffer.
enum ItemKind : int { kItemEnd = 0, kItemChunk = 1, kItemFollow = 2, kItemFinish = 3, kItemNone = 4 };
constexpr int kFinQ = 64;                     // rows a CTA's producer has to finish (ring)
enum : uint32_t { kFNan = 1u, kFEmpty = 2u, kFOver = 4u };

// A race candidate: ratio in the producing chunk's scale, logit, noise, id.
struct Cand {
  float r, x, E;
  int id;
};

// What a chunk files after its first pass (96 bytes).
struct alignas(16) ChunkRec {
  float cmax;        // max of the (penalised) logits; NaN if the chunk holds a NaN
  float u;           // RN(cmax * c1): the chunk's exponent anchor
  int greedy;        // first id holding cmax (the first NaN when kFNan)
  uint32_t flags;
  double S;          // sum over the chunk of 2^(x c1 - u)
  float ceil;        // bound on the ratio (chunk scale) of every token not in cand[]
  int ncand;
  float lk;          // small top-k rows: lower bound on the chunk's k-th largest logit
  int ngather;       // small top-k rows: (x, id) pairs filed in the gather area
  Cand cand[kR];
};

struct GItem {
  float x;
  int id;
};

// The round a row is in, written by the CTA that publishes it.
struct alignas(16) RowRound {
  int type;                  // RoundType
  int level;                 // radix level of a histogram round (0..3)
  uint32_t prefix;           // key bits above the level
  int m;                     // test candidates
  float c0, Sf;              // row exponent offset -RN(xmax c1) and float(S)
  double S;
  float xs[kTC];             // test candidates in race order
  int ids[kTC];
  long long kk;              // exact rounds: count limit min(top_k, |p >= min-p threshold|)
  unsigned long long tfix;   // mass limit (2^-40 units)
  unsigned long long sfix;   // row mass (2^-40 units)
  long long acnt;            // elements above the current key range
  unsigned long long amass;
  uint32_t kkey;             // boundary key
  int ties_all;              // every element with key == kkey is kept
  long long kties;           // kept elements with key == kkey
  long long nkeep;           // size of the kept set
  float thr_m;               // min-p threshold on p (0: off)
  float pad;
};

// Per (row, chunk) result of a follow-up round.
struct alignas(16) Part {
  double mass[kTC];
  long long cnt[kTC];
};

// Per-row radix histogram of an exact round (filled with global atomics).
struct HistAcc {
  unsigned int cnt[256];
  unsigned long long mass[256];
  unsigned int nm;           // min-p count (level 0)
  unsigned int pad[3];
};

// Launch-wide counters, zeroed before every launch; each on its own 128-byte
// line so that polling one does not queue behind atomics on another.
struct alignas(128) Ctl {
  unsigned int qentries;     // follow-up rounds published
  unsigned int pad0[31];
  unsigned int qhead;        // follow-up items claimed
  unsigned int pad1[31];
  unsigned int rows_done;
  unsigned int pad2[31];
  unsigned int err;          // 1: a bounded wait gave up
  unsigned int pad3[31];
};

struct RowCtl {
  unsigned int cnt;          // arrivals in the row's current round
  unsigned int timeout;      // a wait on one of the row's chunks gave up
  unsigned int round;        // the row's current round: 0 = chunk records, else RoundType
  unsigned int pad;
};

// Workspace layout (offsets in bytes from the workspace base).
struct Layout {
  int tpc, cps, nc;
  size_t rowctl, queue, zero_bytes;
  size_t rec, hist, gather, round, part, hacc, total;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Tiles in the longest canonical slice of a row of V ids.
inline int max_slice_tiles(int64_t V) {
  int64_t m = 0;
  for (int s = 0; s < kNumSlices; ++s) {
    const int64_t L = slice_start(s + 1, V) - slice_start(s, V);
    if (L > m) m = L;
  }
  return int((m + kTile - 1) / kTile);
}

// Chunk shape: as many tiles as the buffer holds, halved while the launch
// would have fewer than kTargetItems chunks (small batches).
inline Layout make_layout(int64_t B, int64_t V, int esize) {
  Layout L;
  const int nt = max_slice_tiles(V);
  int tpc = esize == 4 ? kMaxTiles / 2 : kMaxTiles;
  while (tpc > 1 && B * kNumSlices * ((nt + tpc - 1) / tpc) < kTargetItems) tpc /= 2;
  L.tpc = tpc;
  L.cps = nt > 0 ? (nt + tpc - 1) / tpc : 1;
  L.nc = kNumSlices * L.cps;
  const size_t b = size_t(B), nc = size_t(L.nc);
  size_t n = align256(sizeof(Ctl));
  L.rowctl = n;
  n = align256(n + b * sizeof(RowCtl));
  L.queue = n;
  n = align256(n + b * kMaxRounds * sizeof(int));
  L.zero_bytes = n;
  L.rec = n;
  n = align256(n + b * nc * sizeof(ChunkRec));
  L.hist = n;
  n = align256(n + b * nc * kBins * sizeof(float));
  L.gather = n;
  n = align256(n + b * nc * kGCap * sizeof(GItem));
  L.round = n;
  n = align256(n + b * sizeof(RowRound));
  L.part = n;
  n = align256(n + b * nc * sizeof(Part));
  L.hacc = n;
  n = align256(n + b * sizeof(HistAcc));
  L.total = n;
  return L;
}

}  // namespace st
}  // namespace qe
