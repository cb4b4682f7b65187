// qe_sample_fused.cu — the fused single-pass sampler (one thread-block
// cluster per row, the row resident in the cluster's shared memory).
//
// Replaces BatchSampler.forward (src/compute/sampler.py:25-41) for rows
// whose CTA share fits in shared memory.  Every row is read from HBM once,
// by 1-D bulk copies (cp.async.bulk + mbarrier), into the shared memory of
// the 8 CTAs (16 on request) of a cluster; CTA q holds canonical vocab
// slices [qU, qU+U).  Per row:
//
//   noise    while the copy flies, each lane computes the exact minimum and
//            second-smallest noise of its two 32-id groups (one Philox call
//            per group)
//   pass 1   per group: max, then the softmax sum relative to the group max
//            (the only pass with an exponential per token)
//   race     lazy exponential race: a group's best ratio is bounded by
//            max(e_arg / E_min, e_max / E2); each CTA expands, warp by warp,
//            only groups whose bound reaches its running threshold and so
//            finds its exact best tokens and a ceiling over the rest
//   exchange one cluster barrier: each CTA pushes its record (max, sum,
//            candidates, ceiling) into every peer's shared memory; greedy and
//            unfiltered rows are decided here
//   tests    top-k / top-p rows: the best candidate first (groups below it
//            skipped), then the other complete candidates; each round ends
//            in a cluster exchange of the mass and rank ahead of them
//
// Rows with a small top-k, and the rare rows whose candidates all fall
// outside the kept set, gather every token above a proven lower bound of the
// kept set and finish exactly in CTA 0 (sort + prefix mass + race).  Rows
// whose gathered set is too large are finished by the whole cluster with a
// radix selection over the CTAs' own slices.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <string>

#include "qe_common.cuh"
#include "qe_fused_util.cuh"
#include "qe_internal.h"

namespace cg = cooperative_groups;

namespace qe {
namespace fz {

constexpr int kMaxR = 4;          // race candidates tested per row
constexpr int kMaxItems = 1;      // tile pairs a warp owns per row
constexpr int kSlots = 2 * kMaxItems;  // groups per lane
static_assert(kSlots == 2, "slot selects below assume one tile pair per warp");
constexpr int kGatherCap = 768;   // gathered keys per CTA
constexpr int kSmallK = 64;       // top-k rows up to this k take the gather path
constexpr int kSparseGroups = 12; // candidate tests: tiles with at most this many active groups go group by group
constexpr uint32_t kWaitLimit = 1u << 20;   // polls (each suspends up to 1 us)

enum RowType : int { kDone = 0, kRaceTest = 1, kGather = 2, kSlow = 3 };

struct Cand {
  float r;   // ratio e/E in the producing CTA's scale
  float x;   // penalised logit
  float E;   // noise
  int id;    // token id
};

// What a CTA publishes to its cluster peers in the candidate-test and gather
// rounds (read over DSMEM).
struct alignas(16) Share {
  int ngather;
  int overflow;
  int pad[2];
  long long cnt[kMaxR];
  double F[kMaxR];
};

// Exchange-1 record: what a CTA pushes into every peer's inbox (DSMEM
// stores before the cluster barrier; each CTA then reads its own inbox).
struct alignas(16) Rec1 {
  float umax[2];
  float c0;
  int nan;
  int gidx;
  float gval;
  uint32_t lkey;
  int ncand;
  float ceil;            // bound on the ratio of every token not in cand[]
  int pad;
  double S;              // softmax sum in this CTA's scale
  Cand cand[2];
};
static_assert(sizeof(Rec1) % 16 == 0, "Rec1 is copied as 16-byte words");

struct RowState {
  int type;
  int out;
  int status;
  int R;                 // candidates tested this round (gather: keys, -1 = gather pending)
  int cb;                // first candidate tested this round
  int ncand;             // candidates known to precede every unpublished token
  int p_on, k_on, k;
  float tp;
  float c1, nM, xM, Sf;
  double S;
  float L;               // gather lower bound (x' >= L)
  Cand cand[kMaxR];      // global candidates, race order, row-scale ratios
};

template <int CL>
struct Cfg {
  static constexpr int NT = CL == 8 ? 512 : 256;
  static constexpr int NW = NT / 32;
  static constexpr int U = 16 / CL;
};

struct FusedParams {
  KernelArgs a;
  int nclusters;
  int cap;         // data capacity in elements
  int tma_ok;      // logits rows 16-byte aligned
  int noise_vec;   // noise rows 16-byte aligned
  int merge_cap;   // keys CTA 0 can sort in its data buffer (power of two)
};

struct Misc {
  uint64_t mbar;
  unsigned int umaxkey[2];
  int nan;
  unsigned int gmin;
  int err;
  int ngather;
  float e_root;
  int s_mem;
  long long s_gid;
  unsigned int wtop[16 * 8];
  float theta;           // running race threshold of the CTA (positive floats as ints)
  float wbound[16];      // each warp's largest group bound
  float wceil[16];
  float wb[16];
  int wbslot[16];
  double wS[16];
  float wF[16][kMaxR];
  long long wcnt[16][kMaxR];
  float c0peer[16];
  long long tstart[17];
  long long tgbase[16];
  int slow_int[48];
};

// Exact noise of one group, kept in shared memory between the noise pass and
// the expansions (parity mode: e_min is the group's minimum noise).
struct GNoise {
  float e_min, e2;
  int args;  // argmin | second member << 8 (0xFF: none)
};

// ---------------------------------------------------------------- smem layout
template <typename T, int CL>
struct Smem {
  static constexpr int NW = Cfg<CL>::NW;
  static __host__ __device__ size_t data_bytes(int cap) { return size_t(cap) * sizeof(T); }
  static __host__ __device__ size_t pen_off(int cap) { return (data_bytes(cap) + 127) / 128 * 128; }
  static __host__ __device__ size_t gather_off(int cap) { return pen_off(cap) + ((cap / 32 + 1) * 4 + 15) / 16 * 16; }
  static __host__ __device__ size_t share_off(int cap) { return gather_off(cap) + kGatherCap * 8; }
  static __host__ __device__ size_t peer_off(int cap) { return share_off(cap) + 2 * sizeof(Share); }
  static __host__ __device__ size_t wl_off(int cap) { return peer_off(cap) + size_t(CL) * sizeof(Share); }
  static __host__ __device__ size_t rs_off(int cap) { return wl_off(cap) + size_t(NW) * kMaxR * sizeof(Cand); }
  static __host__ __device__ size_t misc_off(int cap) { return (rs_off(cap) + sizeof(RowState) + 15) / 16 * 16; }
  static __host__ __device__ size_t gnz_off(int cap) { return misc_off(cap) + (sizeof(Misc) + 127) / 128 * 128; }
  static __host__ __device__ size_t inbox_off(int cap) {
    return (gnz_off(cap) + size_t(Cfg<CL>::NT) * kSlots * sizeof(GNoise) + 15) / 16 * 16;
  }
  static __host__ __device__ size_t total(int cap) { return inbox_off(cap) + 2 * size_t(CL) * sizeof(Rec1); }
};

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ int ctz_lane(uint32_t m) { return __ffs(m) - 1; }

// Insert (c) into a list sorted by race order, keeping the best n.
__device__ __forceinline__ void list_insert(Cand* l, int n, const Cand& c) {
  if (!rbetter(c.r, c.id, l[n - 1].r, l[n - 1].id)) return;
  int i = n - 1;
  while (i > 0 && rbetter(c.r, c.id, l[i - 1].r, l[i - 1].id)) { l[i] = l[i - 1]; --i; }
  l[i] = c;
}

// Warp-level: merge the 32 lanes' (r, x, E, id) into the warp's sorted list
// of n candidates (lane 0 owns the list in shared memory).  A warp-wide max
// first rejects the common case where no lane can enter the list; otherwise
// each round extracts the best remaining lane through one 64-bit key
// (ordered ratio, inverted id) per shuffle step.
__device__ __forceinline__ void warp_merge(Cand* wl, int n, float r, float x, float E, int id) {
  const int lane = threadIdx.x & 31;
  // ratios are >= 0 or -inf: for r >= 0 the bit pattern orders like the value
  uint32_t k = r >= 0.f ? __float_as_uint(r) + 1u : 0u;
  const uint32_t floor_k = wl[n - 1].r >= 0.f ? __float_as_uint(wl[n - 1].r) + 1u : 0u;
  for (int round = 0; round < n; ++round) {
    const uint32_t km = __reduce_max_sync(0xffffffffu, k);
    if (km == 0u || km < floor_k) break;
    const uint32_t im = __reduce_min_sync(0xffffffffu, k == km ? uint32_t(id) : 0xFFFFFFFFu);
    const int bl = __ffs(__ballot_sync(0xffffffffu, k == km && uint32_t(id) == im)) - 1;
    const float bx = __shfl_sync(0xffffffffu, x, bl);
    const float bE = __shfl_sync(0xffffffffu, E, bl);
    bool stop = false;
    if (lane == 0) {
      const float br = __uint_as_float(km - 1u);
      stop = !rbetter(br, int(im), wl[n - 1].r, wl[n - 1].id);
      if (!stop) list_insert(wl, n, Cand{br, bx, bE, int(im)});
    }
    stop = __shfl_sync(0xffffffffu, stop, 0);
    __syncwarp();
    if (stop) break;
    if (lane == bl) k = 0u;
  }
}

// Lane holding the warp-wide best (r desc, id asc) among the lanes' (r, id),
// or -1 if no lane has r > -inf.  Two warp reductions and a ballot.
__device__ __forceinline__ int warp_best_lane(float r, int id) {
  const uint32_t k = (r > -INFINITY) ? ordered_key(r) : 0u;   // NaN never reaches here
  const uint32_t km = __reduce_max_sync(0xffffffffu, k);
  if (km == 0u) return -1;
  const uint32_t im = __reduce_min_sync(0xffffffffu, k == km ? uint32_t(id) : 0xFFFFFFFFu);
  return __ffs(__ballot_sync(0xffffffffu, k == km && uint32_t(id) == im)) - 1;
}

// ---------------------------------------------------------------- per-row geometry
struct Geo {
  int64_t cta_start, cta_end;  // global ids held by this CTA
  int64_t ustart[2], uend[2];  // global ids of each unit (slice)
  int uoff[2];                 // CTA-local element offset of each unit
  int L[2];
  int ntiles[2], npairs[2];
  int nitems;
  int64_t gbase[2];            // global group id base of each unit
};

template <int U>
__device__ __forceinline__ Geo make_geo(int q, int64_t V) {
  Geo g;
  g.cta_start = slice_start(q * U, V);
  g.cta_end = slice_start(q * U + U, V);
  g.nitems = 0;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (u < U) {
      const int s = q * U + u;
      g.ustart[u] = slice_start(s, V);
      g.uend[u] = slice_start(s + 1, V);
      g.uoff[u] = int(g.ustart[u] - g.cta_start);
      g.L[u] = int(g.uend[u] - g.ustart[u]);
      g.ntiles[u] = (g.L[u] + kTile - 1) / kTile;
      g.npairs[u] = (g.ntiles[u] + 1) / 2;
      g.gbase[u] = slice_group_base(s, V);
      g.nitems += g.npairs[u];
    } else {
      g.ustart[u] = g.uend[u] = g.cta_end;
      g.uoff[u] = 0; g.L[u] = 0; g.ntiles[u] = 0; g.npairs[u] = 0; g.gbase[u] = 0;
    }
  }
  return g;
}
__device__ __forceinline__ void item_of(const Geo& g, int item, int& u, int& p) {
  if (item < g.npairs[0]) { u = 0; p = item; } else { u = 1; p = item - g.npairs[0]; }
}
struct Unit {
  int L, uoff, ntiles;
  int64_t ustart, uend, gbase;
};
__device__ __forceinline__ Unit unit_of(const Geo& g, int u) {
  Unit r;
  r.L = u ? g.L[1] : g.L[0];
  r.uoff = u ? g.uoff[1] : g.uoff[0];
  r.ntiles = u ? g.ntiles[1] : g.ntiles[0];
  r.ustart = u ? g.ustart[1] : g.ustart[0];
  r.uend = u ? g.uend[1] : g.uend[0];
  r.gbase = u ? g.gbase[1] : g.gbase[0];
  return r;
}
// Warp-aggregated append of the flagged elements (bit i of `mask` flags
// element off+i) as (ordered key, inverted id) pairs.  All 32 lanes call it.
__device__ __forceinline__ void gather_append(unsigned mask, const float x[8], int64_t id0,
                                              unsigned long long* gath, int* counter) {
  const int lane = threadIdx.x & 31;
  const int cnt = __popc(mask);
  int incl = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (!total) return;
  int base = 0;
  if (lane == 31) base = atomicAdd(counter, total);
  base = __shfl_sync(0xffffffffu, base, 31);
  int pos = base + incl - cnt;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if ((mask >> i) & 1u) {
      if (pos < kGatherCap) {
        const uint32_t id = uint32_t(id0 + i);
        gath[pos] = (uint64_t(ordered_key(x[i])) << 32) | uint64_t(0xFFFFFFFFu - id);
      }
      ++pos;
    }
}

// Penalised logit of CTA-local element `off` (scalar path).
template <typename T>
__device__ __forceinline__ float load1(const void* buf, const uint32_t* pen, bool use_pen, float rp, int off) {
  float x;
  if constexpr (sizeof(T) == 4) {
    x = static_cast<const float*>(buf)[off];
  } else if constexpr (std::is_same<T, __half>::value) {
    x = __half2float(static_cast<const __half*>(buf)[off]);
  } else {
    x = __uint_as_float(uint32_t(static_cast<const uint16_t*>(buf)[off]) << 16);
  }
  if (use_pen && ((pen[off >> 5] >> (off & 31)) & 1u)) x = penalise(x, rp);
  return x;
}


// Bitonic sort (descending) of n = power of two 64-bit keys in shared memory.
template <int NT>
__device__ void bitonic_desc(unsigned long long* k, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += NT) {
        const int lo = 2 * stride * (i / stride) + (i % stride);
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long a = k[lo], b = k[hi];
        if ((a < b) == desc) { k[lo] = b; k[hi] = a; }
      }
      __syncthreads();
    }
  }
}


// Exact finish of one row by the whole cluster, each CTA working on its own
// slice: the kept set is found by radix selection on the ordered logit keys
// (4 passes of 8 bits; per-CTA shared-memory histograms of counts and of
// probability mass in 2^-40 fixed point, merged over DSMEM), ties at the
// boundary are kept in id order, and the race runs over every kept token.
// Used when the race candidates all fall outside the kept set and the kept
// set is too large to gather.  Every CTA calls it (cluster barriers inside).
template <typename T, int CL>
__device__ __noinline__ void cluster_exact(const FusedParams& P, int64_t row, cg::cluster_group& cluster,
                                           const void* data, const uint32_t* pen, unsigned long long* scratch,
                                           const RowState& rs, bool use_pen, float rpv, int64_t cta_start,
                                           int n_cta, int* s_int, float* s_flt, const GNoise* gnz,
                                           const Geo& geo) {
  constexpr int NT = Cfg<CL>::NT, NW = Cfg<CL>::NW;
  const KernelArgs& a = P.a;
  const int64_t V = a.vocab;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float c1 = rs.c1, nM = rs.nM, Sf = rs.Sf;
  uint32_t* hc = reinterpret_cast<uint32_t*>(scratch);                // [256]
  unsigned long long* hm = scratch + 128;                              // [256]
  long long* pub = reinterpret_cast<long long*>(scratch + 384);        // published scalars [8]
  const int q = int(cluster.block_rank());
  const unsigned long long Sfix = __double2ull_rn(rs.S * kSumScale);
  auto fixe = [&](float x) { return (unsigned long long)__double2ull_rn(double(unnorm_ftz(x, c1, nM)) * kSumScale); };

  uint32_t prefix = 0, msk = 0;
  long long cbase = 0;
  unsigned long long mbase = 0;
  // radix selection: weighted (top-p: last token whose exclusive mass <= T)
  // or counting (top-k: the token at position `pos`); sets the boundary key
  // in `prefix`, the tokens strictly above it in `cbase`, the kept count
  auto select = [&](bool weighted, unsigned long long Tfix, long long pos, long long& keep) {
    prefix = 0; msk = 0; cbase = 0; mbase = 0;
    long long nt = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += NT) { hc[b] = 0; hm[b] = 0; }
      __syncthreads();
      for (int off = threadIdx.x; off < n_cta; off += NT) {
        const float x = load1<T>(data, pen, use_pen, rpv, off);
        const uint32_t kq = ordered_key(x);
        if ((kq & msk) == prefix) {
          const int b = (kq >> shift) & 255;
          atomicAdd(&hc[b], 1u);
          if (weighted && x > -INFINITY) atomicAdd(&hm[b], fixe(x));
        }
      }
      cluster.sync();
      if (warp == 0) {
        // lane l holds bins 255-8l .. 248-8l (descending key order)
        uint32_t c8[8];
        unsigned long long m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) { c8[i] = 0; m8[i] = 0; }
        for (int r = 0; r < CL; ++r) {
          const uint32_t* rc = cluster.map_shared_rank(hc, r);
          const unsigned long long* rm = cluster.map_shared_rank(hm, r);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int b = 255 - (lane * 8 + i);
            c8[i] += rc[b];
            if (weighted) m8[i] += rm[b];
          }
        }
        long long lc = 0;
        unsigned long long lm = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) { lc += c8[i]; lm += m8[i]; }
        long long ic = lc;
        unsigned long long im = lm;
        for (int o = 1; o < 32; o <<= 1) {
          const long long vc = __shfl_up_sync(0xffffffffu, ic, o);
          const unsigned long long vm = __shfl_up_sync(0xffffffffu, im, o);
          if (lane >= o) { ic += vc; im += vm; }
        }
        long long c = cbase + ic - lc;
        unsigned long long m = mbase + im - lm;
        int cand = -1;
        long long cc = 0, ct = 0;
        unsigned long long cm = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (c8[i]) {
            if (weighted) {
              if (m <= Tfix) { cand = 255 - (lane * 8 + i); cc = c; cm = m; ct = c8[i]; }
            } else if (pos >= c && pos < c + (long long)c8[i]) {
              cand = 255 - (lane * 8 + i); cc = c; cm = m; ct = c8[i];
            }
          }
          c += c8[i];
          m += m8[i];
        }
        int pick = cand;
        for (int o = 16; o; o >>= 1) {
          const int other = __shfl_xor_sync(0xffffffffu, pick, o);
          if (other >= 0 && (pick < 0 || (weighted ? other < pick : true))) pick = other;
        }
        if (pick < 0) pick = 0;
        const unsigned who = __ballot_sync(0xffffffffu, cand == pick);
        const int wl_ = who ? __ffs(who) - 1 : 0;
        cc = __shfl_sync(0xffffffffu, cc, wl_);
        cm = __shfl_sync(0xffffffffu, cm, wl_);
        ct = __shfl_sync(0xffffffffu, ct, wl_);
        if (lane == 0) { pub[0] = pick; pub[1] = cc; pub[2] = (long long)cm; pub[3] = ct; }
      }
      __syncthreads();
      prefix |= uint32_t(pub[0]) << shift;
      msk |= 255u << shift;
      cbase = pub[1];
      mbase = (unsigned long long)pub[2];
      nt = pub[3];
      cluster.sync();  // peers are done reading this CTA's histogram
    }
    if (weighted) {
      const unsigned long long f = fixe(key_to_float(prefix));
      long long c = nt;
      if (f > 0) {
        const unsigned long long qq = (Tfix - mbase) / f + 1;
        if (qq < (unsigned long long)nt) c = (long long)qq;
      }
      keep = cbase + c;
    } else {
      keep = pos + 1;
    }
  };

  long long n_keep = V;
  uint32_t vkey = 0;
  bool have = false;
  long long above = 0;
  if (rs.p_on) {
    select(true, (unsigned long long)(double(rs.tp) * double(Sfix)), 0, n_keep);
    vkey = prefix; above = cbase; have = true;
  }
  if (rs.k_on && rs.k < n_keep) {
    select(false, 0ull, rs.k - 1, n_keep);
    vkey = prefix; above = cbase; have = true;
  }
  const long long tie_keep = n_keep - above;
  // id of the last kept tie: tie counts per CTA (id order = CTA order, then
  // offset order), the CTA that holds it finds it with a block scan
  const int per = (n_cta + NT - 1) / NT;
  const int i0 = threadIdx.x * per;
  int myties = 0;
  for (int i = i0; i < i0 + per && i < n_cta; ++i) myties += ordered_key(load1<T>(data, pen, use_pen, rpv, i)) == vkey;
  int incl = myties;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_int[warp] = incl;
  __syncthreads();
  int woff = 0, ctaties = 0;
  for (int w = 0; w < NW; ++w) { if (w < warp) woff += s_int[w]; ctaties += s_int[w]; }
  if (threadIdx.x == 0) pub[4] = ctaties;
  cluster.sync();
  long long before_cta = 0;
  for (int r = 0; r < q; ++r) before_cta += cluster.map_shared_rank(pub, r)[4];
  {
    long long rank = before_cta + woff + incl - myties;
    for (int i = i0; i < i0 + per && i < n_cta; ++i) {
      if (ordered_key(load1<T>(data, pen, use_pen, rpv, i)) == vkey) {
        if (rank == tie_keep - 1) pub[5] = cta_start + i;
        ++rank;
      }
    }
  }
  if (threadIdx.x == 0 && !(tie_keep - 1 >= before_cta && tie_keep - 1 < before_cta + ctaties)) pub[5] = -1;
  cluster.sync();
  long long id_c = 0x7FFFFFFFll;
  for (int r = 0; r < CL; ++r) {
    const long long v = cluster.map_shared_rank(pub, r)[5];
    if (v >= 0) id_c = v;
  }
  if (!have) id_c = 0x7FFFFFFFll;
  // race over the kept tokens of this slice
  const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
  const NoiseKey key = make_noise_key(a.seed, step, a.row_offset + row);
  NoiseRoot rt{0.f, 0};
  int64_t gs = -1;
  int mem_s = 0;
  if (!a.noise) {
    rt = noise_root(key, V);
    token_group(rt.s, V, &gs, &mem_s);
  }
  float br = -INFINITY;
  int bid = 0x7FFFFFFF;
  for (int off = threadIdx.x; off < n_cta; off += NT) {
    const float x = load1<T>(data, pen, use_pen, rpv, off);
    const uint32_t kq = ordered_key(x);
    const int64_t j = cta_start + off;
    const bool in = !have || kq > vkey || (kq == vkey && j <= id_c);
    if (in && x > -INFINITY) {
      const float pv = __fdiv_rn(unnorm_ftz(x, c1, nM), Sf);
      float E;
      if (a.noise) {
        E = __ldg(a.noise + row * a.noise_ld + j);
      } else if (gnz) {
        // the row's group noise is still in the table: only the token word is new
        const int u = (Cfg<CL>::U == 2 && off >= geo.uoff[1]) ? 1 : 0;
        const int o = off - (u ? geo.uoff[1] : geo.uoff[0]);
        const int t = o >> 10, l = (o >> 3) & 31;
        const int item = (u ? geo.npairs[0] : 0) + (t >> 1);
        const GNoise g = gnz[(item * 32 + l) * kSlots + (t & 1)];
        GroupNoise gn;
        gn.e_min = g.e_min;
        gn.e2 = g.e2;
        gn.arg = g.args & 0xFF;
        gn.arg2 = ((g.args >> 8) & 0xFF) == 0xFF ? -1 : ((g.args >> 8) & 0xFF);
        E = noise_token(key, gn, j, member_index(o));
      } else {
        E = tree_noise(key, rt, gs, mem_s, j, V);
      }
      const float rv = __fdiv_rn(pv, E);
      if (rbetter(rv, int(j), br, bid)) { br = rv; bid = int(j); }
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float orr = __shfl_xor_sync(0xffffffffu, br, o);
    const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
    if (rbetter(orr, oid, br, bid)) { br = orr; bid = oid; }
  }
  __syncthreads();
  if (lane == 0) { s_flt[warp] = br; s_int[warp] = bid; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < NW; ++w) if (rbetter(s_flt[w], s_int[w], br, bid)) { br = s_flt[w]; bid = s_int[w]; }
    reinterpret_cast<float*>(pub + 6)[0] = br;
    pub[7] = bid;
  }
  cluster.sync();
  if (q == 0 && threadIdx.x == 0) {
    for (int r = 0; r < CL; ++r) {
      const long long* pr = cluster.map_shared_rank(pub, r);
      const float rr = reinterpret_cast<const float*>(pr + 6)[0];
      const int ri = int(pr[7]);
      if (rbetter(rr, ri, br, bid)) { br = rr; bid = ri; }
    }
    a.out_ids[row] = bid == 0x7FFFFFFF ? rs.out : bid;
    if (a.out_status) a.out_status[row] = QE_ROW_SLOW;
  }
  cluster.sync();  // peers keep their published scalars until CTA 0 has read them
}

// CTA 0 finishes a row from the keys every CTA gathered (all tokens with
// x' >= L, which provably contains the kept set): sort, exclusive prefix
// mass, kept prefix, race over the kept tokens.
template <typename T, int CL>
__device__ __noinline__ void gather_finish(const FusedParams& P, int64_t row, cg::cluster_group& cluster,
                                           void* data, unsigned long long* gath, Share* slot,
                                           const RowState& rs, Misc& ms) {
  constexpr int NT = Cfg<CL>::NT, NW = Cfg<CL>::NW;
  const KernelArgs& a = P.a;
  const int64_t V = a.vocab;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(data);
  const int n = rs.R;
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  int base = 0;
  for (int r = 0; r < CL; ++r) {
    const Share* s = cluster.map_shared_rank(slot, r);
    const int cnt = s->ngather;
    const unsigned long long* src = cluster.map_shared_rank(gath, r);
    for (int i = threadIdx.x; i < cnt; i += NT) keys[base + i] = src[i];
    base += cnt;
  }
  for (int i = n + threadIdx.x; i < np2; i += NT) keys[i] = 0ull;
  __syncthreads();
  bitonic_desc<NT>(keys, np2);
  const float c1 = rs.c1, nM = rs.nM, Sf = rs.Sf;
  const int per = (n + NT - 1) / NT;
  const int i0 = threadIdx.x * per;
  double local = 0.0;
  for (int i = i0; i < i0 + per && i < n; ++i)
    local += double(__fdiv_rn(unnorm_ftz(key_to_float(uint32_t(keys[i] >> 32)), c1, nM), Sf));
  double incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  double* wsum = reinterpret_cast<double*>(ms.wF);
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  double run = incl - local;
  for (int w = 0; w < warp; ++w) run += wsum[w];
  int kept = 0;
  for (int i = i0; i < i0 + per && i < n; ++i) {
    const bool ok = (!rs.p_on || run <= double(rs.tp)) && (!rs.k_on || i < rs.k);
    if (!ok) break;
    ++kept;
    run += double(__fdiv_rn(unnorm_ftz(key_to_float(uint32_t(keys[i] >> 32)), c1, nM), Sf));
  }
  const bool complete = kept == max(0, min(per, n - i0));
  const unsigned bal = __ballot_sync(0xffffffffu, !complete);
  int* kc = reinterpret_cast<int*>(ms.wcnt);
  if (lane == 0) kc[warp] = bal ? (warp * 32 + __ffs(bal) - 1) : 0x7FFFFFFF;
  __syncthreads();
  int first_incomplete = 0x7FFFFFFF;
  for (int w = 0; w < NW; ++w) first_incomplete = min(first_incomplete, kc[w]);
  int* s_nk = ms.slow_int;
  if (int(threadIdx.x) == first_incomplete) *s_nk = i0 + kept;
  if (threadIdx.x == 0 && first_incomplete == 0x7FFFFFFF) *s_nk = n;
  __syncthreads();
  const int nK = max(1, min(*s_nk, n));
  const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
  const NoiseKey key = make_noise_key(a.seed, step, a.row_offset + row);
  NoiseRoot rt{0.f, 0};
  int64_t gs = -1;
  int mem_s = 0;
  if (!a.noise) {
    rt = noise_root(key, V);
    token_group(rt.s, V, &gs, &mem_s);
  }
  float br = -INFINITY;
  int bid = 0x7FFFFFFF;
  for (int i = threadIdx.x; i < nK; i += NT) {
    const float x = key_to_float(uint32_t(keys[i] >> 32));
    const int id = int(0xFFFFFFFFu - uint32_t(keys[i] & 0xFFFFFFFFu));
    const float pv = __fdiv_rn(unnorm_ftz(x, c1, nM), Sf);
    const float E = a.noise ? __ldg(a.noise + row * a.noise_ld + id) : tree_noise(key, rt, gs, mem_s, id, V);
    const float r = __fdiv_rn(pv, E);
    if (rbetter(r, id, br, bid)) { br = r; bid = id; }
  }
  for (int o = 16; o; o >>= 1) {
    const float orr = __shfl_xor_sync(0xffffffffu, br, o);
    const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
    if (rbetter(orr, oid, br, bid)) { br = orr; bid = oid; }
  }
  __syncthreads();
  float* wr = ms.wb;
  int* wi = ms.wbslot;
  if (lane == 0) { wr[warp] = br; wi[warp] = bid; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < NW; ++w) if (rbetter(wr[w], wi[w], br, bid)) { br = wr[w]; bid = wi[w]; }
    if (bid == 0x7FFFFFFF) bid = int(0xFFFFFFFFu - uint32_t(keys[0] & 0xFFFFFFFFu));
    a.out_ids[row] = bid;
    if (a.out_status) a.out_status[row] = QE_ROW_GATHERED;
  }
  __syncthreads();
}

// ---------------------------------------------------------------- the kernel
template <typename T, int CL>
__global__ void __launch_bounds__(Cfg<CL>::NT, CL == 16 ? 4 : 2) fused_kernel(FusedParams P) {
  constexpr int NT = Cfg<CL>::NT, NW = Cfg<CL>::NW, U = Cfg<CL>::U;
  using SM = Smem<T, CL>;
  extern __shared__ __align__(128) unsigned char smem[];
  const KernelArgs& a = P.a;
  void* data = smem;
  uint32_t* pen = reinterpret_cast<uint32_t*>(smem + SM::pen_off(P.cap));
  unsigned long long* gath = reinterpret_cast<unsigned long long*>(smem + SM::gather_off(P.cap));
  Share* share = reinterpret_cast<Share*>(smem + SM::share_off(P.cap));
  Share* peers = reinterpret_cast<Share*>(smem + SM::peer_off(P.cap));
  Cand* wl_all = reinterpret_cast<Cand*>(smem + SM::wl_off(P.cap));
  RowState& rs = *reinterpret_cast<RowState*>(smem + SM::rs_off(P.cap));
  Misc& ms = *reinterpret_cast<Misc*>(smem + SM::misc_off(P.cap));
  GNoise* gnz = reinterpret_cast<GNoise*>(smem + SM::gnz_off(P.cap));
  Rec1* inbox = reinterpret_cast<Rec1*>(smem + SM::inbox_off(P.cap));   // [2][CL]

  cg::cluster_group cluster = cg::this_cluster();
  const int q = int(cluster.block_rank());
  const int cid = int(blockIdx.x) / CL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Cand* wl = wl_all + warp * kMaxR;
  const int64_t V = a.vocab;
  // the CTA's slice geometry lives in shared memory (read where needed)
  __shared__ Geo geo_s;
  if (threadIdx.x == 0) geo_s = make_geo<U>(q, V);
  __syncthreads();
  const Geo& geo = geo_s;
  const int n_cta = int(geo.cta_end - geo.cta_start);
  int ex = 0;

  if (threadIdx.x == 0) {
    mbar_init(&ms.mbar, 1);
    ms.err = 0;
    for (int g = 0; g <= kNumSlices; ++g) ms.tstart[g] = slice_start(g, V);
    for (int g = 0; g < kNumSlices; ++g) ms.tgbase[g] = slice_group_base(g, V);
  }
  __syncthreads();
  uint32_t phase = 0;

  for (int64_t row = cid; row < a.batch; row += P.nclusters) {
    // ------------------------------------------------------------ row parameters
    const float T_ = a.temperatures[row];
    const bool greedy = (a.flags & QE_FLAG_ALL_GREEDY) || !(T_ > kGreedyEps);
    const int kk = a.top_ks ? a.top_ks[row] : 0;
    const bool k_on = kk > 0 && int64_t(kk) < V;
    const float tp = a.top_ps ? a.top_ps[row] : 1.f;
    const bool p_on = (a.flags & QE_FLAG_USE_TOP_P) && a.top_ps && tp < 1.f;
    const float rpv = a.rep_penalties ? a.rep_penalties[row] : 1.f;
    int64_t hlen = 0;
    const int32_t* hist = nullptr;
    if (a.history) {
      hist = a.history + row * a.history_ld;
      hlen = a.history_lens ? a.history_lens[row] : a.history_ld;
      if (hlen > a.history_ld) hlen = a.history_ld;
      if (hlen < 0) hlen = 0;
    }
    const bool use_pen = hist && hlen > 0 && rpv != 1.f;
    const bool small_k = !greedy && k_on && kk <= kSmallK && kk > 1;
    const bool need_race = !greedy && !(k_on && kk == 1) && !small_k;
    const float c1 = greedy ? 0.f : temp_coef(T_);
    const bool parity = a.noise != nullptr;

    // ------------------------------------------------------------ load the CTA's share of the row
    const unsigned char* src_row = static_cast<const unsigned char*>(a.logits) + row * a.ld * int64_t(sizeof(T));
    const size_t nbytes = size_t(n_cta) * sizeof(T);
    const size_t bulk = P.tma_ok ? (nbytes & ~size_t(15)) : 0;
    if (threadIdx.x == 0) {
      ms.nan = 0; ms.gmin = 0xFFFFFFFFu; ms.umaxkey[0] = ms.umaxkey[1] = 0u; ms.ngather = 0; ms.theta = 0.f;
      for (int w = 0; w < NW; ++w) ms.wb[w] = 0.f;
      if (bulk) {
        fence_proxy_async();
        mbar_expect_tx(&ms.mbar, uint32_t(bulk));
        const unsigned char* src = src_row + geo.cta_start * int64_t(sizeof(T));
        for (size_t o = 0; o < bulk; o += 32768) {
          const uint32_t nb = uint32_t((bulk - o) < 32768 ? (bulk - o) : 32768);
          bulk_g2s(static_cast<unsigned char*>(data) + o, src + o, nb, &ms.mbar);
        }
      }
    }
    // the Philox key and the noise root (one lane of the last warp)
    NoiseKey nkey{0, 0, 0, 0, 0};
    if (need_race && !parity) {
      const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
      nkey = make_noise_key(a.seed, step, a.row_offset + row);
      if (threadIdx.x == NT - 1) {
        const NoiseRoot rt = noise_root(nkey, V);
        int g = 0;
#pragma unroll
        for (int st = 8; st >= 1; st >>= 1)
          if (g + st < kNumSlices && ms.tstart[g + st] <= rt.s) g += st;
        const int64_t o = rt.s - ms.tstart[g];
        ms.e_root = rt.e_root;
        ms.s_gid = ms.tgbase[g] + local_group(o);
        ms.s_mem = member_index(o);
      }
    }
    {
      const T* src = reinterpret_cast<const T*>(src_row) + geo.cta_start;
      T* dst = static_cast<T*>(data);
      for (int i = int(bulk / sizeof(T)) + threadIdx.x; i < n_cta; i += NT) dst[i] = src[i];
    }
    if (use_pen) {
      const int nw = n_cta / 32 + 1;
      for (int i = threadIdx.x; i < nw; i += NT) pen[i] = 0u;
    }
    __syncthreads();
    if (use_pen) {
      for (int64_t h = threadIdx.x; h < hlen; h += NT) {
        const int64_t id = hist[h];
        if (id >= geo.cta_start && id < geo.cta_end) {
          const int off = int(id - geo.cta_start);
          atomicOr(&pen[off >> 5], 1u << (off & 31));
        }
      }
    }
    // exact noise of this lane's groups: independent of the logits, so it
    // overlaps the bulk copy
    if (need_race && !parity) {
      const NoiseRoot rt{ms.e_root, 0};
      const int64_t gid_s0 = ms.s_gid;
      const int mem_s0 = ms.s_mem;
#pragma unroll
      for (int k = 0; k < kMaxItems; ++k) {
        const int item = warp + k * NW;
        if (item < geo.nitems) {
          int u, p;
          item_of(geo, item, u, p);
          const Unit un = unit_of(geo, u);
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int t = 2 * p + tt;
            const int lg = t * 32 + lane;
            const int n = t < un.ntiles ? group_size(lg, un.L) : 0;
            if (n > 0) {
              const GroupNoise gn = noise_group(nkey, rt, un.gbase + lg, n, gid_s0, mem_s0);
              gnz[threadIdx.x * kSlots + 2 * k + tt] = GNoise{gn.e_min, gn.e2, gn.arg | ((gn.arg2 & 0xFF) << 8)};
            }
          }
        }
      }
    }
    if (bulk) {
      if (!mbar_wait(&ms.mbar, phase, kWaitLimit)) ms.err = 1;
      phase ^= 1u;
    }
    __syncthreads();

    // ------------------------------------------------------------ pass 1: group max and group-relative sums
    float gmax[kSlots], fsum[kSlots];
    bool lnan = false;
#pragma unroll
    for (int k = 0; k < kMaxItems; ++k) {
      const int item = warp + k * NW;
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) { gmax[2 * k + tt] = -INFINITY; fsum[2 * k + tt] = 0.f; }
      if (item < geo.nitems) {
        int u, p;
        item_of(geo, item, u, p);
        const Unit un = unit_of(geo, u);
        // common case: both tiles complete, no penalty, Philox noise -- every
        // block holds 8 valid elements and needs no per-element checks
        const bool lean = !use_pen && !(parity && need_race) && (2 * p + 2) * kTile <= un.L;
        if (lean) {
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int t = 2 * p + tt;
            float m = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const float mb = Max8<T>::run(data, un.uoff + t * kTile + b * 256 + lane * 8, 8);
              lnan |= (mb != mb);
              m = fmaxf(m, mb);
            }
            gmax[2 * k + tt] = m;
            if (!greedy && m > -INFINITY && m < INFINITY) {
              const float c0g = max_coef(m, c1);
              float fb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                float x[8];
                Load8<T>::run(data, un.uoff + t * kTile + b * 256 + lane * 8, 8, x);
#pragma unroll
                for (int i = 0; i < 8; ++i) fb[b] = __fadd_rn(fb[b], unnorm_ftz(x[i], c1, c0g));
              }
              fsum[2 * k + tt] = __fadd_rn(__fadd_rn(fb[0], fb[1]), __fadd_rn(fb[2], fb[3]));
            }
          }
        }
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
          const int t = 2 * p + tt;
          if (!lean && t < un.ntiles) {
            float m = -INFINITY, em = INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const int local = t * kTile + b * 256 + lane * 8;
              const int nv = un.L - local;
              if (nv > 0) {
                const int off = un.uoff + local;
                const uint32_t pb = use_pen ? ((pen[off >> 5] >> (off & 31)) & 0xFFu) : 0u;
                if (pb) {
                  float x[8];
                  Load8<T>::run(data, off, nv, x);
                  apply_penalty8(pb, rpv, x);
#pragma unroll
                  for (int i = 0; i < 8; ++i) { m = fmaxf(m, x[i]); lnan |= (x[i] != x[i]); }
                } else {
                  const float mb = Max8<T>::run(data, off, nv);
                  lnan |= (mb != mb);
                  m = fmaxf(m, mb);
                }
                if (parity && need_race) {
                  const float* nz = a.noise + row * a.noise_ld + geo.cta_start + off;
                  if (P.noise_vec && nv >= 8) {
                    const float4 v0 = __ldg(reinterpret_cast<const float4*>(nz));
                    const float4 v1 = __ldg(reinterpret_cast<const float4*>(nz) + 1);
                    em = fminf(em, fminf(fminf(fminf(v0.x, v0.y), fminf(v0.z, v0.w)),
                                         fminf(fminf(v1.x, v1.y), fminf(v1.z, v1.w))));
                  } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) if (i < nv) em = fminf(em, __ldg(nz + i));
                  }
                }
              }
            }
            gmax[2 * k + tt] = m;
            if (parity && need_race) gnz[threadIdx.x * kSlots + 2 * k + tt].e_min = em;
            if (!greedy && m > -INFINITY && m < INFINITY) {
              const float c0g = max_coef(m, c1);
              // one partial sum per 8-element block (four independent chains)
              float fb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const int local = t * kTile + b * 256 + lane * 8;
                const int nv = un.L - local;
                if (nv > 0) {
                  const int off = un.uoff + local;
                  float x[8];
                  Load8<T>::run(data, off, nv, x);
                  if (use_pen) apply_penalty8((pen[off >> 5] >> (off & 31)) & 0xFFu, rpv, x);
#pragma unroll
                  for (int i = 0; i < 8; ++i) fb[b] = __fadd_rn(fb[b], unnorm_ftz(x[i], c1, c0g));
                }
              }
              fsum[2 * k + tt] = __fadd_rn(__fadd_rn(fb[0], fb[1]), __fadd_rn(fb[2], fb[3]));
            }
          }
        }
        const float im = fmaxf(gmax[2 * k], gmax[2 * k + 1]);
        const unsigned int key = __reduce_max_sync(0xffffffffu, ordered_key(isnan(im) ? -INFINITY : im));
        if (lane == 0) atomicMax(&ms.umaxkey[u], key);
      }
    }
    if (__any_sync(0xffffffffu, lnan) && lane == 0) ms.nan = 1;
    __syncthreads();
    const bool cnan = ms.nan != 0;
    float umax[2] = {ms.umaxkey[0] ? key_to_float(ms.umaxkey[0]) : -INFINITY,
                     ms.umaxkey[1] ? key_to_float(ms.umaxkey[1]) : -INFINITY};
    const float cmax = fmaxf(umax[0], umax[1]);
    const float c0 = max_coef(cmax, c1);
    {
      // this CTA's softmax sum in its own scale: sum_G fsum(G) 2^(c0 - c0_G)
      double sp = 0.0;
      if (!greedy && !cnan && cmax > -INFINITY && fabsf(c0) < INFINITY) {
#pragma unroll
        for (int s = 0; s < kSlots; ++s)
          if (fsum[s] > 0.f) sp += double(__fmul_rn(fsum[s], qe_ex2_ftz(__fsub_rn(c0, max_coef(gmax[s], c1)))));
      }
      for (int o = 16; o; o >>= 1) sp += __shfl_xor_sync(0xffffffffu, sp, o);
      if (lane == 0) ms.wS[warp] = sp;
    }
    const bool race_ok = need_race && !cnan && cmax > -INFINITY && fabsf(c0) < INFINITY;

    // greedy: first id holding the CTA max (NaN first if any).  Needed for
    // greedy and top-k=1 rows, and for rows that turn out non-finite; only a
    // CTA whose own maximum is NaN, infinite or overflows can make a row
    // non-finite, so the scan is skipped everywhere else.
    const bool need_gidx = greedy || (k_on && kk == 1) || cnan || !(cmax > -INFINITY) ||
                           cmax == INFINITY || !(fabsf(c0) < INFINITY);
#pragma unroll
    for (int k = 0; k < kMaxItems; ++k) {
      const int item = warp + k * NW;
      if (need_gidx && item < geo.nitems) {
        int u, p;
        item_of(geo, item, u, p);
        const Unit un = unit_of(geo, u);
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
          const float gm = gmax[2 * k + tt];
          if (cnan || (gm == cmax && n_cta > 0)) {
            const int lg = (2 * p + tt) * 32 + lane;
            for (int m = 0; m < 32; ++m) {
              const int local = int(member_offset(lg, m));
              if (local >= un.L) continue;
              const float x = load1<T>(data, pen, use_pen, rpv, un.uoff + local);
              if (cnan ? (x != x) : (x == cmax)) {
                atomicMin(&ms.gmin, (unsigned int)(geo.cta_start + un.uoff + local));
                break;
              }
            }
          }
        }
      }
    }

    // small top-k: per-warp top-8 group maxima -> CTA lower bound of the k-th largest
    if (small_k) {
      uint32_t keys[kSlots];
#pragma unroll
      for (int s = 0; s < kSlots; ++s)
        keys[s] = (gmax[s] > -INFINITY && !isnan(gmax[s])) ? ordered_key(gmax[s]) : 0u;
      for (int round = 0; round < 8; ++round) {
        uint32_t lb = 0;
#pragma unroll
        for (int s = 0; s < kSlots; ++s) lb = max(lb, keys[s]);
        const uint32_t m = __reduce_max_sync(0xffffffffu, lb);
        if (lane == 0) ms.wtop[warp * 8 + round] = m;
        const uint32_t who = __ballot_sync(0xffffffffu, lb == m && m != 0u);
        if (who && lane == __ffs(who) - 1) {
          bool cleared = false;
#pragma unroll
          for (int s = 0; s < kSlots; ++s)
            if (!cleared && keys[s] == m) { keys[s] = 0u; cleared = true; }
        }
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kMaxR; ++i) wl[i] = Cand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
    }
    __syncthreads();
    uint32_t topk_lkey = 0u;
    if (small_k && warp == 0) {
      constexpr int PER = NW * 8 / 32;
      uint32_t v[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) v[i] = ms.wtop[lane + 32 * i];
      uint32_t L = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t tryk = L | (1u << bit);
        int c = 0;
#pragma unroll
        for (int i = 0; i < PER; ++i) c += __popc(__ballot_sync(0xffffffffu, v[i] >= tryk));
        if (c >= kk) L = tryk;
      }
      topk_lkey = L;
    }

    // ------------------------------------------------------------ race (local, CTA scale)
    // Every CTA finds its own best Rloc tokens exactly.  A group's best ratio
    // is bounded by max(e_arg / E_min, e_max / E2) (its argmin member against
    // the group minimum, every other member against the second smallest
    // value); each warp expands its best-bound group, then every group whose
    // bound still reaches the CTA's Rloc-th best.  What stays unexpanded is
    // summarised by a ceiling on the ratio of every unpublished token.
    // Bounds use approximate logs and divisions (1e-3 margin).
    const bool filtered = p_on || k_on;
    const int Rloc = filtered ? 2 : 1;   // tokens a CTA publishes
    const int Rr = filtered ? 3 : 1;     // per-warp list length (one more for the ceiling)
    float bnd[kSlots];
    unsigned done_mask = 0;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) bnd[s] = -1.f;
    if (race_ok) {
#pragma unroll
      for (int k = 0; k < kMaxItems; ++k) {
        const int item = warp + k * NW;
        if (item < geo.nitems) {
          int u, p;
          item_of(geo, item, u, p);
          const Unit un = unit_of(geo, u);
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int s = 2 * k + tt;
            const int t = 2 * p + tt;
            const int lg = t * 32 + lane;
            const int n = t < un.ntiles ? group_size(lg, un.L) : 0;
            if (n > 0 && gmax[s] > -INFINITY) {
              const float emax = unnorm_ftz(gmax[s], c1, c0);
              const GNoise g = gnz[threadIdx.x * kSlots + s];
              if (parity) {
                bnd[s] = __fdividef(emax, g.e_min);
              } else {
                const float xa = load1<T>(data, pen, use_pen, rpv, un.uoff + int(member_offset(lg, g.args & 0xFF)));
                float b = __fdividef(unnorm_ftz(xa, c1, c0), g.e_min);
                if (n >= 2) b = fmaxf(b, __fdividef(emax, g.e2));
                bnd[s] = b;
              }
            }
          }
        }
      }
    }
    // warp-cooperative exact evaluation of slot `s` of lane `ol` (lane m
    // takes member m)
    auto eval_group = [&](int s, int ol) {
      const int k = s >> 1, tt = s & 1;
      const int item = warp + k * NW;
      int u, p;
      item_of(geo, item, u, p);
      const Unit un = unit_of(geo, u);
      const int t = 2 * p + tt;
      const int lg = t * 32 + ol;
      const int local = int(member_offset(lg, lane));
      // the owner lane's exact group noise
      const GNoise g = gnz[(warp * 32 + ol) * kSlots + s];
      GroupNoise gn;
      gn.e_min = g.e_min;
      gn.e2 = g.e2;
      gn.arg = g.args & 0xFF;
      gn.arg2 = ((g.args >> 8) & 0xFF) == 0xFF ? -1 : ((g.args >> 8) & 0xFF);
      float r = -INFINITY, x = 0.f, E = 1.f;
      int id = 0x7FFFFFFF;
      if (local < un.L) {
        x = load1<T>(data, pen, use_pen, rpv, un.uoff + local);
        id = int(geo.cta_start + un.uoff + local);
        E = parity ? __ldg(a.noise + row * a.noise_ld + id) : noise_token(nkey, gn, id, lane);
        r = __fdiv_rn(unnorm_ftz(x, c1, c0), E);
        if (r != r) r = -INFINITY;
      }
      warp_merge(wl, Rr, r, x, E, id);
    };
    if (race_ok) {
      // Each warp expands its unexpanded groups in bound order while the
      // bound reaches the CTA's running Rloc-th best (a shared maximum of the
      // warps' own Rloc-th bests, which never exceeds the CTA's).
      volatile float* th_cta = &ms.theta;
      volatile float* wbest = ms.wb;
      // Seeds: only the Rloc warps holding the CTA's largest bounds expand
      // before a threshold exists (the others would expand blindly).
      {
        float mb = fmaxf(bnd[0], bnd[1]);
        mb = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(mb, 0.f))));
        if (lane == 0) ms.wbound[warp] = mb;
        __syncthreads();
        float b1 = 0.f, b2 = 0.f;
        for (int w = 0; w < NW; ++w) {
          const float v = ms.wbound[w];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
        }
        const float cut = Rloc == 1 ? b1 : b2;
        if (mb > 0.f && mb >= cut) {
          int bs = bnd[1] > bnd[0] ? 1 : 0;
          const float bb = bs ? bnd[1] : bnd[0];
          int code = bb == mb ? lane * 8 + bs : 0x7FFFFFFF;
          code = int(__reduce_min_sync(0xffffffffu, uint32_t(code)));
          if (code != 0x7FFFFFFF) {
            if (lane == (code >> 3)) done_mask |= 1u << (code & 7);
            eval_group(code & 7, code >> 3);
            __syncwarp();
            const float mine = wl[Rloc - 1].r;
            if (lane == 0 && mine > 0.f) atomicMax(reinterpret_cast<int*>(&ms.theta), __float_as_int(mine));
            if (lane == 0) wbest[warp] = wl[0].r;
          }
        }
        __syncthreads();
      }
      for (;;) {
        float theta = fmaxf(*th_cta, wl[Rloc - 1].r);
        if (Rloc == 2) {
          // the second largest of the warps' bests also bounds the CTA's 2nd
          // (non-negative floats: bit patterns order like the values)
          const uint32_t v = lane < NW ? __float_as_uint(fmaxf(wbest[lane], 0.f)) : 0u;
          const uint32_t v1 = __reduce_max_sync(0xffffffffu, v);
          const int l1 = __ffs(__ballot_sync(0xffffffffu, v == v1)) - 1;
          const uint32_t v2 = __reduce_max_sync(0xffffffffu, lane == l1 ? 0u : v);
          theta = fmaxf(theta, __uint_as_float(v2));
        }
        float bb = -1.f;
        int bs = -1;
#pragma unroll
        for (int s = 0; s < kSlots; ++s)
          if (!((done_mask >> s) & 1u) && bnd[s] > 0.f && bnd[s] >= theta * 0.9999f && bnd[s] > bb) { bb = bnd[s]; bs = s; }
        int code = bs >= 0 ? lane * 8 + bs : 0x7FFFFFFF;
        for (int o = 16; o; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
          const int oc = __shfl_xor_sync(0xffffffffu, code, o);
          if (ob > bb || (ob == bb && oc < code)) { bb = ob; code = oc; }
        }
        if (code == 0x7FFFFFFF) break;
        if (lane == (code >> 3)) done_mask |= 1u << (code & 7);
        eval_group(code & 7, code >> 3);
        __syncwarp();
        const float mine = wl[Rloc - 1].r;
        if (lane == 0 && mine > 0.f) atomicMax(reinterpret_cast<int*>(&ms.theta), __float_as_int(mine));
        if (lane == 0) wbest[warp] = wl[0].r;
      }
      float cm = 0.f;
#pragma unroll
      for (int s = 0; s < kSlots; ++s) if (!((done_mask >> s) & 1u) && bnd[s] > cm) cm = bnd[s];
      for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      if (lane == 0) ms.wceil[warp] = cm;
    }
    __syncthreads();

    // ------------------------------------------------------------ exchange 1: maxima, greedy, sum, race candidates
    {
      Rec1& my = inbox[(ex & 1) * CL + q];
      if (warp == 0) {
        // the CTA's best Rloc tokens and the ceiling over everything else
        constexpr int PER = (NW * 3 + 31) / 32;
        Cand c[PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int idx = lane + 32 * i;
          const int w = idx / 3, j = idx % 3;
          c[i] = (race_ok && idx < NW * 3 && j < Rr) ? wl_all[w * kMaxR + j] : Cand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
        }
        int n = 0;
        float third = 0.f;
        const int want = race_ok ? Rr : 0;
        for (int round = 0; round < want; ++round) {
          int bi = 0;
#pragma unroll
          for (int i = 1; i < PER; ++i) if (rbetter(c[i].r, c[i].id, c[bi].r, c[bi].id)) bi = i;
          Cand cb = c[0];
#pragma unroll
          for (int i = 1; i < PER; ++i) if (i == bi) cb = c[i];
          const int bl = warp_best_lane(cb.r, cb.id);
          if (bl < 0) break;
          if (round == Rloc) { third = __shfl_sync(0xffffffffu, cb.r, bl); break; }
          if (lane == bl) {
            my.cand[n] = cb;
#pragma unroll
            for (int i = 0; i < PER; ++i) if (i == bi) { c[i].r = -INFINITY; c[i].id = 0x7FFFFFFF; }
          }
          ++n;
        }
        if (lane == 0) {
          float ceil_r = third;
          double sv = 0.0;
          for (int w = 0; w < NW; ++w) {
            if (race_ok) ceil_r = fmaxf(ceil_r, ms.wceil[w] * 1.0001f);
            sv += ms.wS[w];
          }
          my.ncand = n;
          my.ceil = ceil_r;
          my.S = sv;
          my.umax[0] = umax[0]; my.umax[1] = umax[1];
          my.c0 = c0;
          my.nan = cnan ? 1 : 0;
          my.gidx = int(ms.gmin == 0xFFFFFFFFu ? 0x7FFFFFFF : ms.gmin);
          my.gval = cnan ? NAN : cmax;
          my.lkey = topk_lkey;
        }
        __syncwarp();
        // push the record into every peer's inbox (DSMEM stores; the cluster
        // barrier below orders them before the peers' reads)
        if (lane < CL && lane != q) {
          const uint4* src = reinterpret_cast<const uint4*>(&my);
          uint4* dst = reinterpret_cast<uint4*>(cluster.map_shared_rank(&my, lane));
#pragma unroll
          for (int i = 0; i < int(sizeof(Rec1) / 16); ++i) dst[i] = src[i];
        }
      }
      cluster.sync();
      if (warp == 0) {
        // lane r reads peer r
        float pm = -INFINITY, pc0 = 0.f, gv = -INFINITY, pceil = 0.f;
        int pn = 0, gi = 0x7FFFFFFF, pnc = 0;
        double pS = 0.0;
        uint32_t lk = 0u;
        Cand pc[2];
        pc[0] = pc[1] = Cand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
        if (lane < CL) {
          const Rec1* sp = &inbox[(ex & 1) * CL + lane];
          for (int u = 0; u < U; ++u) pm = fmaxf(pm, sp->umax[u]);
          pc0 = sp->c0; pn = sp->nan; gi = sp->gidx; gv = sp->gval; lk = sp->lkey; pnc = sp->ncand;
          pS = sp->S; pceil = sp->ceil;
          if (pnc > 0) pc[0] = sp->cand[0];
          if (pnc > 1) pc[1] = sp->cand[1];
        }
        const bool anynan = __any_sync(0xffffffffu, pn != 0);
        const float xM = key_to_float(__reduce_max_sync(0xffffffffu, ordered_key(pm)));
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
          if (oi != 0x7FFFFFFF && (gi == 0x7FFFFFFF || argmax_better(ov, oi, gv, gi))) { gv = ov; gi = oi; }
        }
        lk = __reduce_max_sync(0xffffffffu, lk);
        const float nM = max_coef(xM, c1);
        // row scale: a CTA's ratios and sum times 2^(nM - c0_cta)
        const double sc = (lane < CL && fabsf(pc0) < INFINITY) ? double(qe_ex2_ftz(__fsub_rn(nM, pc0))) : 0.0;
        double Sv = lane < CL ? pS * sc : 0.0;
        for (int o = 16; o; o >>= 1) Sv += __shfl_xor_sync(0xffffffffu, Sv, o);
        const float scf = float(sc);
        // ceilings are >= 0: their bit patterns order like the values
        const float phif = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(lane < CL ? pceil * scf : 0.f)));
#pragma unroll
        for (int i = 0; i < 2; ++i) pc[i].r = pc[i].r > -INFINITY ? pc[i].r * scf : -INFINITY;
        int n = 0, ncomplete = 0;
        for (int round = 0; round < kMaxR; ++round) {
          const int bi = rbetter(pc[1].r, pc[1].id, pc[0].r, pc[0].id) ? 1 : 0;
          const Cand cb = bi ? pc[1] : pc[0];
          const int bl = warp_best_lane(cb.r, cb.id);
          if (bl < 0) break;
          const float br = __shfl_sync(0xffffffffu, cb.r, bl);
          if (lane == bl) {
            rs.cand[n] = cb;
            if (bi) pc[1].r = -INFINITY; else pc[0].r = -INFINITY;
          }
          ++n;
          if (br > phif) ncomplete = n;   // no unpublished token can beat it
        }
        __syncwarp();
        if (lane == 0) {
          rs.xM = xM; rs.nM = nM; rs.c1 = c1;
          rs.p_on = p_on; rs.k_on = k_on; rs.k = kk; rs.tp = tp;
          rs.L = lk ? key_to_float(lk) : -INFINITY;
          rs.S = Sv;
          rs.Sf = float(Sv);
          const bool nonfinite = anynan || !(xM > -INFINITY) || xM == INFINITY ||
                                 (!greedy && !(fabsf(nM) < INFINITY));
          rs.status = greedy ? QE_ROW_GREEDY : (nonfinite ? QE_ROW_NONFINITE : 0);
          rs.out = gi == 0x7FFFFFFF ? 0 : gi;
          rs.ncand = ncomplete > 0 ? ncomplete : (n > 0 ? 1 : 0);
          rs.cb = 0;
          rs.R = 1;
          if (greedy || nonfinite || (k_on && kk == 1)) {
            rs.type = kDone;
          } else if (small_k) {
            rs.type = kGather;
            rs.R = -1;
          } else if (n == 0 || !(rs.Sf > 0.f) || rs.Sf == INFINITY) {
            rs.type = kDone;
            rs.status = QE_ROW_NONFINITE;
          } else if (!filtered) {
            rs.type = kDone;
            rs.out = rs.cand[0].id;
          } else {
            rs.type = kRaceTest;
            rs.L = -INFINITY;
          }
        }
      }
      ++ex;
      __syncthreads();
    }
    if (rs.type == kDone) {
      if (q == 0 && threadIdx.x == 0) {
        a.out_ids[row] = rs.out;
        if (a.out_status) a.out_status[row] = rs.status;
      }
      __syncthreads();
      continue;
    }

    // ------------------------------------------------------------ pass 2 (sparse): candidate tests, gather
    // Round 0 tests the row's best candidate alone (it is in the kept set for
    // most rows, and its high logit lets most groups be skipped); if it is
    // rejected, round 1 tests the remaining complete candidates; if those
    // are rejected too, a gather round collects every token >= the best
    // rejected candidate (the kept set is a prefix of the order).
    const float nM = rs.nM;
    float Fl[kMaxR];
    int Cl[kMaxR];
#pragma unroll 1
    for (int round = 0; round < 3; ++round) {
      const bool do_test = rs.type == kRaceTest;
      const bool do_gather = rs.type == kGather;
      const int cb = do_test ? rs.cb : 0;
      const int R = do_test ? rs.R : 0;
      float cv[kMaxR];
      int cidv[kMaxR];
#pragma unroll
      for (int c = 0; c < kMaxR; ++c) {
        cv[c] = c < R ? rs.cand[cb + c].x : INFINITY;
        cidv[c] = c < R ? rs.cand[cb + c].id : 0;
        Fl[c] = 0.f;
        Cl[c] = 0;
      }
      float thmin = INFINITY;  // tokens at or below this are behind every candidate
#pragma unroll
      for (int c = 0; c < kMaxR; ++c) if (c < R) thmin = fminf(thmin, cv[c]);
      thmin = nextafterf(thmin, -INFINITY);
      const float Lg = rs.L;
      if (threadIdx.x == 0) ms.ngather = 0;
      __syncthreads();
      const int item = warp;
      if (item < geo.nitems) {
        int u, p;
        item_of(geo, item, u, p);
        const Unit un = unit_of(geo, u);
#pragma unroll 1
        for (int tt = 0; tt < 2; ++tt) {
          const int t = 2 * p + tt;
          const float gm = tt ? gmax[1] : gmax[0];
          const bool q_test = do_test && t < un.ntiles && gm > thmin;
          const bool q_gath = do_gather && t < un.ntiles && gm >= Lg;
          const uint32_t tmask = __ballot_sync(0xffffffffu, q_test);
          if (do_test && __popc(tmask) <= kSparseGroups) {
            // few active groups: the warp walks them one at a time, lane m
            // on member m (each group costs one pass instead of a tile's four)
            uint32_t mleft = tmask;
            while (mleft) {
              const int ol = __ffs(mleft) - 1;
              mleft &= mleft - 1;
              const int local = int(member_offset(t * 32 + ol, lane));
              if (local < un.L) {
                const float x = load1<T>(data, pen, use_pen, rpv, un.uoff + local);
                if (x > thmin) {
                  const int id = int(geo.cta_start) + un.uoff + local;
                  const float e = unnorm_ftz(x, c1, nM);
#pragma unroll
                  for (int c = 0; c < kMaxR; ++c)
                    if (c < R && (x > cv[c] || (x == cv[c] && id < cidv[c]))) { Fl[c] += e; Cl[c] += 1; }
                }
              }
            }
          } else if (__any_sync(0xffffffffu, q_test || q_gath)) {
#pragma unroll 1
            for (int b = 0; b < 4; ++b) {
              const int local = t * kTile + b * 256 + lane * 8;
              const int nv = max(0, min(8, un.L - local));
              const int off = un.uoff + local;
              float x[8];
              Load8<T>::run(data, off, nv, x);
              if (use_pen) apply_penalty8((pen[off >> 5] >> (off & 31)) & 0xFFu, rpv, x);
              if (q_test && R == 1) {
                // one candidate (round 0): a compare, an exponential, two adds
                const int id0 = int(geo.cta_start) + off;
                const float v = cv[0];
                const int cid = cidv[0];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (x[i] > v || (x[i] == v && id0 + i < cid)) { Fl[0] += unnorm_ftz(x[i], c1, nM); Cl[0] += 1; }
              } else if (q_test) {
                const int id0 = int(geo.cta_start) + off;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  if (x[i] > thmin) {
                    // a token is ahead of candidate c iff (x, -id) > (x_c, -id_c)
                    const float e = unnorm_ftz(x[i], c1, nM);
#pragma unroll
                    for (int c = 0; c < kMaxR; ++c) {
                      if (c < R && (x[i] > cv[c] || (x[i] == cv[c] && id0 + i < cidv[c]))) { Fl[c] += e; Cl[c] += 1; }
                    }
                  }
                }
              }
              if (do_gather) {
                unsigned mask = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) mask |= ((q_gath && i < nv && x[i] >= Lg) ? 1u : 0u) << i;
                gather_append(mask, x, geo.cta_start + off, gath, &ms.ngather);
              }
            }
          }
        }
      }
      // reductions and exchange
#pragma unroll
      for (int c = 0; c < kMaxR; ++c) {
        if (c < R) {
          float f = Fl[c];
          int n = Cl[c];
          for (int o = 16; o; o >>= 1) {
            f += __shfl_xor_sync(0xffffffffu, f, o);
            n += __shfl_xor_sync(0xffffffffu, n, o);
          }
          if (lane == 0) { ms.wF[warp][c] = f; ms.wcnt[warp][c] = n; }
        }
      }
      __syncthreads();
      Share& my2 = share[ex & 1];
      if (threadIdx.x == 0) {
        for (int c = 0; c < R; ++c) {
          double f = 0.0; long long n = 0;
          for (int w = 0; w < NW; ++w) { f += double(ms.wF[w][c]); n += ms.wcnt[w][c]; }
          my2.F[c] = f; my2.cnt[c] = n;
        }
        my2.ngather = ms.ngather;
        my2.overflow = ms.ngather > kGatherCap ? 1 : 0;
      }
      cluster.sync();
      if (threadIdx.x < CL) {
        const Share* sh = cluster.map_shared_rank(&share[ex & 1], int(threadIdx.x));
        Share& d = peers[threadIdx.x];
        d.ngather = sh->ngather;
        d.overflow = sh->overflow;
        for (int c = 0; c < R; ++c) { d.F[c] = sh->F[c]; d.cnt[c] = sh->cnt[c]; }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int ngat = 0, ovf = 0;
        for (int r = 0; r < CL; ++r) { ngat += peers[r].ngather; ovf |= peers[r].overflow; }
        if (do_test) {
          // exact ratios; the first candidate in race order inside the kept
          // set wins (selection over a bit mask: no local arrays)
          unsigned left = (1u << R) - 1u;
          int win = -1;
          float Lx = rs.L;
          while (left) {
            int c = -1;
            float rc = 0.f;
            for (int i = 0; i < R; ++i) {
              if (!((left >> i) & 1u)) continue;
              const Cand& ci = rs.cand[cb + i];
              const float ri = __fdiv_rn(__fdiv_rn(unnorm_ftz(ci.x, c1, nM), rs.Sf), ci.E);
              if (c < 0 || rbetter(ri, ci.id, rc, rs.cand[cb + c].id)) { c = i; rc = ri; }
            }
            left &= ~(1u << c);
            double Fc = 0.0;
            long long Cc = 0;
            for (int r = 0; r < CL; ++r) { Fc += peers[r].F[c]; Cc += peers[r].cnt[c]; }
            const bool okp = !p_on || Fc <= double(tp) * rs.S;
            const bool okk = !k_on || Cc < kk;
            if (okp && okk) { win = c; break; }
            Lx = fmaxf(Lx, rs.cand[cb + c].x);
          }
          rs.L = Lx;
          if (win >= 0) {
            rs.type = kDone;
            rs.out = rs.cand[cb + win].id;
          } else if (cb + R < rs.ncand) {
            rs.cb = cb + R;                       // test the remaining complete candidates
            rs.R = rs.ncand - (cb + R);
          } else {
            rs.type = kGather;                    // every kept token is >= the best rejected candidate
            rs.R = -1;
          }
        } else {
          rs.type = (ovf || ngat > P.merge_cap) ? kSlow : kGather;
          rs.R = ngat;
        }
      }
      ++ex;
      __syncthreads();
      if (!(rs.type == kRaceTest || (rs.type == kGather && rs.R == -1))) break;
    }
    if (rs.type == kDone) {
      if (q == 0 && threadIdx.x == 0) {
        a.out_ids[row] = rs.out;
        if (a.out_status) a.out_status[row] = rs.status;
      }
      __syncthreads();
      continue;
    }
    if (rs.type == kGather) {
      if (q == 0) gather_finish<T, CL>(P, row, cluster, data, gath, &share[(ex - 1) & 1], rs, ms);
      __syncthreads();
      continue;
    }
    // kSlow: the cluster finishes the row exactly, each CTA on its own slice
    cluster_exact<T, CL>(P, row, cluster, data, pen, gath, rs, use_pen, rpv, geo.cta_start, n_cta,
                         ms.slow_int, ms.wb, (race_ok && !parity) ? gnz : nullptr, geo);
  }
  // do not leave while peers may still read this CTA's shared memory
  cluster.sync();
  if (threadIdx.x == 0 && ms.err) atomicExch(a.ws.err, 1);
}

// ---------------------------------------------------------------- host launch
template <typename T, int CL>
static int launch_cfg(const KernelArgs& ka, cudaStream_t st, int cap) {
  using SM = Smem<T, CL>;
  constexpr int NT = Cfg<CL>::NT;
  const size_t smem = SM::total(cap);
  static int configured_cap = -1;
  static int max_clusters = 0;
  auto kern = fused_kernel<T, CL>;
  if (configured_cap != cap) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e == cudaSuccess && CL > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("fused: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) return set_error(QE_ERR_CUDA, std::string("fused: occupancy query failed: ") + cudaGetErrorString(e));
    max_clusters = n;
    configured_cap = cap;
    if (const char* dbg = std::getenv("QE_DEBUG")) {
      if (dbg[0] == '1')
        std::fprintf(stderr, "[qe] fused: cluster %d x %d threads, %zu B smem/CTA, cap %d, max active clusters %d\n",
                     CL, NT, smem, cap, n);
    }
  }
  FusedParams P;
  P.a = ka;
  P.cap = cap;
  const uintptr_t base = reinterpret_cast<uintptr_t>(ka.logits);
  P.tma_ok = (base % 16 == 0) && ((ka.ld * int64_t(sizeof(T))) % 16 == 0);
  P.noise_vec = ka.noise && (reinterpret_cast<uintptr_t>(ka.noise) % 16 == 0) && (ka.noise_ld % 4 == 0);
  int mc = 1;
  while (size_t(mc) * 2 * 8 <= size_t(cap) * sizeof(T)) mc *= 2;
  P.merge_cap = mc;
  const int ncl = int(ka.batch < max_clusters ? ka.batch : max_clusters);
  P.nclusters = ncl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(ncl * CL));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr; cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("fused launch: ") + cudaGetErrorString(e));
  return QE_OK;
}

}  // namespace fz

// Capacity (elements per CTA) the fused path needs for V, or 0 if unsupported.
int fused_capacity(int64_t V, int cluster) {
  const int U = 16 / cluster;
  int64_t mx = 0;
  for (int q = 0; q < cluster; ++q) {
    const int64_t n = slice_start(q * U + U, V) - slice_start(q * U, V);
    if (n > mx) mx = n;
  }
  int64_t cap = ((mx + 1023) / 1024) * 1024;
  if (cap < 8192) cap = 8192;  // room for CTA 0 to sort >= 1024 gathered keys
  const int NW = cluster == 8 ? 16 : 8;
  // every warp owns at most kMaxItems tile pairs
  for (int q = 0; q < cluster; ++q) {
    int items = 0;
    for (int u = 0; u < U; ++u) {
      const int64_t L = slice_start(q * U + u + 1, V) - slice_start(q * U + u, V);
      items += int(((L + kTile - 1) / kTile + 1) / 2);
    }
    if (items > fz::kMaxItems * NW) return 0;
  }
  return int(cap);
}

int launch_fused(const KernelArgs& ka, cudaStream_t st, int cluster) {
  const int cap = fused_capacity(ka.vocab, cluster);
  if (!cap) return set_error(QE_ERR_UNSUPPORTED, "fused path: vocab too large");
  if (cluster == 16) {
    switch (ka.dtype) {
      case QE_DTYPE_F32: return fz::launch_cfg<float, 16>(ka, st, cap);
      case QE_DTYPE_BF16: return fz::launch_cfg<__nv_bfloat16, 16>(ka, st, cap);
      case QE_DTYPE_F16: return fz::launch_cfg<__half, 16>(ka, st, cap);
    }
  } else {
    switch (ka.dtype) {
      case QE_DTYPE_F32: return fz::launch_cfg<float, 8>(ka, st, cap);
      case QE_DTYPE_BF16: return fz::launch_cfg<__nv_bfloat16, 8>(ka, st, cap);
      case QE_DTYPE_F16: return fz::launch_cfg<__half, 8>(ka, st, cap);
    }
  }
  return set_error(QE_ERR_INVALID, "unknown dtype");
}

}  // namespace qe
