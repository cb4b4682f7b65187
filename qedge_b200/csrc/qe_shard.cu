// qe_shard.cu — vocab-sharded sampling (tensor-parallel lm_head).
//
// Each GPU holds the logits of a contiguous block of canonical vocab slices
// (16 / nshards slices, so every shard boundary is a slice boundary and the
// Philox noise tree is the same as on one GPU).  A step is:
//
//   summarize   one CTA per (row, local slice): slice max, greedy id, the
//               slice's softmax sum in its own scale, its exact local race
//               top-2 with a ceiling over every other token (the same lazy
//               race as the fused kernel), and, for rows with top-k <= 64,
//               the slice's top-k tokens (ordered keys with their noise)
//   all-gather  of the fixed-size slice records (the caller, e.g. NCCL)
//   merge       one CTA per row, identical on every GPU: row max and sum,
//               greedy rows, small top-k rows (sorted merge, prefix mass,
//               race over the kept set), unfiltered race rows (best complete
//               candidate).  Rows with a top-p filter and no small top-k keep
//               up to four complete candidates for a test round.
//   test        one CTA per (row, local slice) of the pending rows: mass and
//               count of the slice's tokens ahead of each candidate
//   all-gather  of the test partials
//   decide      one warp per pending row: the first candidate in race order
//               inside the kept set wins; if none is, the row is marked
//               QE_ROW_SLOW with id -1 and the caller finishes it exactly
//               (e.g. by gathering that row and calling qe_sample).
//
// The sums are combined in slice order in double, so every GPU reaches the
// same decision.  Replaces the single-GPU BatchSampler.forward
// (src/compute/sampler.py:25-41) when the lm_head output is vocab-sharded.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "qe_common.cuh"
#include "qe_fused_util.cuh"
#include "qe_internal.h"

namespace qe {
namespace sh {
using namespace fz;

constexpr int kNT = 256;            // threads per summary / test CTA
constexpr int kNW = kNT / 32;
constexpr int kTopK = 64;           // small top-k rows: keys a slice keeps
constexpr int kGatherMax = 2048;    // elements >= the top-k bound held for sorting
constexpr int kMaxCand = 4;         // race candidates tested per pending row
constexpr int kMaxSliceLen = 16384; // two tiles per warp
constexpr int kSmallK = 64;

struct ShCand {
  float r;   // ratio e/E (slice scale in a record, row scale in a test)
  float x;   // penalised logit
  float E;   // noise
  int id;    // global token id
};

struct alignas(16) SliceRec {
  float xmax;   // max penalised logit (NaN ignored; -inf if none)
  float c0;     // max_coef(xmax, c1)
  int nan;
  int gidx;     // greedy id (global) or 0x7FFFFFFF
  float gval;
  int ncand;
  float ceil;   // ratio bound of every token of the slice not in cand[]
  int nk;       // keys in the top-k list
  double S;     // softmax sum relative to c0
  double pad;
  ShCand cand[2];
  unsigned long long keys[kTopK];   // (ordered x << 32) | ~id, descending
  float kE[kTopK];                  // noise of each listed token
};

struct alignas(16) RowTest {
  int pending;
  int R;
  float nM, Sf;
  double S;
  ShCand cand[kMaxCand];            // race order (approximate), all complete
};

struct alignas(16) TestRec {
  double F[kMaxCand];
  long long cnt[kMaxCand];
};

struct RowParams {
  float T, tp, rp, c1;
  int k;
  bool greedy, k_on, p_on, use_pen, small_k;
  const int32_t* hist;
  int64_t hlen;
};

__device__ __forceinline__ RowParams row_params(const KernelArgs& a, int64_t row) {
  RowParams p;
  p.T = a.temperatures[row];
  p.greedy = (a.flags & QE_FLAG_ALL_GREEDY) || !(p.T > kGreedyEps);
  p.k = a.top_ks ? a.top_ks[row] : 0;
  p.k_on = p.k > 0 && int64_t(p.k) < a.vocab;
  p.tp = a.top_ps ? a.top_ps[row] : 1.f;
  p.p_on = (a.flags & QE_FLAG_USE_TOP_P) && a.top_ps && p.tp < 1.f;
  p.rp = a.rep_penalties ? a.rep_penalties[row] : 1.f;
  p.hist = nullptr;
  p.hlen = 0;
  if (a.history) {
    p.hist = a.history + row * a.history_ld;
    p.hlen = a.history_lens ? a.history_lens[row] : a.history_ld;
    if (p.hlen > a.history_ld) p.hlen = a.history_ld;
    if (p.hlen < 0) p.hlen = 0;
  }
  p.use_pen = p.hist && p.hlen > 0 && p.rp != 1.f;
  p.small_k = !p.greedy && p.k_on && p.k <= kSmallK && p.k > 1;
  p.c1 = p.greedy ? 0.f : temp_coef(p.T);
  return p;
}

__device__ __forceinline__ unsigned long long elem_key(float x, int id) {
  return (uint64_t(ordered_key(x)) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(id));
}

// Shared memory of the summary kernel (after the slice data).
struct SumSmem {
  unsigned long long keys[kGatherMax];
  uint32_t pen[kMaxSliceLen / 32 + 1];
  float g_emin[kNT * 2], g_e2[kNT * 2];
  int g_args[kNT * 2];
  ShCand wl[kNW][3];
  float wceil[kNW], wbest[kNW];
  double wS[kNW];
  unsigned int wtop[kNW * 8];
  unsigned int umaxkey, gmin;
  int nan, ngather, nk;
  float theta;
  unsigned int lkey;
};

template <typename T>
__device__ __forceinline__ float load1(const T* data, const uint32_t* pen, bool use_pen, float rp, int off) {
  float x;
  if constexpr (sizeof(T) == 4) x = reinterpret_cast<const float*>(data)[off];
  else if constexpr (std::is_same<T, __half>::value) x = __half2float(data[off]);
  else x = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(data)[off]) << 16);
  if (use_pen && ((pen[off >> 5] >> (off & 31)) & 1u)) x = penalise(x, rp);
  return x;
}

// Insert into a warp's sorted 3-entry list (lane 0 owns it).
__device__ __forceinline__ void list3_insert(ShCand* l, int n, const ShCand& c) {
  if (!rbetter(c.r, c.id, l[n - 1].r, l[n - 1].id)) return;
  int i = n - 1;
  while (i > 0 && rbetter(c.r, c.id, l[i - 1].r, l[i - 1].id)) { l[i] = l[i - 1]; --i; }
  l[i] = c;
}

// ---------------------------------------------------------------- summarize
template <typename T>
__global__ void __launch_bounds__(kNT) summarize_kernel(KernelArgs a, int shard, int nsl, int64_t shard_start,
                                                        SliceRec* out) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* data = reinterpret_cast<T*>(smem_raw);
  SumSmem& sm = *reinterpret_cast<SumSmem*>(smem_raw + kMaxSliceLen * sizeof(T));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t V = a.vocab;
  const int64_t row = blockIdx.y;
  const int g = shard * nsl + int(blockIdx.x);
  const int64_t s0 = slice_start(g, V), s1 = slice_start(g + 1, V);
  const int L = int(s1 - s0);
  const int ntiles = (L + kTile - 1) / kTile;
  const RowParams rp = row_params(a, row);
  const bool parity = a.noise != nullptr;
  const bool need_race = !rp.greedy && !(rp.k_on && rp.k == 1) && !rp.small_k;
  const float c1 = rp.c1;

  // load the slice (16-byte vectors when the row allows it)
  const T* src = static_cast<const T*>(a.logits) + row * a.ld + (s0 - shard_start);
  const bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0);
  constexpr int EPV = 16 / sizeof(T);
  if (vec) {
    const int nv = L / EPV;
    for (int i = threadIdx.x; i < nv; i += kNT)
      reinterpret_cast<uint4*>(data)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    for (int i = nv * EPV + threadIdx.x; i < L; i += kNT) data[i] = src[i];
  } else {
    for (int i = threadIdx.x; i < L; i += kNT) data[i] = src[i];
  }
  for (int i = threadIdx.x; i < kMaxSliceLen / 32 + 1; i += kNT) sm.pen[i] = 0u;
  if (threadIdx.x == 0) {
    sm.umaxkey = 0u; sm.gmin = 0xFFFFFFFFu; sm.nan = 0; sm.ngather = 0; sm.theta = 0.f; sm.nk = 0;
  }
  if (threadIdx.x < kNW) sm.wbest[threadIdx.x] = 0.f;
  __syncthreads();
  if (rp.use_pen) {
    for (int64_t h = threadIdx.x; h < rp.hlen; h += kNT) {
      const int64_t id = rp.hist[h];
      if (id >= s0 && id < s1) atomicOr(&sm.pen[(id - s0) >> 5], 1u << ((id - s0) & 31));
    }
  }
  __syncthreads();

  // pass 1: group max and group-relative sums (lane owns groups of tiles 2w, 2w+1)
  float gmax[2], fsum[2], gEmin[2];
  bool lnan = false;
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    gmax[tt] = -INFINITY; fsum[tt] = 0.f; gEmin[tt] = INFINITY;
    const int t = 2 * warp + tt;
    if (t < ntiles) {
      float m = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int off = t * kTile + b * 256 + lane * 8;
        const int nv = L - off;
        if (nv > 0) {
          float x[8];
          Load8<T>::run(data, off, nv, x);
          if (rp.use_pen) apply_penalty8((sm.pen[off >> 5] >> (off & 31)) & 0xFFu, rp.rp, x);
#pragma unroll
          for (int i = 0; i < 8; ++i) { m = fmaxf(m, x[i]); lnan |= (x[i] != x[i]); }
          if (parity && need_race) {
            const float* nz = a.noise + row * a.noise_ld + (s0 - shard_start) + off;
#pragma unroll
            for (int i = 0; i < 8; ++i) if (i < nv) gEmin[tt] = fminf(gEmin[tt], __ldg(nz + i));
          }
        }
      }
      gmax[tt] = m;
      if (!rp.greedy && m > -INFINITY && m < INFINITY) {
        const float c0g = max_coef(m, c1);
        float fs = 0.f;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int off = t * kTile + b * 256 + lane * 8;
          const int nv = L - off;
          if (nv > 0) {
            float x[8];
            Load8<T>::run(data, off, nv, x);
            if (rp.use_pen) apply_penalty8((sm.pen[off >> 5] >> (off & 31)) & 0xFFu, rp.rp, x);
#pragma unroll
            for (int i = 0; i < 8; ++i) fs = __fadd_rn(fs, unnorm_ftz(x[i], c1, c0g));
          }
        }
        fsum[tt] = fs;
      }
    }
  }
  {
    const float im = fmaxf(isnan(gmax[0]) ? -INFINITY : gmax[0], isnan(gmax[1]) ? -INFINITY : gmax[1]);
    const unsigned key = __reduce_max_sync(0xffffffffu, im > -INFINITY ? ordered_key(im) : 0u);
    if (lane == 0 && key) atomicMax(&sm.umaxkey, key);
    if (__any_sync(0xffffffffu, lnan) && lane == 0) sm.nan = 1;
  }
  __syncthreads();
  const bool cnan = sm.nan != 0;
  const float cmax = sm.umaxkey ? key_to_float(sm.umaxkey) : -INFINITY;
  const float c0 = max_coef(cmax, c1);
  const bool finite = !cnan && cmax > -INFINITY && fabsf(c0) < INFINITY;
  {
    double sp = 0.0;
    if (!rp.greedy && finite) {
#pragma unroll
      for (int tt = 0; tt < 2; ++tt)
        if (fsum[tt] > 0.f) sp += double(__fmul_rn(fsum[tt], qe_ex2_ftz(__fsub_rn(c0, max_coef(gmax[tt], c1)))));
    }
    for (int o = 16; o; o >>= 1) sp += __shfl_xor_sync(0xffffffffu, sp, o);
    if (lane == 0) sm.wS[warp] = sp;
  }
  // greedy id: first id holding the slice max (NaN first if any)
  const bool need_gidx = rp.greedy || (rp.k_on && rp.k == 1) || cnan || !(cmax > -INFINITY) || cmax == INFINITY ||
                         !(fabsf(c0) < INFINITY);
  if (need_gidx) {
    for (int i = threadIdx.x; i < L; i += kNT) {
      const float x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, i);
      if (cnan ? (x != x) : (x == cmax)) atomicMin(&sm.gmin, unsigned(s0 + i));
    }
  }

  // race: exact local top-2 (one for unfiltered rows) and a ceiling
  const bool filtered = rp.p_on || rp.k_on;
  const int Rloc = filtered ? 2 : 1;
  const int Rr = filtered ? 3 : 1;
  const bool race_ok = need_race && finite;
  if (lane == 0)
    for (int i = 0; i < 3; ++i) sm.wl[warp][i] = ShCand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
  NoiseKey nkey{0, 0, 0, 0, 0};
  NoiseRoot rt{0.f, 0};
  int64_t gid_s = -1;
  int mem_s = 0;
  if (!parity && (race_ok || rp.small_k)) {
    const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
    nkey = make_noise_key(row_seed(a, row), step, a.row_offset + row);
    rt = noise_root(nkey, V);
    token_group(rt.s, V, &gid_s, &mem_s);
  }
  float bnd[2] = {-1.f, -1.f};
  unsigned done_mask = 0;
  if (race_ok) {
    const int64_t gbase = slice_group_base(g, V);
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      const int t = 2 * warp + tt;
      const int lg = t * 32 + lane;
      const int n = t < ntiles ? group_size(lg, L) : 0;
      if (n > 0 && gmax[tt] > -INFINITY) {
        const float emax = unnorm_ftz(gmax[tt], c1, c0);
        if (parity) {
          sm.g_emin[threadIdx.x * 2 + tt] = gEmin[tt];
          bnd[tt] = __fdividef(emax, gEmin[tt]);
        } else {
          const GroupNoise gn = noise_group(nkey, rt, gbase + lg, n, gid_s, mem_s);
          sm.g_emin[threadIdx.x * 2 + tt] = gn.e_min;
          sm.g_e2[threadIdx.x * 2 + tt] = gn.e2;
          sm.g_args[threadIdx.x * 2 + tt] = gn.arg | ((gn.arg2 & 0xFF) << 8);
          const float xa = load1<T>(data, sm.pen, rp.use_pen, rp.rp, int(member_offset(lg, gn.arg)));
          float b = __fdividef(unnorm_ftz(xa, c1, c0), gn.e_min);
          if (n >= 2) b = fmaxf(b, __fdividef(emax, gn.e2));
          bnd[tt] = b;
        }
      }
    }
  }
  __syncthreads();
  if (race_ok) {
    volatile float* th = &sm.theta;
    volatile float* wbest = sm.wbest;
    for (;;) {
      float theta = fmaxf(*th, sm.wl[warp][Rloc - 1].r);
      if (Rloc == 2) {
        float b1 = 0.f, b2 = 0.f;
        for (int w = 0; w < kNW; ++w) {
          const float v = wbest[w];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
        }
        theta = fmaxf(theta, b2);
      }
      float bb = -1.f;
      int bs = -1;
#pragma unroll
      for (int tt = 0; tt < 2; ++tt)
        if (!((done_mask >> tt) & 1u) && bnd[tt] > 0.f && bnd[tt] >= theta * 0.9999f && bnd[tt] > bb) { bb = bnd[tt]; bs = tt; }
      int code = bs >= 0 ? lane * 8 + bs : 0x7FFFFFFF;
      for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
        const int oc = __shfl_xor_sync(0xffffffffu, code, o);
        if (ob > bb || (ob == bb && oc < code)) { bb = ob; code = oc; }
      }
      if (code == 0x7FFFFFFF) break;
      const int ol = code >> 3, tt = code & 7;
      if (lane == ol) done_mask |= 1u << tt;
      // expand group (tile 2w+tt, lane ol): lane m takes member m
      const int t = 2 * warp + tt;
      const int lg = t * 32 + ol;
      const int local = int(member_offset(lg, lane));
      float r = -INFINITY, x = 0.f, E = 1.f;
      int id = 0x7FFFFFFF;
      if (local < L) {
        x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, local);
        id = int(s0 + local);
        if (parity) {
          E = __ldg(a.noise + row * a.noise_ld + (id - shard_start));
        } else {
          const int idx = ol * 2 + tt + warp * 64;
          GroupNoise gn;
          gn.e_min = sm.g_emin[idx];
          gn.e2 = sm.g_e2[idx];
          gn.arg = sm.g_args[idx] & 0xFF;
          const int a2 = (sm.g_args[idx] >> 8) & 0xFF;
          gn.arg2 = a2 == 0xFF ? -1 : a2;
          E = noise_token(nkey, gn, id, lane);
        }
        r = __fdiv_rn(unnorm_ftz(x, c1, c0), E);
        if (r != r) r = -INFINITY;
      }
      // merge the 32 members into the warp's list (best Rr)
      for (int round = 0; round < Rr; ++round) {
        const uint32_t k = r > -INFINITY ? ordered_key(r) : 0u;
        const uint32_t km = __reduce_max_sync(0xffffffffu, k);
        if (km == 0u) break;
        const uint32_t im = __reduce_min_sync(0xffffffffu, k == km ? uint32_t(id) : 0xFFFFFFFFu);
        const int bl = __ffs(__ballot_sync(0xffffffffu, k == km && uint32_t(id) == im)) - 1;
        const ShCand c{__shfl_sync(0xffffffffu, r, bl), __shfl_sync(0xffffffffu, x, bl),
                       __shfl_sync(0xffffffffu, E, bl), __shfl_sync(0xffffffffu, id, bl)};
        bool stop = false;
        if (lane == 0) {
          stop = !rbetter(c.r, c.id, sm.wl[warp][Rr - 1].r, sm.wl[warp][Rr - 1].id);
          if (!stop) list3_insert(sm.wl[warp], Rr, c);
        }
        stop = __shfl_sync(0xffffffffu, stop, 0);
        if (stop) break;
        if (lane == bl) r = -INFINITY;
      }
      __syncwarp();
      const float mine = sm.wl[warp][Rloc - 1].r;
      if (lane == 0 && mine > 0.f) atomicMax(reinterpret_cast<int*>(&sm.theta), __float_as_int(mine));
      if (lane == 0) wbest[warp] = sm.wl[warp][0].r;
    }
    float cm = 0.f;
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) if (!((done_mask >> tt) & 1u) && bnd[tt] > cm) cm = bnd[tt];
    cm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(cm)));
    if (lane == 0) sm.wceil[warp] = cm;
  }

  // small top-k: per-warp top-8 group maxima give a bound L of the slice's k-th
  // largest logit (64 distinct elements >= L when k <= 64)
  if (rp.small_k) {
    uint32_t keys[2];
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) keys[tt] = (gmax[tt] > -INFINITY && !isnan(gmax[tt])) ? ordered_key(gmax[tt]) : 0u;
    for (int round = 0; round < 8; ++round) {
      const uint32_t lb = max(keys[0], keys[1]);
      const uint32_t m = __reduce_max_sync(0xffffffffu, lb);
      if (lane == 0) sm.wtop[warp * 8 + round] = m;
      const uint32_t who = __ballot_sync(0xffffffffu, lb == m && m != 0u);
      if (who && lane == __ffs(who) - 1) { if (keys[0] == m) keys[0] = 0u; else keys[1] = 0u; }
    }
  }
  __syncthreads();
  if (rp.small_k && warp == 0) {
    uint32_t v0 = sm.wtop[lane], v1 = sm.wtop[lane + 32];
    uint32_t Lk = 0;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t tryk = Lk | (1u << bit);
      const int c = __popc(__ballot_sync(0xffffffffu, v0 >= tryk)) + __popc(__ballot_sync(0xffffffffu, v1 >= tryk));
      if (c >= rp.k) Lk = tryk;
    }
    if (lane == 0) sm.lkey = Lk;   // 0: fewer than k groups, keep everything
  }
  __syncthreads();
  if (rp.small_k) {
    const uint32_t Lk = sm.lkey;
    for (int i = threadIdx.x; i < L; i += kNT) {
      const float x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, i);
      if (x != x) continue;
      if (ordered_key(x) >= Lk) {
        const int pos = atomicAdd(&sm.ngather, 1);
        if (pos < kGatherMax) sm.keys[pos] = elem_key(x, int(s0 + i));
      }
    }
    __syncthreads();
    int n = sm.ngather;
    if (n > kGatherMax) {
      // heavy ties: find the k-th largest value key exactly, then keep every
      // larger token and the lowest-id ties
      uint32_t kth = 0;
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t tryk = kth | (1u << bit);
        int c = 0;
        for (int i = threadIdx.x; i < L; i += kNT) {
          const float x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, i);
          c += (x == x && ordered_key(x) >= tryk) ? 1 : 0;
        }
        for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (lane == 0) sm.wtop[warp] = unsigned(c);
        __syncthreads();
        int tot = 0;
        for (int w = 0; w < kNW; ++w) tot += int(sm.wtop[w]);
        __syncthreads();
        if (tot >= rp.k) kth = tryk;
      }
      if (threadIdx.x == 0) sm.ngather = 0;
      __syncthreads();
      // strictly larger ones (fewer than k), then ties in id order
      for (int i = threadIdx.x; i < L; i += kNT) {
        const float x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, i);
        if (x == x && ordered_key(x) > kth) {
          const int pos = atomicAdd(&sm.ngather, 1);
          if (pos < kGatherMax) sm.keys[pos] = elem_key(x, int(s0 + i));
        }
      }
      __syncthreads();
      int base = sm.ngather;
      for (int c0i = 0; c0i < L && base < rp.k; c0i += kNT) {
        const int i = c0i + int(threadIdx.x);
        bool tie = false;
        float x = 0.f;
        if (i < L) { x = load1<T>(data, sm.pen, rp.use_pen, rp.rp, i); tie = (x == x && ordered_key(x) == kth); }
        const unsigned bal = __ballot_sync(0xffffffffu, tie);
        if (lane == 0) sm.wtop[warp] = __popc(bal);
        __syncthreads();
        int before = 0, tot = 0;
        for (int w = 0; w < kNW; ++w) { if (w < warp) before += int(sm.wtop[w]); tot += int(sm.wtop[w]); }
        const int rank = base + before + __popc(bal & ((1u << lane) - 1u));
        if (tie && rank < rp.k && rank < kGatherMax) sm.keys[rank] = elem_key(x, int(s0 + i));
        __syncthreads();
        base += tot;
      }
      n = min(base, rp.k);
      __syncthreads();
    }
    // sort the held keys (descending) and keep the first k
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = n + threadIdx.x; i < np2; i += kNT) sm.keys[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < np2 / 2; i += kNT) {
          const int lo = 2 * stride * (i / stride) + (i % stride), hi = lo + stride;
          const bool desc = ((lo & size) == 0);
          const unsigned long long x0 = sm.keys[lo], x1 = sm.keys[hi];
          if ((x0 < x1) == desc) { sm.keys[lo] = x1; sm.keys[hi] = x0; }
        }
        __syncthreads();
      }
    }
    if (threadIdx.x == 0) sm.nk = min(n, rp.k);
  }
  __syncthreads();

  // the record
  SliceRec& rec = out[row * nsl + blockIdx.x];
  if (rp.small_k && int(threadIdx.x) < sm.nk) {
    const unsigned long long k = sm.keys[threadIdx.x];
    rec.keys[threadIdx.x] = k;
    const int id = int(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFu));
    rec.kE[threadIdx.x] = parity ? __ldg(a.noise + row * a.noise_ld + (id - shard_start))
                                 : tree_noise(nkey, rt, gid_s, mem_s, id, V);
  }
  if (warp == 0) {
    ShCand c = (race_ok && lane < kNW * 3 && (lane % 3) < Rr) ? sm.wl[lane / 3][lane % 3]
                                                               : ShCand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
    int n = 0;
    float third = 0.f;
    for (int round = 0; round < (race_ok ? Rr : 0); ++round) {
      const uint32_t k = c.r > -INFINITY ? ordered_key(c.r) : 0u;
      const uint32_t km = __reduce_max_sync(0xffffffffu, k);
      if (km == 0u) break;
      const uint32_t im = __reduce_min_sync(0xffffffffu, k == km ? uint32_t(c.id) : 0xFFFFFFFFu);
      const int bl = __ffs(__ballot_sync(0xffffffffu, k == km && uint32_t(c.id) == im)) - 1;
      if (round == Rloc) { third = __shfl_sync(0xffffffffu, c.r, bl); break; }
      if (lane == bl) { rec.cand[n] = c; c.r = -INFINITY; }
      ++n;
    }
    if (lane == 0) {
      float ceil_r = third;
      double sv = 0.0;
      for (int w = 0; w < kNW; ++w) {
        if (race_ok) ceil_r = fmaxf(ceil_r, sm.wceil[w] * 1.0001f);
        sv += sm.wS[w];
      }
      rec.xmax = cmax;
      rec.c0 = c0;
      rec.nan = cnan ? 1 : 0;
      rec.gidx = sm.gmin == 0xFFFFFFFFu ? 0x7FFFFFFF : int(sm.gmin);
      rec.gval = cnan ? NAN : cmax;
      rec.ncand = n;
      rec.ceil = ceil_r;
      rec.nk = rp.small_k ? sm.nk : 0;
      rec.S = sv;
      rec.pad = 0.0;
    }
  }
}

// ---------------------------------------------------------------- merge
__device__ __forceinline__ const SliceRec& rec_of(const SliceRec* all, int64_t B, int nsl, int64_t row, int g) {
  return all[(int64_t(g / nsl) * B + row) * nsl + (g % nsl)];
}

__global__ void __launch_bounds__(kNT) merge_kernel(KernelArgs a, int nshards, const SliceRec* all, RowTest* tests) {
  __shared__ unsigned long long keys[kNumSlices * kTopK];
  __shared__ float kE[kNumSlices * kTopK];
  __shared__ double wsum[kNW];
  __shared__ int wkc[kNW];
  __shared__ int s_nk;
  __shared__ float s_nM, s_Sf;
  __shared__ int s_type, s_out, s_status;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x, B = a.batch;
  const int nsl = kNumSlices / nshards;
  const RowParams rp = row_params(a, row);
  RowTest& rt = tests[row];
  if (warp == 0) {
    float pm = -INFINITY, gv = -INFINITY, pc0 = 0.f, pceil = 0.f;
    int pn = 0, gi = 0x7FFFFFFF;
    double pS = 0.0;
    ShCand pc[2];
    pc[0] = pc[1] = ShCand{-INFINITY, 0.f, 1.f, 0x7FFFFFFF};
    if (lane < kNumSlices) {
      const SliceRec& r = rec_of(all, B, nsl, row, lane);
      pm = r.xmax; pn = r.nan; gi = r.gidx; gv = r.gval; pc0 = r.c0; pS = r.S; pceil = r.ceil;
      if (r.ncand > 0) pc[0] = r.cand[0];
      if (r.ncand > 1) pc[1] = r.cand[1];
    }
    const bool anynan = __any_sync(0xffffffffu, pn != 0);
    const float xM = key_to_float(__reduce_max_sync(0xffffffffu, pm > -INFINITY ? ordered_key(pm) : ordered_key(-INFINITY)));
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
      if (oi != 0x7FFFFFFF && (gi == 0x7FFFFFFF || argmax_better(ov, oi, gv, gi))) { gv = ov; gi = oi; }
    }
    const float nM = max_coef(xM, rp.c1);
    const float sc = (lane < kNumSlices && fabsf(pc0) < INFINITY) ? qe_ex2_ftz(__fsub_rn(nM, pc0)) : 0.f;
    // the row sum in slice order (every GPU adds in the same order)
    double S = 0.0;
    for (int g = 0; g < kNumSlices; ++g) S += __shfl_sync(0xffffffffu, pS * double(sc), g);
    const float phi = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(lane < kNumSlices ? pceil * sc : 0.f)));
#pragma unroll
    for (int i = 0; i < 2; ++i) pc[i].r = pc[i].r > -INFINITY ? pc[i].r * sc : -INFINITY;
    int n = 0, ncomplete = 0;
    for (int round = 0; round < kMaxCand; ++round) {
      const int bi = rbetter(pc[1].r, pc[1].id, pc[0].r, pc[0].id) ? 1 : 0;
      const ShCand cb = bi ? pc[1] : pc[0];
      const uint32_t k = cb.r > -INFINITY ? ordered_key(cb.r) : 0u;
      const uint32_t km = __reduce_max_sync(0xffffffffu, k);
      if (km == 0u) break;
      const uint32_t im = __reduce_min_sync(0xffffffffu, k == km ? uint32_t(cb.id) : 0xFFFFFFFFu);
      const int bl = __ffs(__ballot_sync(0xffffffffu, k == km && uint32_t(cb.id) == im)) - 1;
      const float br = __shfl_sync(0xffffffffu, cb.r, bl);
      if (lane == bl) {
        rt.cand[n] = cb;
        if (bi) pc[1].r = -INFINITY; else pc[0].r = -INFINITY;
      }
      ++n;
      if (br > phi) ncomplete = n;
    }
    __syncwarp();
    if (lane == 0) {
      const bool nonfinite = anynan || !(xM > -INFINITY) || xM == INFINITY || (!rp.greedy && !(fabsf(nM) < INFINITY));
      const float Sf = float(S);
      int type = 0, out = gi == 0x7FFFFFFF ? 0 : gi;
      int status = rp.greedy ? QE_ROW_GREEDY : (nonfinite ? QE_ROW_NONFINITE : 0);
      rt.pending = 0;
      rt.R = 0;
      if (rp.greedy || nonfinite || (rp.k_on && rp.k == 1)) {
        type = 0;
      } else if (!(Sf > 0.f) || Sf == INFINITY) {
        status = QE_ROW_NONFINITE;
      } else if (rp.small_k) {
        type = 1;
        status = QE_ROW_GATHERED;
      } else if (n == 0) {
        status = QE_ROW_NONFINITE;
      } else if (!(rp.p_on || rp.k_on)) {
        out = rt.cand[0].id;
      } else {
        type = 2;
        out = -1;
        rt.pending = 1;
        rt.R = ncomplete > 0 ? ncomplete : 1;
        rt.nM = nM;
        rt.S = S;
        rt.Sf = Sf;
      }
      s_type = type; s_out = out; s_status = status;
      s_nM = nM; s_Sf = Sf;
    }
  }
  __syncthreads();
  if (s_type == 1) {
    // small top-k: the row's k largest keys are among the slices' lists
    int n = 0;
    for (int g = 0; g < kNumSlices; ++g) {
      const SliceRec& r = rec_of(all, B, nsl, row, g);
      const int nk = r.nk;
      for (int i = threadIdx.x; i < nk; i += kNT) { keys[n + i] = r.keys[i]; kE[n + i] = r.kE[i]; }
      n += nk;
    }
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = n + threadIdx.x; i < np2; i += kNT) { keys[i] = 0ull; kE[i] = 1.f; }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < np2 / 2; i += kNT) {
          const int lo = 2 * stride * (i / stride) + (i % stride), hi = lo + stride;
          const bool desc = ((lo & size) == 0);
          const unsigned long long x0 = keys[lo], x1 = keys[hi];
          if ((x0 < x1) == desc) {
            keys[lo] = x1; keys[hi] = x0;
            const float e0 = kE[lo]; kE[lo] = kE[hi]; kE[hi] = e0;
          }
        }
        __syncthreads();
      }
    }
    const int nn = min(n, rp.k);
    // kept prefix: exclusive mass <= top_p and rank < k (in probabilities)
    const float c1 = rp.c1, nM = s_nM, Sf = s_Sf;
    const int per = (nn + kNT - 1) / kNT;
    const int i0 = threadIdx.x * per;
    double local = 0.0;
    for (int i = i0; i < i0 + per && i < nn; ++i)
      local += double(__fdiv_rn(unnorm_ftz(key_to_float(uint32_t(keys[i] >> 32)), c1, nM), Sf));
    double incl = local;
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    double run = incl - local;
    for (int w = 0; w < warp; ++w) run += wsum[w];
    int kept = 0;
    for (int i = i0; i < i0 + per && i < nn; ++i) {
      if (rp.p_on && !(run <= double(rp.tp))) break;
      ++kept;
      run += double(__fdiv_rn(unnorm_ftz(key_to_float(uint32_t(keys[i] >> 32)), c1, nM), Sf));
    }
    const bool complete = kept == max(0, min(per, nn - i0));
    const unsigned bal = __ballot_sync(0xffffffffu, !complete);
    if (lane == 0) wkc[warp] = bal ? (warp * 32 + __ffs(bal) - 1) : 0x7FFFFFFF;
    __syncthreads();
    int first = 0x7FFFFFFF;
    for (int w = 0; w < kNW; ++w) first = min(first, wkc[w]);
    if (int(threadIdx.x) == first) s_nk = i0 + kept;
    if (threadIdx.x == 0 && first == 0x7FFFFFFF) s_nk = nn;
    __syncthreads();
    const int nK = max(1, min(s_nk, nn));
    float br = -INFINITY;
    int bid = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < nK; i += kNT) {
      const float x = key_to_float(uint32_t(keys[i] >> 32));
      const int id = int(0xFFFFFFFFu - uint32_t(keys[i] & 0xFFFFFFFFu));
      const float r = __fdiv_rn(__fdiv_rn(unnorm_ftz(x, c1, nM), Sf), kE[i]);
      if (rbetter(r, id, br, bid)) { br = r; bid = id; }
    }
    for (int o = 16; o; o >>= 1) {
      const float orr = __shfl_xor_sync(0xffffffffu, br, o);
      const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
      if (rbetter(orr, oid, br, bid)) { br = orr; bid = oid; }
    }
    if (lane == 0) { wsum[warp] = double(br); wkc[warp] = bid; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kNW; ++w)
        if (rbetter(float(wsum[w]), wkc[w], br, bid)) { br = float(wsum[w]); bid = wkc[w]; }
      if (bid == 0x7FFFFFFF) bid = nn > 0 ? int(0xFFFFFFFFu - uint32_t(keys[0] & 0xFFFFFFFFu)) : s_out;
      s_out = bid;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    a.out_ids[row] = s_out;
    if (a.out_status) a.out_status[row] = s_status;
  }
}

// ---------------------------------------------------------------- test and decide
template <typename T>
__global__ void __launch_bounds__(kNT) test_kernel(KernelArgs a, int shard, int nsl, int64_t shard_start,
                                                   const RowTest* tests, TestRec* out) {
  __shared__ uint32_t pen[kMaxSliceLen / 32 + 1];
  __shared__ double wF[kNW][kMaxCand];
  __shared__ long long wC[kNW][kMaxCand];
  const int64_t row = blockIdx.y;
  const RowTest& rt = tests[row];
  if (!rt.pending) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t V = a.vocab;
  const int g = shard * nsl + int(blockIdx.x);
  const int64_t s0 = slice_start(g, V), s1 = slice_start(g + 1, V);
  const int L = int(s1 - s0);
  const RowParams rp = row_params(a, row);
  for (int i = threadIdx.x; i < kMaxSliceLen / 32 + 1; i += kNT) pen[i] = 0u;
  __syncthreads();
  if (rp.use_pen) {
    for (int64_t h = threadIdx.x; h < rp.hlen; h += kNT) {
      const int64_t id = rp.hist[h];
      if (id >= s0 && id < s1) atomicOr(&pen[(id - s0) >> 5], 1u << ((id - s0) & 31));
    }
  }
  __syncthreads();
  const T* src = static_cast<const T*>(a.logits) + row * a.ld + (s0 - shard_start);
  const int R = rt.R;
  float cv[kMaxCand];
  int cid[kMaxCand];
#pragma unroll
  for (int c = 0; c < kMaxCand; ++c) { cv[c] = c < R ? rt.cand[c].x : INFINITY; cid[c] = c < R ? rt.cand[c].id : 0; }
  float F[kMaxCand];
  int C[kMaxCand];
#pragma unroll
  for (int c = 0; c < kMaxCand; ++c) { F[c] = 0.f; C[c] = 0; }
  const float c1 = rp.c1, nM = rt.nM;
  for (int i = threadIdx.x; i < L; i += kNT) {
    float x = float(src[i]);
    if (rp.use_pen && ((pen[i >> 5] >> (i & 31)) & 1u)) x = penalise(x, rp.rp);
    const int id = int(s0 + i);
    bool any = false;
#pragma unroll
    for (int c = 0; c < kMaxCand; ++c) any |= c < R && (x > cv[c] || (x == cv[c] && id < cid[c]));
    if (any) {
      const float e = unnorm_ftz(x, c1, nM);
#pragma unroll
      for (int c = 0; c < kMaxCand; ++c)
        if (c < R && (x > cv[c] || (x == cv[c] && id < cid[c]))) { F[c] += e; C[c] += 1; }
    }
  }
#pragma unroll
  for (int c = 0; c < kMaxCand; ++c) {
    double f = double(F[c]);
    long long n = C[c];
    for (int o = 16; o; o >>= 1) { f += __shfl_xor_sync(0xffffffffu, f, o); n += __shfl_xor_sync(0xffffffffu, n, o); }
    if (lane == 0) { wF[warp][c] = f; wC[warp][c] = n; }
  }
  __syncthreads();
  if (threadIdx.x < kMaxCand) {
    double f = 0.0;
    long long n = 0;
    for (int w = 0; w < kNW; ++w) { f += wF[w][threadIdx.x]; n += wC[w][threadIdx.x]; }
    TestRec& o = out[row * nsl + blockIdx.x];
    o.F[threadIdx.x] = f;
    o.cnt[threadIdx.x] = n;
  }
}

__global__ void decide_kernel(KernelArgs a, int nshards, const RowTest* tests, const TestRec* all) {
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.batch) return;
  const RowTest& rt = tests[row];
  if (!rt.pending) return;
  const int nsl = kNumSlices / nshards;
  const RowParams rp = row_params(a, row);
  // lane c (< R) sums candidate c's partials in slice order
  double F = 0.0;
  long long C = 0;
  if (lane < rt.R) {
    for (int g = 0; g < kNumSlices; ++g) {
      const TestRec& t = all[(int64_t(g / nsl) * a.batch + row) * nsl + (g % nsl)];
      F += t.F[lane];
      C += t.cnt[lane];
    }
  }
  float r = -INFINITY;
  int id = 0x7FFFFFFF;
  bool ok = false;
  if (lane < rt.R) {
    const ShCand& c = rt.cand[lane];
    r = __fdiv_rn(__fdiv_rn(unnorm_ftz(c.x, rp.c1, rt.nM), rt.Sf), c.E);
    id = c.id;
    ok = (!rp.p_on || F <= double(rp.tp) * rt.S) && (!rp.k_on || C < rp.k);
  }
  // the first candidate in race order that is kept
  float br = ok ? r : -INFINITY;
  int bid = ok ? id : 0x7FFFFFFF;
  for (int o = 16; o; o >>= 1) {
    const float orr = __shfl_xor_sync(0xffffffffu, br, o);
    const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
    if (rbetter(orr, oid, br, bid)) { br = orr; bid = oid; }
  }
  // a rejected candidate ahead of it in race order hides nothing (it is not
  // kept), but an accepted one must not be preceded by an untested token:
  // all tested candidates are complete, so the best kept one wins
  if (lane == 0) {
    if (bid != 0x7FFFFFFF) {
      a.out_ids[row] = bid;
      if (a.out_status) a.out_status[row] = 0;
    } else {
      a.out_ids[row] = -1;
      if (a.out_status) a.out_status[row] = QE_ROW_SLOW;
    }
  }
}

template <typename T>
static size_t summary_smem() { return size_t(kMaxSliceLen) * sizeof(T) + sizeof(SumSmem); }

}  // namespace sh
}  // namespace qe

using namespace qe;

namespace {

// Validation shared by the sharded entry points.  `logits` / `noise` point
// at the shard's first column; `vocab` is the full vocabulary.
int shard_args(const qe_sample_args* a, int nshards, KernelArgs& ka) {
  if (!a) return set_error(QE_ERR_INVALID, "args is NULL");
  if (a->struct_size != sizeof(qe_sample_args))
    return set_error(QE_ERR_INVALID, "struct_size mismatch (header/library version skew)");
  if (nshards != 1 && nshards != 2 && nshards != 4 && nshards != 8 && nshards != 16)
    return set_error(QE_ERR_INVALID, "nshards must divide 16 (1, 2, 4, 8 or 16)");
  if (a->batch < 0) return set_error(QE_ERR_INVALID, "batch < 0");
  if (a->vocab < kNumSlices * 8 || a->vocab >= (int64_t(1) << 24))
    return set_error(QE_ERR_INVALID, "vocab must be in [128, 2^24)");
  for (int g = 0; g < kNumSlices; ++g)
    if (slice_start(g + 1, a->vocab) - slice_start(g, a->vocab) > sh::kMaxSliceLen)
      return set_error(QE_ERR_UNSUPPORTED, "sharded path: vocab slices longer than 16384 ids (vocab > 262144)");
  if (a->dtype != QE_DTYPE_F32 && a->dtype != QE_DTYPE_BF16 && a->dtype != QE_DTYPE_F16)
    return set_error(QE_ERR_INVALID, "unknown dtype");
  if (!a->temperatures || !a->out_ids) return set_error(QE_ERR_INVALID, "temperatures and out_ids are required");
  if (a->history && a->history_ld < 0) return set_error(QE_ERR_INVALID, "history_ld < 0");
  if (a->min_ps || a->out_kept || a->out_norm || a->out_probs)
    return set_error(QE_ERR_UNSUPPORTED, "sharded path: min_ps, out_kept, out_norm and out_probs are not supported");
  ka = KernelArgs{};
  ka.dtype = a->dtype;
  ka.batch = a->batch; ka.vocab = a->vocab; ka.ld = a->ld;
  ka.logits = a->logits;
  ka.temperatures = a->temperatures;
  ka.top_ps = a->top_ps;
  ka.top_ks = a->top_ks;
  ka.rep_penalties = a->rep_penalties;
  ka.history = a->history; ka.history_lens = a->history_lens; ka.history_ld = a->history_ld;
  ka.noise = a->noise; ka.noise_ld = a->noise_ld;
  ka.seed = a->seed; ka.seeds = a->seeds; ka.step = a->step; ka.step_ptr = a->step_ptr;
  ka.row_offset = a->row_offset;
  ka.flags = a->flags;
  ka.out_ids = a->out_ids;
  ka.out_status = a->out_status;
  return QE_OK;
}

int launch_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return QE_OK;
}

template <typename T>
int summarize_t(const KernelArgs& ka, int shard, int nsl, int64_t shard_start, sh::SliceRec* out, cudaStream_t st) {
  const size_t smem = sh::summary_smem<T>();
  const cudaError_t e = cudaFuncSetAttribute(sh::summarize_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("shard summarize: ") + cudaGetErrorString(e));
  sh::summarize_kernel<T><<<dim3(unsigned(nsl), unsigned(ka.batch)), sh::kNT, smem, st>>>(ka, shard, nsl, shard_start, out);
  return launch_check("shard summarize launch");
}

template <typename T>
int test_t(const KernelArgs& ka, int shard, int nsl, int64_t shard_start, const sh::RowTest* tests,
           sh::TestRec* out, cudaStream_t st) {
  sh::test_kernel<T><<<dim3(unsigned(nsl), unsigned(ka.batch)), sh::kNT, 0, st>>>(ka, shard, nsl, shard_start, tests, out);
  return launch_check("shard test launch");
}

}  // namespace

extern "C" size_t qe_shard_record_bytes(void) { return sizeof(sh::SliceRec); }
extern "C" size_t qe_shard_test_bytes(void) { return sizeof(sh::RowTest); }
extern "C" size_t qe_shard_partial_bytes(void) { return sizeof(sh::TestRec); }

extern "C" int qe_shard_summarize(const qe_sample_args* a, int shard, int nshards, void* records, void* stream) {
  KernelArgs ka;
  int rc = shard_args(a, nshards, ka);
  if (rc != QE_OK) return rc;
  if (shard < 0 || shard >= nshards) return set_error(QE_ERR_INVALID, "shard out of range");
  if (!a->logits || !records) return set_error(QE_ERR_INVALID, "logits and records are required");
  if (reinterpret_cast<uintptr_t>(records) % 16) return set_error(QE_ERR_INVALID, "records must be 16-byte aligned");
  const int nsl = kNumSlices / nshards;
  const int64_t start = slice_start(shard * nsl, a->vocab);
  const int64_t width = slice_start((shard + 1) * nsl, a->vocab) - start;
  if (a->ld < width) return set_error(QE_ERR_INVALID, "ld < shard width");
  if (a->noise && a->noise_ld < width) return set_error(QE_ERR_INVALID, "noise_ld < shard width");
  if (a->batch == 0) return QE_OK;
  auto* out = static_cast<sh::SliceRec*>(records);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case QE_DTYPE_F32: return summarize_t<float>(ka, shard, nsl, start, out, st);
    case QE_DTYPE_BF16: return summarize_t<__nv_bfloat16>(ka, shard, nsl, start, out, st);
    default: return summarize_t<__half>(ka, shard, nsl, start, out, st);
  }
}

extern "C" int qe_shard_merge(const qe_sample_args* a, int nshards, const void* all_records, void* tests,
                              void* stream) {
  KernelArgs ka;
  int rc = shard_args(a, nshards, ka);
  if (rc != QE_OK) return rc;
  if (!all_records || !tests) return set_error(QE_ERR_INVALID, "all_records and tests are required");
  if (a->batch == 0) return QE_OK;
  sh::merge_kernel<<<unsigned(a->batch), sh::kNT, 0, static_cast<cudaStream_t>(stream)>>>(
      ka, nshards, static_cast<const sh::SliceRec*>(all_records), static_cast<sh::RowTest*>(tests));
  return launch_check("shard merge launch");
}

extern "C" int qe_shard_test(const qe_sample_args* a, int shard, int nshards, const void* tests, void* partials,
                             void* stream) {
  KernelArgs ka;
  int rc = shard_args(a, nshards, ka);
  if (rc != QE_OK) return rc;
  if (shard < 0 || shard >= nshards) return set_error(QE_ERR_INVALID, "shard out of range");
  if (!a->logits || !tests || !partials) return set_error(QE_ERR_INVALID, "logits, tests and partials are required");
  if (a->batch == 0) return QE_OK;
  const int nsl = kNumSlices / nshards;
  const int64_t start = slice_start(shard * nsl, a->vocab);
  auto* t = static_cast<const sh::RowTest*>(tests);
  auto* out = static_cast<sh::TestRec*>(partials);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case QE_DTYPE_F32: return test_t<float>(ka, shard, nsl, start, t, out, st);
    case QE_DTYPE_BF16: return test_t<__nv_bfloat16>(ka, shard, nsl, start, t, out, st);
    default: return test_t<__half>(ka, shard, nsl, start, t, out, st);
  }
}

extern "C" int qe_shard_decide(const qe_sample_args* a, int nshards, const void* tests, const void* all_partials,
                               void* stream) {
  KernelArgs ka;
  int rc = shard_args(a, nshards, ka);
  if (rc != QE_OK) return rc;
  if (!tests || !all_partials) return set_error(QE_ERR_INVALID, "tests and all_partials are required");
  if (a->batch == 0) return QE_OK;
  const unsigned blocks = unsigned((a->batch + 7) / 8);
  sh::decide_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      ka, nshards, static_cast<const sh::RowTest*>(tests), static_cast<const sh::TestRec*>(all_partials));
  return launch_check("shard decide launch");
}
