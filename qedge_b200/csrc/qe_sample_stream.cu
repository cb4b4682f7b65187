// qe_sample_stream.cu — the default sampler path: two launches, the logits
// read from HBM once.
//
// Replaces BatchSampler.forward (src/compute/sampler.py:25-41) and the
// extensions of this library (top-k, min-p, repetition penalty, Philox
// noise).  The semantics of a sample are those of qe_sample_ref.cu and the
// CPU oracle: softmax of the penalised logits / T, kept set = the longest
// prefix of the order (x desc, id asc) allowed by top-k, top-p and min-p,
// token = argmax over the kept set of rho = RN(RN(e/S)/E).
//
// 1. summ_kernel streams the logits: one warp per task of `tpw` tiles (4 KB
//    of logits), each lane one 32-id group at a time held in registers
//    (16-byte loads), reduced to (max, group-relative exponential sum).  No
//    barriers, no shared memory beyond the penalty bits, so enough warps are
//    resident to keep HBM busy.
// 2. row_kernel, one CTA per row, works from the row's group summaries
//    (8 bytes per 32 ids, still in L2):
//      * row max, softmax normaliser S, greedy / top-1 / non-finite rows;
//      * the exponential race: every group's best ratio is bounded by its
//        largest term over its noise minimum (one Philox call per four
//        groups); only groups whose bound reaches 1/16 (the 4th best ratio
//        of a race is below that with probability ~1e-4) are re-read and
//        raced exactly, and the 4 best are complete above that threshold;
//      * the kept-set test of those candidates: bounded from the summaries,
//        or counted exactly over the groups whose max is at or above them;
//      * top-k rows with k <= 64: the k-th largest group max bounds the
//        k-th largest logit, so only those groups are read, sorted and raced;
//      * the exact fallback (candidates all outside the kept set, or the
//        kept-set size asked for): radix rounds over the keys of the groups
//        at or above a floor, the tie rank, and the race over the kept set.
// No kernel waits for another CTA or on any flag.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstring>
#include <mutex>
#include <string>

#include "qe_common.cuh"
#include "qe_fused_util.cuh"
#include "qe_internal.h"
#include "qe_stream.cuh"

namespace qe {
namespace st {

using fz::key_to_float;
using fz::ordered_key;
using fz::rbetter;

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ float lg2_approx(float x) {
  float r;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint32_t nan_key(float v) { return ordered_key(v); }   // NaN above +inf
// Repetition penalty (Hugging Face rule), inline.
__device__ __forceinline__ float pen_x(float x, float rp) { return x < 0.f ? __fmul_rn(x, rp) : __fdiv_rn(x, rp); }
__device__ __forceinline__ bool finite_f(float x) { return x == x && x > -INFINITY && x < INFINITY; }

// ---------------------------------------------------------------- launch parameters
struct Params {
  KernelArgs a;
  int esize;                    // bytes per logit
  int vec_ok;                   // 16-byte loads of logits
  int noise_vec;                // 16-byte loads of caller noise
  int tpw;                      // tiles per warp task (2 for 16-bit types, 1 for fp32)
  int tasks_row;                // warp tasks per row
  int force_exact;              // the kept-set size is asked for
  int dtype_level;              // last radix level that separates the dtype's values
  int64_t G;                    // groups per row
  int64_t sstart[kNumSlices + 1];
  int64_t gbase[kNumSlices + 1];
  int snt[kNumSlices];          // tiles per slice
  int tbase[kNumSlices + 1];    // first warp task of each slice
  Ctl* ctl;
  GroupSum* summ;               // [B][G]
  float* emin;                  // [B][G] noise minimum per group (caller-noise mode)
};

// ---------------------------------------------------------------- row parameters
struct RowP {
  int kind;                     // RowKind
  bool p_on, k_on, m_on, filtered, pen, exact, hash_ok;
  float T, c1, tp, minp, rp;
  long long k;
  const int32_t* hist;          // the row's history ids (repetition penalty)
  int hlen;
  float e_root;                 // noise-tree root (Philox mode)
  int s_mem;
  long long s_gid;
  NoiseKey key;
};

__device__ __forceinline__ RowP row_params(const Params& P, int row) {
  const KernelArgs& a = P.a;
  RowP r;
  const int64_t V = a.vocab;
  r.T = a.temperatures[row];
  const bool greedy = (a.flags & QE_FLAG_ALL_GREEDY) || r.T <= kGreedyEps;
  r.c1 = temp_coef(r.T);
  const long long k = a.top_ks ? (long long)a.top_ks[row] : 0;
  r.k_on = k > 0 && k < V;
  r.k = r.k_on ? k : V;
  r.tp = a.top_ps ? a.top_ps[row] : 1.f;
  r.p_on = (a.flags & QE_FLAG_USE_TOP_P) && a.top_ps && r.tp < 1.f;
  r.minp = a.min_ps ? a.min_ps[row] : 0.f;
  r.m_on = r.minp > 0.f;
  r.filtered = r.k_on || r.p_on || r.m_on;
  r.rp = a.rep_penalties ? a.rep_penalties[row] : 1.f;
  int hl = 0;
  if (a.history && a.rep_penalties) {
    hl = a.history_lens ? a.history_lens[row] : int(a.history_ld);
    hl = hl < 0 ? 0 : (hl > int(a.history_ld) ? int(a.history_ld) : hl);
  }
  r.hlen = hl;
  r.hist = a.history ? a.history + row * a.history_ld : nullptr;
  r.pen = hl > 0 && !(r.rp == 1.f);
  r.hash_ok = hl <= kHashCap / 2;
  r.kind = greedy ? kKindGreedy
                  : (r.k_on && k == 1) ? kKindArgmax : (r.k_on && k <= kSmallK) ? kKindSmallK : kKindRace;
  r.exact = P.force_exact && r.filtered && !greedy && r.kind == kKindRace;
  const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
  r.key = make_noise_key(row_seed(a, row), step, a.row_offset + row);
  r.e_root = 0.f;
  r.s_gid = -1;
  r.s_mem = 0;
  return r;
}

// Slice of global group g of a row.
__device__ __forceinline__ int slice_of_group(const Params& P, int64_t g) {
  int s = 0;
#pragma unroll 1
  while (s + 1 < kNumSlices && P.gbase[s + 1] <= g) ++s;
  return s;
}
__device__ __forceinline__ void token_group_p(const Params& P, int64_t j, int64_t* gid, int* mem) {
  int sl = 0;
#pragma unroll 1
  while (sl + 1 < kNumSlices && P.sstart[sl + 1] <= j) ++sl;
  const int64_t o = j - P.sstart[sl];
  *gid = P.gbase[sl] + local_group(o);
  *mem = member_index(o);
}

// ---------------------------------------------------------------- element loads
template <typename T> struct Cvt;
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
  static __device__ __forceinline__ float one(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
  static __device__ __forceinline__ float one(uint16_t h) { return __half2float(__ushort_as_half(h)); }
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __half2 r = __hmax2_nan(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
};

// The 32 members of the group in lane position l of tile `tile` of a slice
// (member b*8+i at slice offset tile*1024 + b*256 + l*8 + i), -inf past the
// slice's end L.  src: the slice's first logit.
template <typename T>
__device__ __forceinline__ void load_members(const Params& P, const unsigned char* src, int tile, int l, int L,
                                             float x[32]) {
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int off = tile * kTile + b * 256 + l * 8;
    const int nb = L - off;
    if (nb >= 8 && P.vec_ok) {
      if constexpr (sizeof(T) == 2) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(src + size_t(off) * 2));
        x[8 * b + 0] = Cvt<T>::lo(q.x); x[8 * b + 1] = Cvt<T>::hi(q.x);
        x[8 * b + 2] = Cvt<T>::lo(q.y); x[8 * b + 3] = Cvt<T>::hi(q.y);
        x[8 * b + 4] = Cvt<T>::lo(q.z); x[8 * b + 5] = Cvt<T>::hi(q.z);
        x[8 * b + 6] = Cvt<T>::lo(q.w); x[8 * b + 7] = Cvt<T>::hi(q.w);
      } else {
        const float4 q0 = __ldg(reinterpret_cast<const float4*>(src + size_t(off) * 4));
        const float4 q1 = __ldg(reinterpret_cast<const float4*>(src + size_t(off) * 4 + 16));
        x[8 * b + 0] = q0.x; x[8 * b + 1] = q0.y; x[8 * b + 2] = q0.z; x[8 * b + 3] = q0.w;
        x[8 * b + 4] = q1.x; x[8 * b + 5] = q1.y; x[8 * b + 6] = q1.z; x[8 * b + 7] = q1.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float v = -INFINITY;
        if (i < nb) {
          if constexpr (sizeof(T) == 2) v = Cvt<T>::one(__ldg(reinterpret_cast<const uint16_t*>(src) + off + i));
          else v = __ldg(reinterpret_cast<const float*>(src) + off + i);
        }
        x[8 * b + i] = v;
      }
    }
  }
}

// Sum of 2^(x c1 + c0) over 32 values in four chains (chain = member & 3).
__device__ __forceinline__ float group_sum(const float* x, float c1, float c0) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int m = 0; m < 32; m += 4) {
    s0 += qe_ex2_ftz(__fmaf_rn(x[m], c1, c0));
    s1 += qe_ex2_ftz(__fmaf_rn(x[m + 1], c1, c0));
    s2 += qe_ex2_ftz(__fmaf_rn(x[m + 2], c1, c0));
    s3 += qe_ex2_ftz(__fmaf_rn(x[m + 3], c1, c0));
  }
  return (s0 + s1) + (s2 + s3);
}

// First member equal to v (the first NaN when v is NaN).
__device__ __forceinline__ int first_member(const float x[32], float v) {
  const bool vn = v != v;
  int f = 31;
#pragma unroll
  for (int m = 31; m >= 0; --m)
    if (vn ? x[m] != x[m] : x[m] == v) f = m;
  return f;
}

// The same two reductions on 32 packed 16-bit values (word i holds members
// 2i and 2i+1), in group_sum's order.
template <typename T>
__device__ __forceinline__ float group_sum_packed(const uint32_t w[16], float c1, float c0) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    s0 += qe_ex2_ftz(__fmaf_rn(Cvt<T>::lo(w[i]), c1, c0));
    s1 += qe_ex2_ftz(__fmaf_rn(Cvt<T>::hi(w[i]), c1, c0));
    s2 += qe_ex2_ftz(__fmaf_rn(Cvt<T>::lo(w[i + 1]), c1, c0));
    s3 += qe_ex2_ftz(__fmaf_rn(Cvt<T>::hi(w[i + 1]), c1, c0));
  }
  return (s0 + s1) + (s2 + s3);
}
template <typename T>
__device__ __forceinline__ int first_member_packed(const uint32_t w[16], float v) {
  const bool vn = v != v;
  int f = 31;
#pragma unroll
  for (int i = 15; i >= 0; --i) {
    const float hi = Cvt<T>::hi(w[i]), lo = Cvt<T>::lo(w[i]);
    if (vn ? hi != hi : hi == v) f = 2 * i + 1;
    if (vn ? lo != lo : lo == v) f = 2 * i;
  }
  return f;
}

// ---------------------------------------------------------------- 1. summaries
template <typename T>
__global__ void __launch_bounds__(kSumThreads, 3) summ_kernel(const __grid_constant__ Params P) {
  __shared__ uint32_t pen_bits[kSumThreads / 32][64];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const long long task = (long long)blockIdx.x * (blockDim.x >> 5) + wib;
  if (task >= (long long)P.a.batch * P.tasks_row) return;   // the whole warp
  const int row = int(task / P.tasks_row), t = int(task % P.tasks_row);
  int s = 0;
#pragma unroll 1
  while (s + 1 < kNumSlices && P.tbase[s + 1] <= t) ++s;
  const int tile0 = (t - P.tbase[s]) * P.tpw;
  const int64_t sa = P.sstart[s];
  const int L = int(P.sstart[s + 1] - sa);
  const KernelArgs& a = P.a;
  const float temp = a.temperatures[row];
  const long long k = a.top_ks ? (long long)a.top_ks[row] : 0;
  const bool idx_mode = (a.flags & QE_FLAG_ALL_GREEDY) || temp <= kGreedyEps || (k == 1 && a.vocab > 1);
  const float c1 = temp_coef(temp);
  float rpen = 1.f;
  int hl = 0;
  if (a.history && a.rep_penalties) {
    rpen = a.rep_penalties[row];
    hl = a.history_lens ? a.history_lens[row] : int(a.history_ld);
    hl = hl < 0 ? 0 : (hl > int(a.history_ld) ? int(a.history_ld) : hl);
  }
  const bool pen = hl > 0 && !(rpen == 1.f);
  if (pen) {
    pen_bits[wib][lane] = 0u;
    pen_bits[wib][lane + 32] = 0u;
    __syncwarp();
    const int32_t* hist = a.history + row * a.history_ld;
    const int64_t base = int64_t(tile0) * kTile;   // slice offset of the task's first id
    for (int h = lane; h < hl; h += 32) {
      const int64_t o = int64_t(hist[h]) - sa - base;
      if (o >= 0 && o < int64_t(P.tpw) * kTile && base + o < L)
        atomicOr(&pen_bits[wib][(o >> 10) * 32 + ((o >> 3) & 31)], 1u << int(((o >> 8) & 3) * 8 + (o & 7)));
    }
    __syncwarp();
  }
  const unsigned char* src = static_cast<const unsigned char*>(a.logits) + (size_t(row) * size_t(a.ld) + size_t(sa)) * P.esize;
  GroupSum* out = P.summ + size_t(row) * size_t(P.G) + size_t(P.gbase[s]);
  // 16-bit types: both tiles' loads in flight before any arithmetic
  uint32_t wv[2][16];
  bool fast[2] = {false, false};
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      const int tile = tile0 + tt;
      const uint32_t pb = pen ? pen_bits[wib][tt * 32 + lane] : 0u;
      fast[tt] = tt < P.tpw && tile < P.snt[s] && pb == 0u && tile * kTile + kTile <= L && P.vec_ok;
      if (fast[tt]) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(src + size_t(tile * kTile + b * 256 + lane * 8) * 2));
          wv[tt][4 * b] = q.x; wv[tt][4 * b + 1] = q.y; wv[tt][4 * b + 2] = q.z; wv[tt][4 * b + 3] = q.w;
        }
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    if (tt >= P.tpw) break;
    const int tile = tile0 + tt;
    if (tile >= P.snt[s]) break;
    GroupSum r;
    bool done = false;
    if constexpr (sizeof(T) == 2) {
     if (fast[tt]) {
      done = true;
      const uint32_t* w = wv[tt];
      const uint32_t m0 = Cvt<T>::max2(Cvt<T>::max2(w[0], w[1]), Cvt<T>::max2(w[2], w[3]));
      const uint32_t m1 = Cvt<T>::max2(Cvt<T>::max2(w[4], w[5]), Cvt<T>::max2(w[6], w[7]));
      const uint32_t m2 = Cvt<T>::max2(Cvt<T>::max2(w[8], w[9]), Cvt<T>::max2(w[10], w[11]));
      const uint32_t m3 = Cvt<T>::max2(Cvt<T>::max2(w[12], w[13]), Cvt<T>::max2(w[14], w[15]));
      const uint32_t mm = Cvt<T>::max2(Cvt<T>::max2(m0, m1), Cvt<T>::max2(m2, m3));
      const float lo = Cvt<T>::lo(mm), hi = Cvt<T>::hi(mm);
      const float gmax = (lo != lo || hi != hi) ? __int_as_float(0x7FFFFFFF) : fmaxf(lo, hi);
      r.gmax = gmax;
      if (idx_mode || gmax != gmax || (gmax > -INFINITY && !finite_f(__fmul_rn(gmax, c1))))
        r.aux = __int_as_float(first_member_packed<T>(w, gmax));
      else
        r.aux = gmax > -INFINITY ? group_sum_packed<T>(w, c1, -__fmul_rn(gmax, c1)) : 0.f;
     }
    }
    if (!done) {
      float x[32];
      const uint32_t pb = pen ? pen_bits[wib][tt * 32 + lane] : 0u;
      load_members<T>(P, src, tile, lane, L, x);
      if (pb) {
#pragma unroll
        for (int m = 0; m < 32; ++m)
          if ((pb >> m) & 1u) x[m] = pen_x(x[m], rpen);
      }
      float gmax = x[0];
#pragma unroll
      for (int m = 1; m < 32; ++m) gmax = fmax_nan(gmax, x[m]);
      r.gmax = gmax;
      // rows that only need the max's position, and groups whose softmax terms
      // are not finite (the row then falls back to the greedy id), keep the
      // position of the group's max instead of its sum
      if (idx_mode || gmax != gmax || (gmax > -INFINITY && !finite_f(__fmul_rn(gmax, c1))))
        r.aux = __int_as_float(first_member(x, gmax));
      else
        r.aux = gmax > -INFINITY ? group_sum(x, c1, -__fmul_rn(gmax, c1)) : 0.f;
    }
    out[tile * 32 + lane] = r;
    if (a.noise && !idx_mode) {
      // caller-noise mode: the group's smallest noise bounds its best ratio
      const float* nz = a.noise + size_t(row) * size_t(a.noise_ld) + size_t(sa);
      float e = INFINITY;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int off = tile * kTile + b * 256 + lane * 8;
        const int nb = L - off;
        if (nb >= 8 && P.noise_vec) {
          const float4 q0 = __ldg(reinterpret_cast<const float4*>(nz + off));
          const float4 q1 = __ldg(reinterpret_cast<const float4*>(nz + off + 4));
          e = fminf(e, fminf(fminf(fminf(q0.x, q0.y), fminf(q0.z, q0.w)), fminf(fminf(q1.x, q1.y), fminf(q1.z, q1.w))));
        } else {
          for (int i = 0; i < 8 && i < nb; ++i) e = fminf(e, __ldg(nz + off + i));
        }
      }
      P.emin[size_t(row) * size_t(P.G) + size_t(P.gbase[s]) + size_t(tile * 32 + lane)] = e;
    }
  }
}

// ---------------------------------------------------------------- 2. row kernel: shared state
struct Cand {
  float r, x, E;
  int id;
};

// The kTC best (rho desc, id asc) one thread has seen.
struct Top4 {
  float r[kTC], x[kTC], E[kTC];
  int id[kTC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      r[i] = -1.f;
      x[i] = 0.f;
      E[i] = 1.f;
      id[i] = INT_MAX;
    }
  }
  __device__ __forceinline__ void add(float rr, float xx, float EE, int ii) {
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      if (rbetter(rr, ii, r[i], id[i])) {
        const float tr = r[i], tx = x[i], tE = E[i];
        const int ti = id[i];
        r[i] = rr; x[i] = xx; E[i] = EE; id[i] = ii;
        rr = tr; xx = tx; EE = tE; ii = ti;
      }
    }
  }
};

struct alignas(16) RowSm {
  RowP rp;
  uint32_t red_u[kRowWarps];
  int red_i[kRowWarps];
  double red_d[kRowWarps];
  long long red_l[kRowWarps];
  double pd[kRowWarps][kTC];
  long long pl[kRowWarps][kTC];
  Cand wtop[kRowWarps][kTC];
  Cand top[kTC];
  int ntop;
  int n;
  long long bcast;
  unsigned int scnt[256];        // selection histograms (never overlaps the keys they select from)
  int wq[kRowWarps][64];         // per-warp queues of groups to visit
  uint32_t wqw[kRowWarps][64];
  unsigned long long sortk[kSortCap];
  int hash[kHashCap];
  union {
    struct {
      unsigned int cnt[256];
      unsigned long long mass[256];
      unsigned int nm;
    } h;
    unsigned long long keys[kSelCap];
    struct {
      float p[kSmallK];
      int keep[kSmallK];
    } sk;
  } u;
};

__device__ __forceinline__ uint32_t block_max_u(RowSm& sm, uint32_t v) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) sm.red_u[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0u;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r = max(r, sm.red_u[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ uint32_t block_min_u(RowSm& sm, uint32_t v) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) sm.red_u[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0xFFFFFFFFu;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r = min(r, sm.red_u[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ double block_sum_d(RowSm& sm, double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) sm.red_d[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r += sm.red_d[w];
  __syncthreads();
  return r;
}
__device__ __forceinline__ long long block_sum_l(RowSm& sm, long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) sm.red_l[threadIdx.x >> 5] = v;
  __syncthreads();
  long long r = 0;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r += sm.red_l[w];
  __syncthreads();
  return r;
}
// kTC doubles and counts summed over the CTA; totals in every thread.
__device__ __forceinline__ void block_sum4(RowSm& sm, double* ms, long long* ct) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ms[i] += __shfl_xor_sync(0xFFFFFFFFu, ms[i], o);
      ct[i] += __shfl_xor_sync(0xFFFFFFFFu, ct[i], o);
    }
    if (lane == 0) {
      sm.pd[warp][i] = ms[i];
      sm.pl[warp][i] = ct[i];
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    double a = 0.0;
    long long b = 0;
    for (int w = 0; w < kRowWarps; ++w) {
      a += sm.pd[w][i];
      b += sm.pl[w][i];
    }
    ms[i] = a;
    ct[i] = b;
  }
  __syncthreads();
}

// ---------------------------------------------------------------- history hash (repetition penalty)
__device__ __forceinline__ uint32_t hslot(int id) { return (uint32_t(id) * 2654435761u) >> 19; }   // 13 bits
__device__ __forceinline__ void hash_build(RowSm& sm, const RowP& rp, int64_t V) {
  for (int i = threadIdx.x; i < kHashCap; i += kRowThreads) sm.hash[i] = -1;
  __syncthreads();
  if (rp.hash_ok) {
    for (int h = threadIdx.x; h < rp.hlen; h += kRowThreads) {
      const int id = rp.hist[h];
      if (id < 0 || int64_t(id) >= V) continue;
      uint32_t s = hslot(id);
#pragma unroll 1
      for (int probe = 0; probe < kHashCap; ++probe) {
        const int prev = atomicCAS(&sm.hash[s], -1, id);
        if (prev == -1 || prev == id) break;
        s = (s + 1u) & uint32_t(kHashCap - 1);
      }
    }
  }
  __syncthreads();
}
__device__ __forceinline__ bool in_history(const RowSm& sm, const RowP& rp, int id) {
  if (rp.hash_ok) {
    uint32_t s = hslot(id);
#pragma unroll 1
    for (int probe = 0; probe < kHashCap; ++probe) {
      const int v = sm.hash[s];
      if (v == id) return true;
      if (v == -1) return false;
      s = (s + 1u) & uint32_t(kHashCap - 1);
    }
    return false;
  }
#pragma unroll 1
  for (int h = 0; h < rp.hlen; ++h)
    if (rp.hist[h] == id) return true;
  return false;
}

// Geometry of global group g of a row.
struct GrpGeo {
  int s, lg, L, n;
  int64_t base;   // id of slice offset 0
};
__device__ __forceinline__ GrpGeo grp_geo(const Params& P, int64_t g) {
  GrpGeo q;
  q.s = slice_of_group(P, g);
  q.lg = int(g - P.gbase[q.s]);
  q.base = P.sstart[q.s];
  q.L = int(P.sstart[q.s + 1] - q.base);
  q.n = group_size(q.lg, q.L);
  return q;
}
template <typename T>
__device__ __forceinline__ float load_one(const Params& P, int row, int64_t j) {
  const size_t o = size_t(row) * size_t(P.a.ld) + size_t(j);
  if constexpr (sizeof(T) == 2) return Cvt<T>::one(__ldg(static_cast<const uint16_t*>(P.a.logits) + o));
  else return __ldg(static_cast<const float*>(P.a.logits) + o);
}

// Lane-parallel visit of selected groups.  The warps split the row's groups
// in runs of 32 (one per lane); want(g, summary, min word) selects, the
// selected groups queue up per warp, and every 32 of them are visited at
// once, one group per lane: vis(g, geo, min word, x) with the group's 32
// members in registers (penalised, -inf past the group).  With kMin the
// lanes also get their group's noise-minimum word (one Philox call per four
// groups).
template <typename T, bool kMin, typename Want, typename Vis>
__device__ __forceinline__ void lane_visit(const Params& P, RowSm& sm, const RowP& rp, int row, Want want, Vis vis) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const GroupSum* gs = P.summ + size_t(row) * size_t(P.G);
  const unsigned char* rsrc = static_cast<const unsigned char*>(P.a.logits) + size_t(row) * size_t(P.a.ld) * P.esize;
  int* qg = sm.wq[warp];
  uint32_t* qw = sm.wqw[warp];
  auto run = [&](int64_t g, uint32_t wm) {
    if (g < 0) return;
    const GrpGeo q = grp_geo(P, g);
    float x[32];
    load_members<T>(P, rsrc + size_t(q.base) * P.esize, q.lg >> 5, q.lg & 31, q.L, x);
    if (rp.pen) {
      const int bid = int(q.base) + (q.lg >> 5) * kTile + (q.lg & 31) * 8;
#pragma unroll
      for (int m = 0; m < 32; ++m)
        if (m < q.n && in_history(sm, rp, bid + (m >> 3) * 256 + (m & 7))) x[m] = pen_x(x[m], rp.rp);
    }
    vis(g, q, wm, x);
  };
  int qn = 0;   // warp-uniform queue length
#pragma unroll 1
  for (int64_t base = int64_t(warp) * 32; base < P.G; base += kRowThreads) {
    const int64_t g = base + lane;
    uint32_t wm = 0u;
    if constexpr (kMin) {
      U4 w{0u, 0u, 0u, 0u};
      if (lane < 8) w = philox_at(rp.key, uint32_t((base >> 2) + lane), kTagGroupMin);
      const int src = lane >> 2;
      const U4 v{__shfl_sync(0xFFFFFFFFu, w.x, src), __shfl_sync(0xFFFFFFFFu, w.y, src),
                 __shfl_sync(0xFFFFFFFFu, w.z, src), __shfl_sync(0xFFFFFFFFu, w.w, src)};
      wm = pick_word(v, uint32_t(lane & 3));
    }
    const bool sel = g < P.G && want(g, gs[g], wm);
    const unsigned mask = __ballot_sync(0xFFFFFFFFu, sel);
    if (sel) {
      const int pos = qn + __popc(mask & ((1u << lane) - 1u));
      qg[pos] = int(g);
      qw[pos] = wm;
    }
    qn += __popc(mask);
    __syncwarp();
    if (qn >= 32) {
      const int64_t gg = qg[lane];
      const uint32_t ww = qw[lane];
      __syncwarp();
      if (lane < qn - 32) {
        qg[lane] = qg[32 + lane];
        qw[lane] = qw[32 + lane];
      }
      qn -= 32;
      __syncwarp();
      run(gg, ww);
    }
  }
  if (qn > 0) {
    const int64_t gg = lane < qn ? int64_t(qg[lane]) : int64_t(-1);
    const uint32_t ww = lane < qn ? qw[lane] : 0u;
    __syncwarp();
    run(gg, ww);
  }
  __syncwarp();
}

// Id of member m of a group: base id (member 0) + block and element offsets.
__device__ __forceinline__ int group_base_id(const GrpGeo& q) {
  return int(q.base) + (q.lg >> 5) * kTile + (q.lg & 31) * 8;
}
__device__ __forceinline__ int member_id(int bid, int m) { return bid + (m >> 3) * 256 + (m & 7); }

// ---------------------------------------------------------------- race
// Kept-set predicate of the exact rounds: key(x) >> sh above kkey, or equal
// to it with id <= id_lim (all such ids when ties_all).
struct Keep {
  int on, sh;
  uint32_t kkey;
  int ties_all, id_lim;
  __device__ __forceinline__ bool operator()(float x, int id) const {
    if (!on) return true;
    const uint32_t k = ordered_key(x) >> sh;
    if (k != kkey) return k > kkey;
    return ties_all || id <= id_lim;
  }
  __device__ __forceinline__ uint32_t gkey_min() const { return on ? (kkey << sh) : 0u; }
};

// The race over the row: sm.top[0..ntop) gets the kTC best (rho desc, id
// asc) among the ids `keep` allows, exact for every id whose rho >= theta.
// A group is visited only if its bound (largest term over a lower bound of
// its noise minimum, taken with n = 32 members, which only lowers it)
// reaches theta and its max is not below the kept-set boundary.  In a
// visited group the noise-minimum and second-minimum members get their exact
// noise; every other member's ratio is bounded by RN(p/E2) (RN is monotone
// and E >= E2), and only those reaching theta and the lane's 4th best get
// their token noise.
template <typename T>
__device__ void race_row(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, float theta,
                         const Keep& keep) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* em = P.emin + size_t(row) * size_t(P.G);
  const uint32_t gk = keep.gkey_min();
  const float c1 = rp.c1;
  const bool cnoise = P.a.noise != nullptr;
  Top4 top;
  top.init();
  auto want = [&](int64_t g, const GroupSum& sg, uint32_t wm) -> bool {
    if (!(sg.gmax > -INFINITY) || ordered_key(sg.gmax) < gk) return false;
    float lo1;
    if (cnoise) {
      lo1 = __ldg(em + g);
    } else if (g == rp.s_gid) {
      lo1 = rp.e_root;
    } else {
      const float la = -lg2_approx(uniform_open(wm)) * 0.6931472f;
      lo1 = (rp.e_root + fmaxf(0.f, la * (1.f - 3e-5f) - 3e-5f) * 0.03125f) * (1.f - 2e-6f);
    }
    if (!(lo1 > 0.f)) return true;
    const float ub = __fdividef(__fdividef(qe_ex2_ftz(__fmaf_rn(sg.gmax, c1, c0)), Sf), lo1) * (1.f + 2e-5f);
    return ub >= theta;
  };
  auto vis = [&](int64_t g, const GrpGeo& q, uint32_t wm, const float (&x)[32]) {
    const int bid = group_base_id(q);
    const int n = q.n;
    if (cnoise) {
      const float* nz = P.a.noise + size_t(row) * size_t(P.a.noise_ld);
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const int id = member_id(bid, m);
        if (m >= n || !keep(x[m], id)) continue;
        const float p = __fdiv_rn(qe_ex2_ftz(__fmaf_rn(x[m], c1, c0)), Sf);
        const float E = __ldg(nz + id);
        top.add(__fdiv_rn(p, E), x[m], E, id);
      }
      return;
    }
    const bool holds = g == rp.s_gid;
    const U4 wd = philox_at(rp.key, uint32_t(g), kTagGroup);
    int a;
    float emin;
    if (holds) {
      a = rp.s_mem;
      emin = rp.e_root;
    } else {
      a = int(select_index32(wd.y, uint32_t(n)));
      const float l = neglog(uniform_open(wm));
      emin = __fadd_rn(rp.e_root, n == 32 ? __fmul_rn(l, 0.03125f) : __fdiv_rn(l, float(n)));
    }
    int a2 = -1;
    float e2 = INFINITY;
    if (n >= 2) {
      e2 = __fadd_rn(emin, __fdiv_rn(neglog(uniform_open(wd.z)), float(n - 1)));
      const int i2 = int(select_index32(wd.w, uint32_t(n - 1)));
      a2 = i2 < a ? i2 : i2 + 1;
    }
    // the noise-minimum and second members exactly; the others bounded by
    // RN(p/E2) first, their token noise only when that reaches theta
    uint32_t need = 0u;
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      const int id = member_id(bid, m);
      if (m >= n || !keep(x[m], id)) continue;
      const float p = __fdiv_rn(qe_ex2_ftz(__fmaf_rn(x[m], c1, c0)), Sf);
      if (m == a) top.add(__fdiv_rn(p, emin), x[m], emin, id);
      else if (m == a2) top.add(__fdiv_rn(p, e2), x[m], e2, id);
      else if (__fdiv_rn(p, e2) >= theta) need |= 1u << m;
    }
#pragma unroll 1
    while (need) {
      const int m = __ffs(need) - 1;
      need &= need - 1u;
      const int id = member_id(bid, m);
      float xv = load_one<T>(P, row, id);
      if (rp.pen && in_history(sm, rp, id)) xv = pen_x(xv, rp.rp);
      const float p = __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xv, c1, c0)), Sf);
      if (!rbetter(__fdiv_rn(p, e2), id, top.r[kTC - 1], top.id[kTC - 1])) continue;
      const float E = __fadd_rn(e2, neglog(uniform_open(pick_word(philox_at(rp.key, uint32_t(id >> 2), kTagToken),
                                                                   uint32_t(id & 3)))));
      top.add(__fdiv_rn(p, E), xv, E, id);
    }
  };
  if (cnoise) lane_visit<T, false>(P, sm, rp, row, want, vis);
  else lane_visit<T, true>(P, sm, rp, row, want, vis);
  // the warp's kTC best: pop the lanes' sorted lists
  int h = 0;
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    float r = -1.f, xx = 0.f, EE = 1.f;
    int id = INT_MAX;
#pragma unroll
    for (int k = 0; k < kTC; ++k)
      if (k == h) {
        r = top.r[k];
        xx = top.x[k];
        EE = top.E[k];
        id = top.id[k];
      }
    const uint32_t kr = r >= 0.f ? __float_as_uint(r) + 1u : 0u;
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
    const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(id) : 0xFFFFFFFFu);
    const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(id) == im)) - 1;
    const Cand c{__shfl_sync(0xFFFFFFFFu, r, src), __shfl_sync(0xFFFFFFFFu, xx, src),
                 __shfl_sync(0xFFFFFFFFu, EE, src), int(im)};
    if (lane == src && km != 0u) ++h;
    if (lane == 0) sm.wtop[warp][i] = km != 0u ? c : Cand{-1.f, 0.f, 1.f, INT_MAX};
  }
  __syncthreads();
  if (tid == 0) {
    Top4 t;
    t.init();
    for (int w = 0; w < kRowWarps; ++w)
#pragma unroll
      for (int i = 0; i < kTC; ++i) {
        const Cand c = sm.wtop[w][i];
        if (c.r >= 0.f) t.add(c.r, c.x, c.E, c.id);
      }
    int n = 0;
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      sm.top[i] = Cand{t.r[i], t.x[i], t.E[i], t.id[i]};
      if (t.r[i] >= 0.f) ++n;
    }
    sm.ntop = n;
  }
  __syncthreads();
}

// ---------------------------------------------------------------- outputs
__device__ __forceinline__ void write_row(const Params& P, int row, long long id, int status, long long kept) {
  if (threadIdx.x != 0) return;
  const KernelArgs& a = P.a;
  a.out_ids[row] = id;
  if (a.out_status) a.out_status[row] = status;
  if (a.out_kept) a.out_kept[row] = kept;
}

__device__ __forceinline__ unsigned long long efix(float x, float c1, float c0) {
  return __float2ull_rn(qe_ex2_ftz(__fmaf_rn(x, c1, c0)) * 1099511627776.0f);   // 2^40 fixed point
}

// ---------------------------------------------------------------- exact path
// Radix rounds over the element keys of the groups at or above the floor xf
// (ids below it are known to be outside the kept set), the tie rank at the
// boundary, then the race over the kept set.
template <typename T>
__device__ void exact_path(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, double S,
                           float thr_m, float xf) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int final_level = rp.pen ? 3 : P.dtype_level;
  const float c1 = rp.c1;
  if (thr_m > 0.f) xf = -INFINITY;   // the min-p count needs every id
  // thread 0's running state
  uint32_t prefix = 0u;
  long long acnt = 0, kk = rp.k;
  unsigned long long amass = 0ull, tfix = ~0ull;
  uint32_t kkey = 0u;
  int ties_all = 1, lvl = 0;
  long long kties = 0, nkeep = 0;
  unsigned long long mass_keep = 0ull;
  if (tid == 0) sm.bcast = 0;
#pragma unroll 1
  for (int L = 0; L < 4; ++L) {
    for (int i = tid; i < 256; i += kRowThreads) {
      sm.u.h.cnt[i] = 0u;
      sm.u.h.mass[i] = 0ull;
    }
    if (tid == 0) sm.u.h.nm = 0u;
    __syncthreads();
    const int shift = 24 - 8 * L;
    const uint32_t pre = uint32_t(sm.bcast);
    unsigned int nm = 0u;
    auto want = [&](int64_t, const GroupSum& sg, uint32_t) -> bool {
      if (!(sg.gmax > -INFINITY) || !(sg.gmax >= xf)) return false;
      return L == 0 || (ordered_key(sg.gmax) >> (32 - 8 * L)) >= pre;
    };
    auto vis = [&](int64_t, const GrpGeo& q, uint32_t, const float (&x)[32]) {
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const float v = x[m];
        if (m >= q.n || v < xf) continue;
        const uint32_t k = ordered_key(v);
        if (L > 0 && (k >> (32 - 8 * L)) != pre) continue;
        const int bin = int((k >> shift) & 255u);
        atomicAdd(&sm.u.h.cnt[bin], 1u);
        atomicAdd(&sm.u.h.mass[bin], efix(v, c1, c0));
        if (L == 0 && thr_m > 0.f && __fdiv_rn(qe_ex2_ftz(__fmaf_rn(v, c1, c0)), Sf) >= thr_m) ++nm;
      }
    };
    lane_visit<T, false>(P, sm, rp, row, want, vis);
    nm = __reduce_add_sync(0xFFFFFFFFu, nm);
    if (lane == 0 && nm) atomicAdd(&sm.u.h.nm, nm);
    __syncthreads();
    if (tid == 0) {
      int next = 0;
      if (L == 0) {
        unsigned long long sf = 0ull;
        if (xf > -INFINITY) {
          // ids below the floor were not binned: the row mass comes from S
          sf = static_cast<unsigned long long>(llrint(S * 1099511627776.0));
        } else {
          for (int b = 0; b < 256; ++b) sf += sm.u.h.mass[b];
        }
        tfix = rp.p_on ? static_cast<unsigned long long>(floor(double(rp.tp) * double(sf))) : ~0ull;
        kk = rp.k;
        if (rp.m_on) kk = min(kk, (long long)sm.u.h.nm);
      }
      int d = -1;
      for (int b = 255; b >= 0; --b) {
        const long long c = sm.u.h.cnt[b];
        const unsigned long long ms = sm.u.h.mass[b];
        if (acnt + c > kk || amass + ms > tfix) {
          d = b;
          break;
        }
        acnt += c;
        amass += ms;
      }
      if (d < 0) {   // every binned id is kept
        lvl = 3;
        kkey = xf > -INFINITY ? ordered_key(xf) : 0u;
        ties_all = 1;
        kties = 0;
        nkeep = acnt;
        mass_keep = amass;
      } else {
        const uint32_t key_hi = L == 0 ? uint32_t(d) : ((prefix << 8) | uint32_t(d));
        if (L < final_level) {
          prefix = key_hi;
          next = 1;
        } else {
          // key_hi fixes the value: its ids are ties of equal mass
          const int sh = 24 - 8 * L;
          const uint32_t hi = key_hi << sh;
          const uint32_t fullk = hi | ((hi & 0x80000000u) ? 0u : ((1u << sh) - 1u));
          const unsigned long long ed = efix(key_to_float(fullk), c1, c0);
          long long t = min((long long)sm.u.h.cnt[d], kk - acnt);
          if (rp.p_on && ed > 0ull) {
            const unsigned long long qq = (tfix - amass) / ed + 1ull;
            if (qq < static_cast<unsigned long long>(t)) t = (long long)qq;
          }
          if (t < 0) t = 0;
          lvl = L;
          kkey = key_hi;
          kties = t;
          ties_all = t == (long long)sm.u.h.cnt[d];
          nkeep = acnt + t;
          mass_keep = amass + (unsigned long long)t * ed;
        }
      }
      sm.n = next;
      sm.bcast = (long long)prefix;
    }
    __syncthreads();
    const int next = sm.n;
    __syncthreads();
    if (!next) break;
  }
  // broadcast the boundary
  if (tid == 0) {
    sm.u.h.cnt[0] = uint32_t(lvl);
    sm.u.h.cnt[1] = kkey;
    sm.u.h.cnt[2] = uint32_t(ties_all);
    sm.u.h.mass[1] = (unsigned long long)kties;
    sm.u.h.mass[2] = (unsigned long long)nkeep;
    sm.u.h.mass[3] = mass_keep;
  }
  __syncthreads();
  lvl = int(sm.u.h.cnt[0]);
  kkey = sm.u.h.cnt[1];
  ties_all = int(sm.u.h.cnt[2]);
  kties = (long long)sm.u.h.mass[1];
  nkeep = (long long)sm.u.h.mass[2];
  mass_keep = sm.u.h.mass[3];
  __syncthreads();
  Keep keep{1, 24 - 8 * lvl, kkey, ties_all, INT_MAX};
  if (!ties_all) {
    keep.id_lim = -1;
    if (kties > 0) {
      // the kties-th smallest id among the boundary ties: radix over ids
      uint32_t ipre = 0u;
      long long need = kties;
      const int ksh = keep.sh;
#pragma unroll 1
      for (int il = 0; il < 3; ++il) {
        const int ish = 16 - 8 * il;
        for (int i = tid; i < 256; i += kRowThreads) sm.u.h.cnt[i] = 0u;
        __syncthreads();
        auto want = [&](int64_t, const GroupSum& sg, uint32_t) -> bool {
          return sg.gmax > -INFINITY && (ordered_key(sg.gmax) >> ksh) >= kkey;
        };
        auto vis = [&](int64_t, const GrpGeo& q, uint32_t, const float (&x)[32]) {
          const int bid = group_base_id(q);
#pragma unroll
          for (int m = 0; m < 32; ++m) {
            if (m >= q.n || (ordered_key(x[m]) >> ksh) != kkey) continue;
            const uint32_t u = uint32_t(member_id(bid, m));
            if (il > 0 && (u >> (ish + 8)) != ipre) continue;
            atomicAdd(&sm.u.h.cnt[(u >> ish) & 255u], 1u);
          }
        };
        lane_visit<T, false>(P, sm, rp, row, want, vis);
        __syncthreads();
        if (tid == 0) {
          long long run = 0;
          int d = 255;
          for (int b = 0; b < 256; ++b) {
            const long long c = sm.u.h.cnt[b];
            if (run + c >= need) {
              d = b;
              break;
            }
            run += c;
          }
          sm.bcast = ((long long)d << 40) | (need - run);
        }
        __syncthreads();
        const long long bb = sm.bcast;
        const uint32_t d = uint32_t(bb >> 40);
        need = bb & ((1ll << 40) - 1);
        ipre = il == 0 ? d : ((ipre << 8) | d);
        __syncthreads();
      }
      keep.id_lim = int(ipre);
    }
  }
  // the race over the kept set; its best is below 1/16 of its mass with
  // probability e^-16, and then everything it keeps is raced exactly
  const double mk = double(mass_keep) * (1.0 / 1099511627776.0);
  const float theta = float(mk / S / 16.0);
  race_row<T>(P, sm, rp, row, c0, Sf, theta, keep);
  if (!(sm.ntop > 0 && sm.top[0].r >= theta)) race_row<T>(P, sm, rp, row, c0, Sf, 0.f, keep);
  if (sm.ntop == 0 && tid == 0) atomicOr(&P.ctl->err, 4u);
  write_row(P, row, sm.ntop > 0 ? sm.top[0].id : -1, QE_ROW_SLOW, nkeep);
}

// ---------------------------------------------------------------- direct top-k (k <= kSmallK)
// k-th largest (1-based) high word of keys[0..n), radix over shared memory.
__device__ uint32_t radix_kth_keys(RowSm& sm, const unsigned long long* keys, int n, int k) {
  uint32_t prefix = 0u;
  int need = k;
#pragma unroll 1
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int i = threadIdx.x; i < 256; i += kRowThreads) sm.scnt[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kRowThreads) {
      const uint32_t v = uint32_t(keys[i] >> 32);
      if (level == 0 || (v >> (shift + 8)) == prefix) atomicAdd(&sm.scnt[(v >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0, d = 0;
      for (int b = 255; b >= 0; --b) {
        const int c = int(sm.scnt[b]);
        if (run + c >= need) {
          d = b;
          break;
        }
        run += c;
      }
      sm.bcast = ((long long)d << 32) | (long long)(need - run);
    }
    __syncthreads();
    const long long bb = sm.bcast;
    const uint32_t d = uint32_t(bb >> 32);
    need = int(bb & 0xFFFFFFFFll);
    prefix = level == 0 ? d : ((prefix << 8) | d);
    __syncthreads();
  }
  return prefix;
}

// The k-th largest group max key of the row.
__device__ uint32_t kth_group_key(const Params& P, RowSm& sm, int row, int k) {
  const GroupSum* gs = P.summ + size_t(row) * size_t(P.G);
  uint32_t prefix = 0u;
  int need = k;
#pragma unroll 1
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int i = threadIdx.x; i < 256; i += kRowThreads) sm.scnt[i] = 0u;
    __syncthreads();
    for (int64_t g = threadIdx.x; g < P.G; g += kRowThreads) {
      const uint32_t v = ordered_key(gs[g].gmax);
      if (level == 0 || (v >> (shift + 8)) == prefix) atomicAdd(&sm.scnt[(v >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0, d = 0;
      for (int b = 255; b >= 0; --b) {
        const int c = int(sm.scnt[b]);
        if (run + c >= need) {
          d = b;
          break;
        }
        run += c;
      }
      sm.bcast = ((long long)d << 32) | (long long)(need - run);
    }
    __syncthreads();
    const long long bb = sm.bcast;
    const uint32_t d = uint32_t(bb >> 32);
    need = int(bb & 0xFFFFFFFFll);
    prefix = level == 0 ? d : ((prefix << 8) | d);
    __syncthreads();
  }
  return prefix;
}

// Top-k rows with k <= kSmallK: every id of the top k lies in a group whose
// max is at or above the k-th largest group max, so only those groups are
// read.  The k largest are sorted, top-p and min-p applied in that order
// (reference rule), and the kept ones raced with exact noise.  Returns false
// when a capacity ran out (the caller takes the exact path).
template <typename T>
__device__ bool small_k(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, float thr_m) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = int(rp.k);
  const uint32_t tk = kth_group_key(P, sm, row, k);
  if (tid == 0) sm.n = 0;
  __syncthreads();
  {
    auto want = [&](int64_t, const GroupSum& sg, uint32_t) -> bool { return ordered_key(sg.gmax) >= tk; };
    auto vis = [&](int64_t, const GrpGeo& q, uint32_t, const float (&x)[32]) {
      const int bid = group_base_id(q);
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        const uint32_t key = ordered_key(x[m]);
        if (m >= q.n || key < tk) continue;
        const int at = atomicAdd(&sm.n, 1);
        if (at < kSelCap)
          sm.u.keys[at] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFull - uint32_t(member_id(bid, m)));
      }
    };
    lane_visit<T, false>(P, sm, rp, row, want, vis);
  }
  __syncthreads();
  const int n1 = sm.n;
  __syncthreads();
  if (n1 > kSelCap || n1 < k) return false;
  const uint32_t tk2 = radix_kth_keys(sm, sm.u.keys, n1, k);
  if (tid == 0) sm.n = 0;
  __syncthreads();
  for (int i = tid; i < n1; i += kRowThreads) {
    const unsigned long long key = sm.u.keys[i];
    if (uint32_t(key >> 32) < tk2) continue;
    const int at = atomicAdd(&sm.n, 1);
    if (at < kSortCap) sm.sortk[at] = key;
  }
  __syncthreads();
  const int n = sm.n;
  __syncthreads();
  if (n > kSortCap || n < 1) return false;
  int N = 2;
  while (N < n) N <<= 1;
  for (int i = n + tid; i < N; i += kRowThreads) sm.sortk[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending: x desc, then id asc
  for (int kk = 2; kk <= N; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < N; i += kRowThreads) {
        const int p = i ^ j;
        if (p > i) {
          const unsigned long long a = sm.sortk[i], b = sm.sortk[p];
          const bool desc = (i & kk) == 0;
          if (desc ? a < b : a > b) {
            sm.sortk[i] = b;
            sm.sortk[p] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const int nk = k < n ? k : n;
  const unsigned long long mykey = tid < nk ? sm.sortk[tid] : 0ull;
  const float xi = key_to_float(uint32_t(mykey >> 32));
  const int idi = int(0xFFFFFFFFu - uint32_t(mykey & 0xFFFFFFFFull));
  const float pi = tid < nk ? __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xi, rp.c1, c0)), Sf) : 0.f;
  if (tid < nk) sm.u.sk.p[tid] = pi;
  __syncthreads();
  if (tid == 0) {
    // top-p in sorted order: fp64 cumulative sum rounded to fp32 (as CPU
    // torch.cumsum of fp32), drop where RN(cs - p) > top_p; min-p elementwise
    double cum = 0.0;
    int kept = 0;
    for (int i = 0; i < nk; ++i) {
      const float p = sm.u.sk.p[i];
      cum += double(p);
      const float cs = float(cum);
      bool rem = rp.p_on && __fsub_rn(cs, p) > rp.tp;
      rem = rem || (rp.m_on && p < thr_m);
      sm.u.sk.keep[i] = rem ? 0 : 1;
      kept += rem ? 0 : 1;
    }
    sm.n = kept;
  }
  __syncthreads();
  float rho = -1.f;
  int rid = INT_MAX;
  if (tid < nk && sm.u.sk.keep[tid] && idi >= 0 && int64_t(idi) < P.a.vocab) {
    float E;
    if (P.a.noise) {
      E = __ldg(P.a.noise + size_t(row) * size_t(P.a.noise_ld) + size_t(idi));
    } else {
      const NoiseRoot rt{rp.e_root, 0};
      E = tree_noise(rp.key, rt, rp.s_gid, rp.s_mem, idi, P.a.vocab);
    }
    rho = __fdiv_rn(pi, E);
    rid = idi;
  }
  const long long kept = sm.n;
  const uint32_t kr = rho >= 0.f ? __float_as_uint(rho) + 1u : 0u;
  const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
  const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(rid) : 0xFFFFFFFFu);
  if (lane == 0) {
    sm.red_u[warp] = km;
    sm.red_i[warp] = int(im);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t bk = 0u;
    int bid = -1;
    for (int w = 0; w < kRowWarps; ++w) {
      const uint32_t kx = sm.red_u[w];
      const int i = sm.red_i[w];
      if (kx > bk || (kx == bk && kx != 0u && i < bid)) {
        bk = kx;
        bid = i;
      }
    }
    if (!bk) atomicOr(&P.ctl->err, 4u);
    write_row(P, row, bk ? bid : -1, QE_ROW_GATHERED, kept);
  }
  return true;
}

// ---------------------------------------------------------------- the row kernel
template <typename T>
__global__ void __launch_bounds__(kRowThreads) row_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowSm& sm = *reinterpret_cast<RowSm*>(smem_raw);
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int64_t V = P.a.vocab;
  if (row == 0 && tid == 0) P.ctl->err = 0u;
  if (tid == 0) {
    RowP r = row_params(P, row);
    if (!P.a.noise && r.kind != kKindGreedy && r.kind != kKindArgmax) {
      const NoiseRoot rt = noise_root(r.key, V);
      int64_t gsd = -1;
      int rm = 0;
      token_group_p(P, rt.s, &gsd, &rm);
      r.e_root = rt.e_root;
      r.s_gid = gsd;
      r.s_mem = rm;
    }
    sm.rp = r;
  }
  __syncthreads();
  const RowP rp = sm.rp;
  const GroupSum* gs = P.summ + size_t(row) * size_t(P.G);
  const bool idx_mode = rp.kind == kKindGreedy || rp.kind == kKindArgmax;
  // one pass: row max (NaN-aware) and, in each thread's own running scale,
  // the sum of the group terms
  uint32_t kmax = 0u;
  float mt = -INFINITY;
  double st = 0.0;
  const int64_t nq = (P.G + 3) / 4;
#pragma unroll 2
  for (int64_t qd = tid; qd < nq; qd += kRowThreads) {
    GroupSum sg[4];
    if (qd * 4 + 4 <= P.G) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(gs + qd * 4));
      const float4 b = __ldg(reinterpret_cast<const float4*>(gs + qd * 4 + 2));
      sg[0] = GroupSum{a.x, a.y};
      sg[1] = GroupSum{a.z, a.w};
      sg[2] = GroupSum{b.x, b.y};
      sg[3] = GroupSum{b.z, b.w};
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) sg[j] = qd * 4 + j < P.G ? gs[qd * 4 + j] : GroupSum{-INFINITY, 0.f};
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kmax = max(kmax, nan_key(sg[j].gmax));
      if (!idx_mode && sg[j].gmax > -INFINITY) {
        const float ug = __fmul_rn(sg[j].gmax, rp.c1);
        if (ug > mt) {
          st = st * double(qe_ex2_ftz(__fsub_rn(mt, ug))) + double(sg[j].aux);
          mt = ug;
        } else {
          st += double(sg[j].aux * qe_ex2_ftz(__fsub_rn(ug, mt)));
        }
      }
    }
  }
  kmax = block_max_u(sm, kmax);
  const float xmax = kmax == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : key_to_float(kmax);
  const float u = __fmul_rn(xmax, rp.c1);
  bool fin = finite_f(xmax) && finite_f(u);
  double S = 0.0;
  if (!idx_mode && fin) {
    S = block_sum_d(sm, mt > -INFINITY && finite_f(mt) ? st * double(qe_ex2_ftz(__fsub_rn(mt, u))) : 0.0);
    if (!(S > 0.0) || !(float(S) < INFINITY)) fin = false;
  }
  if (tid == 0 && P.a.out_norm)
    P.a.out_norm[row] = (!idx_mode && fin) ? S * exp2(double(u) - double(xmax) * double(rp.c1))
                                           : __longlong_as_double(0x7FF8000000000000LL);
  if (idx_mode || !fin) {
    // the first id holding the max (torch.argmax: NaN maximal, first index)
    uint32_t first = 0xFFFFFFFFu;
    if (xmax > -INFINITY || xmax != xmax) {
      const bool xn = xmax != xmax;
      for (int64_t g = tid; g < P.G; g += kRowThreads) {
        const GroupSum sg = gs[g];
        if (!(xn ? sg.gmax != sg.gmax : sg.gmax == xmax)) continue;
        const GrpGeo q = grp_geo(P, g);
        first = min(first, uint32_t(q.base + member_offset(q.lg, __float_as_int(sg.aux))));
      }
      first = block_min_u(sm, first);
    } else {
      first = 0u;   // every logit is -inf: torch.argmax returns 0
    }
    const int status = rp.kind == kKindGreedy ? QE_ROW_GREEDY : (!fin ? QE_ROW_NONFINITE : 0);
    write_row(P, row, first, status, rp.kind == kKindArgmax && fin ? 1 : 0);
    return;
  }
  if (rp.pen) hash_build(sm, rp, V);
  const float c0 = -u;
  const float Sf = float(S);
  const float thr_m = rp.m_on ? __fmul_rn(rp.minp, __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xmax, rp.c1, c0)), Sf)) : 0.f;
  if (rp.kind == kKindSmallK) {
    if (small_k<T>(P, sm, rp, row, c0, Sf, thr_m)) return;
    exact_path<T>(P, sm, rp, row, c0, Sf, S, thr_m, -INFINITY);
    return;
  }
  if (rp.exact) {
    exact_path<T>(P, sm, rp, row, c0, Sf, S, thr_m, -INFINITY);
    return;
  }
  const Keep all{0, 0, 0u, 1, INT_MAX};
  // first race: complete above 1/4 (the best ratio of a race is below that
  // with probability e^-4); enough when its best is in the kept set
  float theta = 0.25f;
  race_row<T>(P, sm, rp, row, c0, Sf, theta, all);
  if (!rp.filtered) {
    if (!(sm.ntop > 0 && sm.top[0].r >= theta)) race_row<T>(P, sm, rp, row, c0, Sf, 0.f, all);
    if (sm.ntop == 0 && tid == 0) atomicOr(&P.ctl->err, 4u);
    write_row(P, row, sm.ntop > 0 ? sm.top[0].id : -1, 0, V);
    return;
  }
  // kept-set test of the complete candidates, in race order; a second race
  // (complete above 1/64) when the first did not settle the row
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      theta = 1.f / 64.f;
      race_row<T>(P, sm, rp, row, c0, Sf, theta, all);
    }
    const int ntop = sm.ntop;
#pragma unroll 1
    for (int i = 0; i < kTC; ++i) {
      if (i >= ntop) break;
      const Cand c = sm.top[i];
      if (!(c.r >= theta)) break;
      const float e = qe_ex2_ftz(__fmaf_rn(c.x, rp.c1, c0));
      if (rp.m_on && __fdiv_rn(e, Sf) < thr_m) continue;
      // bound from the summaries: every id ahead lies in a group whose max
      // is at or above the candidate
      double ub = 0.0;
      long long nb = 0;
      for (int64_t g = tid; g < P.G; g += kRowThreads) {
        const GroupSum sg = gs[g];
        if (!(sg.gmax >= c.x)) continue;
        ub += double(sg.aux * qe_ex2_ftz(__fsub_rn(__fmul_rn(sg.gmax, rp.c1), u)));
        nb += 32;
      }
      ub = block_sum_d(sm, ub);
      nb = block_sum_l(sm, nb);
      bool in_k = (!rp.k_on || nb - 1 < rp.k) && (!rp.p_on || ub * (1.0 + 1e-5) - double(e) <= double(rp.tp) * S);
      if (!in_k) {
        // exact count and mass ahead over those groups
        double ms = 0.0;
        long long ct = 0;
        auto want = [&](int64_t, const GroupSum& sg, uint32_t) -> bool { return sg.gmax >= c.x; };
        auto vis = [&](int64_t, const GrpGeo& q, uint32_t, const float (&x)[32]) {
          const int bid = group_base_id(q);
          float part = 0.f;
#pragma unroll
          for (int m = 0; m < 32; ++m) {
            const float v = x[m];
            if (m < q.n && (v > c.x || (v == c.x && member_id(bid, m) < c.id))) {
              part += qe_ex2_ftz(__fmaf_rn(v, rp.c1, c0));
              ct += 1;
            }
          }
          ms += double(part);
        };
        lane_visit<T, false>(P, sm, rp, row, want, vis);
        ms = block_sum_d(sm, ms);
        ct = block_sum_l(sm, ct);
        in_k = (!rp.k_on || ct < rp.k) && (!rp.p_on || ms <= double(rp.tp) * S);
        if (!in_k) {
          // every id after it in the order is outside as well: a floor
          if (pass == 1 || i + 1 < ntop) continue;
        }
      }
      if (in_k) {
        write_row(P, row, c.id, 0, 0);
        return;
      }
    }
  }
  exact_path<T>(P, sm, rp, row, c0, Sf, S, thr_m, -INFINITY);
}

// ---------------------------------------------------------------- host
struct DevInfo {
  bool ready = false;
  int sms = 0;
};
std::mutex g_mu;
DevInfo g_dev[64];

template <typename T>
cudaError_t prepare() {
  return cudaFuncSetAttribute(row_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(RowSm)));
}

// Kernel attributes, set once per device (they are per-device state).
int device_setup(int* sms) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QE_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  DevInfo& d = g_dev[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = prepare<float>();
    if (e == cudaSuccess) e = prepare<__nv_bfloat16>();
    if (e == cudaSuccess) e = prepare<__half>();
    if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("stream sampler setup: ") + cudaGetErrorString(e));
    d.ready = true;
  }
  *sms = d.sms;
  return QE_OK;
}

}  // namespace st

bool stream_supports(int64_t vocab) { return vocab >= 1 && vocab < (int64_t(1) << 24); }

size_t stream_workspace_bytes(int64_t batch, int64_t vocab) { return st::make_layout(batch, vocab).total; }

const void* stream_error_word(const void* workspace) {
  return static_cast<const char*>(workspace) + offsetof(st::Ctl, err);
}

int launch_stream(const KernelArgs& ka, cudaStream_t stream) {
  using namespace st;
  const int esize = ka.dtype == QE_DTYPE_F32 ? 4 : 2;
  const Layout L = make_layout(ka.batch, ka.vocab);
  if (ka.batch >= (int64_t(1) << 31)) return set_error(QE_ERR_UNSUPPORTED, "batch too large");
  int sms = 0;
  const int rc = device_setup(&sms);
  if (rc != QE_OK) return rc;
  Params P;
  std::memset(&P, 0, sizeof(P));
  P.a = ka;
  P.esize = esize;
  const uintptr_t lp = reinterpret_cast<uintptr_t>(ka.logits);
  P.vec_ok = (lp % 16 == 0) && ((ka.ld * esize) % 16 == 0);
  const uintptr_t np = reinterpret_cast<uintptr_t>(ka.noise);
  P.noise_vec = ka.noise && (np % 16 == 0) && ((ka.noise_ld * 4) % 16 == 0);
  P.tpw = esize == 4 ? 1 : 2;
  P.force_exact = ka.out_kept != nullptr;
  P.dtype_level = ka.dtype == QE_DTYPE_BF16 ? 1 : ka.dtype == QE_DTYPE_F16 ? 2 : 3;
  P.G = L.G;
  int64_t gb = 0;
  int tb = 0;
  for (int s = 0; s < kNumSlices; ++s) {
    const int64_t a0 = slice_start(s, ka.vocab), a1 = slice_start(s + 1, ka.vocab);
    P.sstart[s] = a0;
    P.gbase[s] = gb;
    P.snt[s] = int((a1 - a0 + kTile - 1) / kTile);
    P.tbase[s] = tb;
    gb += int64_t(P.snt[s]) * 32;
    tb += (P.snt[s] + P.tpw - 1) / P.tpw;
  }
  P.sstart[kNumSlices] = ka.vocab;
  P.gbase[kNumSlices] = gb;
  P.tbase[kNumSlices] = tb;
  P.tasks_row = tb;
  char* base = static_cast<char*>(ka.workspace);
  P.ctl = reinterpret_cast<Ctl*>(base);
  P.summ = reinterpret_cast<GroupSum*>(base + L.summ);
  P.emin = reinterpret_cast<float*>(base + L.emin);
  // summary kernel: one warp per task; narrower CTAs when there are few
  // tasks, so that they spread over the SMs
  const long long tasks = (long long)ka.batch * tb;
  int wpc = kSumThreads / 32;
  while (wpc > 1 && tasks < (long long)wpc * sms * 2) wpc >>= 1;
  const unsigned g1 = unsigned((tasks + wpc - 1) / wpc);
  const unsigned g2 = unsigned(ka.batch);
  switch (ka.dtype) {
    case QE_DTYPE_F32:
      summ_kernel<float><<<g1, wpc * 32, 0, stream>>>(P);
      row_kernel<float><<<g2, kRowThreads, sizeof(RowSm), stream>>>(P);
      break;
    case QE_DTYPE_BF16:
      summ_kernel<__nv_bfloat16><<<g1, wpc * 32, 0, stream>>>(P);
      row_kernel<__nv_bfloat16><<<g2, kRowThreads, sizeof(RowSm), stream>>>(P);
      break;
    default:
      summ_kernel<__half><<<g1, wpc * 32, 0, stream>>>(P);
      row_kernel<__half><<<g2, kRowThreads, sizeof(RowSm), stream>>>(P);
      break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("stream sampler launch: ") + cudaGetErrorString(e));
  return QE_OK;
}

}  // namespace qe
