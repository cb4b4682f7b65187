// qe_sample_stream.cu — the default sampler path: the logits read from HBM
// once, six launches on the caller's stream.
//
// Replaces BatchSampler.forward (src/compute/sampler.py:25-41) and the
// extensions of this library (top-k, min-p, repetition penalty, Philox
// noise).  The semantics of a sample are those of qe_sample_ref.cu and the
// CPU oracle: softmax of the penalised logits / T, kept set = the longest
// prefix of the order (x desc, id asc) allowed by top-k, top-p and min-p,
// token = argmax over the kept set of rho = RN(RN(e/S)/E).
//
// 1. scan_kernel streams the logits: one warp per task of `tpw` tiles (8 KB
//    of bf16 logits), copied into shared memory with cp.async before any
//    arithmetic; each lane reduces one 32-id group at a time to a GroupSum
//    (max, group-relative exponential sum, packed bf16x2 / f32x2 math) and
//    its noise bound key; per task a TaskRec: max, sum in the task's scale,
//    the two largest group bound keys with a ceiling for the rest (one Philox
//    call per four groups).  No barriers.
// 2. decide_kernel, one CTA per row, from the task records (still in L2):
//      * row max, softmax normaliser S, greedy / top-1 / non-finite rows;
//      * the exponential race over the groups whose bound reaches 1/4 (the
//        best ratio of a race is below that with probability e^-4), then
//        1/16: one group per thread, re-read and raced exactly;
//      * the kept-set test of the 4 best candidates from the task records,
//        then from the group records; a candidate outside the kept set
//        restricts the next race to the ids ahead of it.
// 3. count_kernel counts exactly, over all SMs, the ids ahead of the
//    candidates of the rows the records could not settle; the warp that
//    completes a row decides it (an atomic counter, no waiting).
// 4. retry_kernel races again, restricted, the rows whose counted candidates
//    were all outside the kept set; 5. count_kernel counts those.
// 6. finish_kernel (persistent CTAs) takes the rest: top-k rows with
//    k <= 64 (the k largest, sorted), rows whose kept-set size is asked for,
//    and the exact fallback (radix rounds over the keys, the tie rank, the
//    race over the kept set).
// Launches 2-6 use programmatic stream serialization (wait_prior_grid).
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
using fz::smem_u32;

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
  int tpw;                      // tiles per scan task
  int tasks_row;                // scan tasks per row
  int force_exact;              // the kept-set size is asked for
  int dtype_level;              // last radix level that separates the dtype's values
  int64_t G;                    // groups per row
  int64_t sstart[kNumSlices + 1];
  int64_t gbase[kNumSlices + 1];
  int snt[kNumSlices];          // tiles per slice
  int tbase[kNumSlices + 1];    // first scan task of each slice
  Ctl* ctl;
  GroupSum* summ;               // [B][G]
  TaskRec* trec;                // [B][tasks_row]
  float* emin;                  // [B][G] per group: noise minimum (caller-noise mode) or bound key (Philox mode)
  RowState* rstate;             // [B]
  int* plist;                   // [2][B] rows queued for the count kernel (per round)
  int* rlist;                   // rows queued for the retry round
  int* flist;                   // rows queued for the finish kernel (row | kind << 28)
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

// Packed fp32 pairs (Blackwell f32x2 FMA / add: two IEEE operations each, so
// the results are those of the scalar group_sum).
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// group_sum on 32 packed 16-bit values (word i holds members 2i and 2i+1),
// in its order: chains (s0, s1) and (s2, s3) as f32x2 pairs.
template <typename T>
__device__ __forceinline__ float group_sum_packed(const uint32_t w[16], float c1, float c0) {
  const unsigned long long cc1 = pk2(c1, c1), cc0 = pk2(c0, c0);
  unsigned long long s01 = 0ull, s23 = 0ull;   // (s0, s1), (s2, s3): +0.0f pairs
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    float a, b;
    upk2(fma2(pk2(Cvt<T>::lo(w[i]), Cvt<T>::hi(w[i])), cc1, cc0), a, b);
    s01 = add2(s01, pk2(qe_ex2_ftz(a), qe_ex2_ftz(b)));
    upk2(fma2(pk2(Cvt<T>::lo(w[i + 1]), Cvt<T>::hi(w[i + 1])), cc1, cc0), a, b);
    s23 = add2(s23, pk2(qe_ex2_ftz(a), qe_ex2_ftz(b)));
  }
  float s0, s1, s2, s3;
  upk2(s01, s0, s1);
  upk2(s23, s2, s3);
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


// ---------------------------------------------------------------- 1. scan
// Penalty bits of up to two tiles of a slice: bit (b*8+i) of word tt*32+l
// is set when slice offset (tile0+tt)*1024 + b*256 + l*8 + i is in the
// history.  Warp-local; the caller's warp runs it together.
__device__ __forceinline__ void pen_bits_build(uint32_t* bits, const int32_t* hist, int hl, int64_t sa, int tile0,
                                               int nt, int L) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  bits[lane] = 0u;
  bits[lane + 32] = 0u;
  __syncwarp();
  const int64_t base = int64_t(tile0) * kTile;
  for (int h = lane; h < hl; h += 32) {
    const int64_t o = int64_t(hist[h]) - sa - base;
    if (o >= 0 && o < int64_t(nt) * kTile && base + o < L)
      atomicOr(&bits[(o >> 10) * 32 + ((o >> 3) & 31)], 1u << int(((o >> 8) & 3) * 8 + (o & 7)));
  }
  __syncwarp();
}

// Lower bound of a group's noise minimum in Philox mode without the tree's
// root: E_min = E_root + (-ln u)/n >= (-ln u)/32.  The approximate log is
// pulled down by more than its error, so the bound holds; the group holding
// the root token is added to every race by the decide kernel instead.
__device__ __forceinline__ float emin_lower(uint32_t wmin) {
  const float la = -lg2_approx(uniform_open(wmin)) * 0.6931472f;
  return fmaxf(0.f, la * (1.f - 3e-5f) - 3e-5f) * 0.03125f * (1.f - 2e-6f);
}

// A lane's three largest bound keys (group ids kept for the first two).
struct Top3 {
  float b0, b1, b2;
  int g0, g1;
  __device__ __forceinline__ void init() {
    b0 = b1 = b2 = -INFINITY;
    g0 = g1 = -1;
  }
  __device__ __forceinline__ void add(float k, int g) {
    if (!(k > b2)) return;
    if (k > b1) {
      b2 = b1;
      if (k > b0) {
        b1 = b0; g1 = g0;
        b0 = k; g0 = g;
      } else {
        b1 = k; g1 = g;
      }
    } else {
      b2 = k;
    }
  }
};

// Programmatic dependent launch: the kernels after the scan are launched with
// programmatic stream serialization, so they start during their
// predecessor's tail; each waits here (a hardware dependency on the
// predecessor grid's completion and memory flush, not a spin) before it
// reads the predecessor's output.  Without such a launch it returns at once.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// cp.async (16 bytes, L2 only) and its group waits.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kScanRounds = 2;   // rounds of two tiles per task whose copies are issued up front (tpw <= 4)
constexpr size_t kScanSmem = size_t(kSumThreads / 32) * kScanRounds * 2 * 4 * 32 * sizeof(uint4);

// Scan task t of `row` by one warp: GroupSums of its groups, its TaskRec.
template <typename T>
__device__ __forceinline__ void scan_task(const Params& P, int row, int t, uint4* sbuf, uint32_t (*pen_bits)[64]) {
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  int s = 0;
#pragma unroll
  for (int step = 8; step > 0; step >>= 1)
    if (s + step < kNumSlices && P.tbase[s + step] <= t) s += step;
  const int tile0 = (t - P.tbase[s]) * P.tpw;
  const int ntile = min(P.tpw, P.snt[s] - tile0);
  const int64_t sa = P.sstart[s];
  const int L = int(P.sstart[s + 1] - sa);
  const KernelArgs& a = P.a;
  const unsigned char* src = static_cast<const unsigned char*>(a.logits) + (size_t(row) * size_t(a.ld) + size_t(sa)) * P.esize;
  // 16-bit rows: every full tile of the task on its way into shared memory
  // before any arithmetic (one commit group per round of two tiles)
  constexpr bool k16 = sizeof(T) == 2;
  const bool cp_ok = k16 && P.vec_ok && P.tpw <= 2 * kScanRounds;
  uint4* wb = sbuf + size_t(wib) * (kScanRounds * 2 * 4 * 32);
  if (cp_ok) {
#pragma unroll
    for (int r = 0; r < kScanRounds; ++r) {
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const int tl = 2 * r + tt;
        const int tile = tile0 + tl;
        if (tl < ntile && tile * kTile + kTile <= L) {
#pragma unroll
          for (int b = 0; b < 4; ++b)
            cp_async16(wb + ((r * 2 + tt) * 4 + b) * 32 + lane, src + size_t(tile * kTile + b * 256 + lane * 8) * 2);
        }
      }
      cp_async_commit();
    }
  }
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
  const int32_t* hist = pen ? a.history + row * a.history_ld : nullptr;
  const NoiseKey key = make_noise_key(row_seed(a, row), a.step_ptr ? *a.step_ptr : a.step, a.row_offset + row);
  const int64_t g_first = P.gbase[s] + int64_t(tile0) * 32;   // global id of the task's first group
  GroupSum* out = P.summ + size_t(row) * size_t(P.G) + size_t(g_first);
  const float* nzrow = a.noise ? a.noise + size_t(row) * size_t(a.noise_ld) + size_t(sa) : nullptr;
  // per-lane task state: NaN-aware max, sum in the lane's running scale, bound keys
  float lmax = -INFINITY, lu = -INFINITY, lsum = 0.f;
  Top3 top;
  top.init();
  constexpr int kStep = k16 ? 2 : 1;   // tiles per round
#pragma unroll 1
  for (int tp = 0, r = 0; tp < ntile; tp += kStep, ++r) {
    const int nt = min(kStep, ntile - tp);
    const int tbase = tile0 + tp;
    if (cp_ok) {
      if (r == 0) cp_async_wait<kScanRounds - 1>();
      else cp_async_wait<0>();
    }
    if (pen) pen_bits_build(pen_bits[wib], hist, hl, sa, tbase, nt, L);
    // group-minimum noise words of the round's groups (one Philox call per four)
    uint32_t wmin[2] = {0u, 0u};
    if (!idx_mode && !a.noise) {
      U4 w{0u, 0u, 0u, 0u};
      const int64_t gq = (g_first + int64_t(tp) * 32) >> 2;   // the round's groups start at a multiple of 32
      if (lane < nt * 8) w = philox_at(key, uint32_t(gq + lane), kTagGroupMin);
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const int srcl = tt * 8 + (lane >> 2);
        const U4 v{__shfl_sync(0xFFFFFFFFu, w.x, srcl), __shfl_sync(0xFFFFFFFFu, w.y, srcl),
                   __shfl_sync(0xFFFFFFFFu, w.z, srcl), __shfl_sync(0xFFFFFFFFu, w.w, srcl)};
        wmin[tt] = pick_word(v, uint32_t(lane & 3));
      }
    }
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      if (tt >= nt) break;
      const int tile = tbase + tt;
      const uint32_t pb = pen ? pen_bits[wib][tt * 32 + lane] : 0u;
      const bool in_smem = cp_ok && tile * kTile + kTile <= L;
      GroupSum r_;
      bool done = false;
      uint32_t w[16];
      if constexpr (k16) {
        if (in_smem) {
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint4 q = wb[((r * 2 + tt) * 4 + b) * 32 + lane];
            w[4 * b] = q.x; w[4 * b + 1] = q.y; w[4 * b + 2] = q.z; w[4 * b + 3] = q.w;
          }
          if (pb == 0u) {
            done = true;
            const uint32_t m0 = Cvt<T>::max2(Cvt<T>::max2(w[0], w[1]), Cvt<T>::max2(w[2], w[3]));
            const uint32_t m1 = Cvt<T>::max2(Cvt<T>::max2(w[4], w[5]), Cvt<T>::max2(w[6], w[7]));
            const uint32_t m2 = Cvt<T>::max2(Cvt<T>::max2(w[8], w[9]), Cvt<T>::max2(w[10], w[11]));
            const uint32_t m3 = Cvt<T>::max2(Cvt<T>::max2(w[12], w[13]), Cvt<T>::max2(w[14], w[15]));
            const uint32_t mm = Cvt<T>::max2(Cvt<T>::max2(m0, m1), Cvt<T>::max2(m2, m3));
            const float lo = Cvt<T>::lo(mm), hi = Cvt<T>::hi(mm);
            const float gmax = (lo != lo || hi != hi) ? __int_as_float(0x7FFFFFFF) : fmaxf(lo, hi);
            r_.gmax = gmax;
            if (idx_mode || gmax != gmax || (gmax > -INFINITY && !finite_f(__fmul_rn(gmax, c1))))
              r_.aux = __int_as_float(first_member_packed<T>(w, gmax));
            else
              r_.aux = gmax > -INFINITY ? group_sum_packed<T>(w, c1, -__fmul_rn(gmax, c1)) : 0.f;
          }
        }
      }
      if (!done) {
        float x[32];
        if constexpr (k16) {
          if (in_smem) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              x[2 * i] = Cvt<T>::lo(w[i]);
              x[2 * i + 1] = Cvt<T>::hi(w[i]);
            }
          } else {
            load_members<T>(P, src, tile, lane, L, x);
          }
        } else {
          load_members<T>(P, src, tile, lane, L, x);
        }
        if (pb) {
#pragma unroll
          for (int m = 0; m < 32; ++m)
            if ((pb >> m) & 1u) x[m] = pen_x(x[m], rpen);
        }
        float gmax = x[0];
#pragma unroll
        for (int m = 1; m < 32; ++m) gmax = fmax_nan(gmax, x[m]);
        r_.gmax = gmax;
        // rows that only need the max's position, and groups whose softmax terms
        // are not finite (the row then falls back to the greedy id), keep the
        // position of the group's max instead of its sum
        if (idx_mode || gmax != gmax || (gmax > -INFINITY && !finite_f(__fmul_rn(gmax, c1))))
          r_.aux = __int_as_float(first_member(x, gmax));
        else
          r_.aux = gmax > -INFINITY ? group_sum(x, c1, -__fmul_rn(gmax, c1)) : 0.f;
      }
      const int gl = (tp + tt) * 32 + lane;   // group index inside the task
      out[gl] = r_;
      lmax = fmax_nan(lmax, r_.gmax);
      if (idx_mode || !(r_.gmax > -INFINITY) || !finite_f(__fmul_rn(r_.gmax, c1))) continue;
      // the group's lower bound of its noise minimum
      float lo;
      if (nzrow) {
        float e = INFINITY;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int off = tile * kTile + b * 256 + lane * 8;
          const int nb = L - off;
          if (nb >= 8 && P.noise_vec) {
            const float4 q0 = __ldg(reinterpret_cast<const float4*>(nzrow + off));
            const float4 q1 = __ldg(reinterpret_cast<const float4*>(nzrow + off + 4));
            e = fminf(e, fminf(fminf(fminf(q0.x, q0.y), fminf(q0.z, q0.w)), fminf(fminf(q1.x, q1.y), fminf(q1.z, q1.w))));
          } else {
            for (int i = 0; i < 8 && i < nb; ++i) e = fminf(e, __ldg(nzrow + off + i));
          }
        }
        P.emin[size_t(row) * size_t(P.G) + size_t(g_first + gl)] = e;
        lo = e;
      } else {
        lo = emin_lower(wmin[tt]);
      }
      const float ug = __fmul_rn(r_.gmax, c1);
      const float bkey = lo > 0.f ? ug - lg2_approx(lo) : INFINITY;
      // Philox mode: the group's bound key itself, for the decide kernel's rescans
      if (!nzrow) P.emin[size_t(row) * size_t(P.G) + size_t(g_first + gl)] = bkey;
      if (ug > lu) {
        lsum = __fmaf_rn(lsum, qe_ex2_ftz(__fsub_rn(lu, ug)), r_.aux);
        lu = ug;
      } else {
        lsum = __fmaf_rn(r_.aux, qe_ex2_ftz(__fsub_rn(ug, lu)), lsum);
      }
      top.add(bkey, int(g_first + gl));
    }
  }
  if (cp_ok) cp_async_wait<0>();   // no copy outlives the warp (tiles past the task's end were not issued)
  // task record: warp reductions
  const uint32_t kmax = __reduce_max_sync(0xFFFFFFFFu, nan_key(lmax));
  const float tmax = kmax == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : key_to_float(kmax);
  TaskRec tr;
  tr.tmax = tmax;
  double ts = 0.0;
  if (!idx_mode) {
    const float ut = __fmul_rn(tmax, c1);
    if (lu > -INFINITY && finite_f(ut)) ts = double(lsum) * double(qe_ex2_ftz(__fsub_rn(lu, ut)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ts += __shfl_xor_sync(0xFFFFFFFFu, ts, o);
  }
  tr.tsum = ts;
  float kv[3];
  int kg[2];
  int h = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float hv = h == 0 ? top.b0 : h == 1 ? top.b1 : h == 2 ? top.b2 : -INFINITY;
    const int hg = h == 0 ? top.g0 : h == 1 ? top.g1 : -1;
    const uint32_t kk = ordered_key(hv);
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kk);
    const int srcl = __ffs(__ballot_sync(0xFFFFFFFFu, kk == km)) - 1;
    kv[i] = __shfl_sync(0xFFFFFFFFu, hv, srcl);
    if (i < 2) kg[i] = __shfl_sync(0xFFFFFFFFu, hg, srcl);
    if (lane == srcl) ++h;
  }
  tr.bk0 = kv[0];
  tr.bk1 = kv[1];
  tr.bceil = kv[2];
  tr.bg0 = kv[0] > -INFINITY ? kg[0] : -1;
  tr.bg1 = kv[1] > -INFINITY ? kg[1] : -1;
  if (lane == 0) P.trec[size_t(row) * size_t(P.tasks_row) + size_t(t)] = tr;
}

template <typename T>
__global__ void __launch_bounds__(kSumThreads, 3) scan_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) uint4 sbuf[];   // [warp][round][tile][block][lane]
  __shared__ uint32_t pen_bits[kSumThreads / 32][64];
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    P.ctl->err = 0u;
    P.ctl->n_pend[0] = 0u;
    P.ctl->n_pend[1] = 0u;
    P.ctl->n_retry = 0u;
    P.ctl->n_fin = 0u;
  }
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= P.tasks_row) return;   // the whole warp
#pragma unroll 1
  for (int row = blockIdx.y; row < int(P.a.batch); row += gridDim.y) {
    scan_task<T>(P, row, t, sbuf, pen_bits);
    __syncwarp();
  }
}


// ---------------------------------------------------------------- shared row helpers
// ---------------------------------------------------------------- 2. row kernel: shared state

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
      unsigned int cntw[kRowWarps][256];          // per-warp copies: less atomic contention
      unsigned long long massw[kRowWarps][256];
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
__device__ __forceinline__ void hash_build(int* hash, const RowP& rp, int64_t V) {
  for (int i = threadIdx.x; i < kHashCap; i += kRowThreads) hash[i] = -1;
  __syncthreads();
  if (rp.hash_ok) {
    for (int h = threadIdx.x; h < rp.hlen; h += kRowThreads) {
      const int id = rp.hist[h];
      if (id < 0 || int64_t(id) >= V) continue;
      uint32_t s = hslot(id);
#pragma unroll 1
      for (int probe = 0; probe < kHashCap; ++probe) {
        const int prev = atomicCAS(&hash[s], -1, id);
        if (prev == -1 || prev == id) break;
        s = (s + 1u) & uint32_t(kHashCap - 1);
      }
    }
  }
  __syncthreads();
}
__device__ __forceinline__ bool in_history(const int* hash, const RowP& rp, int id) {
  if (rp.hash_ok) {
    uint32_t s = hslot(id);
#pragma unroll 1
    for (int probe = 0; probe < kHashCap; ++probe) {
      const int v = hash[s];
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
        if (m < q.n && in_history(sm.hash, rp, bid + (m >> 3) * 256 + (m & 7))) x[m] = pen_x(x[m], rp.rp);
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
__device__ __noinline__ void race_row(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, float theta,
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
    // the noise-minimum and second members exactly (selected without
    // branches); the others bounded by their ratio with E2 first, their token
    // noise only when that can reach theta
    const float pre2 = __fmul_rn(__fmul_rn(__fmul_rn(theta, Sf), e2), 1.f - 1e-5f);
    float xa = -INFINITY, xb = -INFINITY;
    uint32_t need = 0u;
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      xa = m == a ? x[m] : xa;
      xb = m == a2 ? x[m] : xb;
      const bool pass = m < n && m != a && m != a2 && qe_ex2_ftz(__fmaf_rn(x[m], c1, c0)) >= pre2 &&
                        keep(x[m], member_id(bid, m));
      need |= pass ? (1u << m) : 0u;
    }
    if (a < n && keep(xa, member_id(bid, a)))
      top.add(__fdiv_rn(__fdiv_rn(qe_ex2_ftz(__fmaf_rn(xa, c1, c0)), Sf), emin), xa, emin, member_id(bid, a));
    if (a2 >= 0 && a2 < n && keep(xb, member_id(bid, a2)))
      top.add(__fdiv_rn(__fdiv_rn(qe_ex2_ftz(__fmaf_rn(xb, c1, c0)), Sf), e2), xb, e2, member_id(bid, a2));
#pragma unroll 1
    while (need) {
      const int m = __ffs(need) - 1;
      need &= need - 1u;
      const int id = member_id(bid, m);
      float xv = load_one<T>(P, row, id);
      if (rp.pen && in_history(sm.hash, rp, id)) xv = pen_x(xv, rp.rp);
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
__device__ __noinline__ void exact_path(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, double S,
                           float thr_m, float xf) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    for (int i = tid; i < kRowWarps * 256; i += kRowThreads) {
      (&sm.u.h.cntw[0][0])[i] = 0u;
      (&sm.u.h.massw[0][0])[i] = 0ull;
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
        atomicAdd(&sm.u.h.cntw[warp][bin], 1u);
        atomicAdd(&sm.u.h.massw[warp][bin], efix(v, c1, c0));
        if (L == 0 && thr_m > 0.f && __fdiv_rn(qe_ex2_ftz(__fmaf_rn(v, c1, c0)), Sf) >= thr_m) ++nm;
      }
    };
    lane_visit<T, false>(P, sm, rp, row, want, vis);
    nm = __reduce_add_sync(0xFFFFFFFFu, nm);
    if (lane == 0 && nm) atomicAdd(&sm.u.h.nm, nm);
    __syncthreads();
    for (int b = tid; b < 256; b += kRowThreads) {
      unsigned int c = 0u;
      unsigned long long ms = 0ull;
#pragma unroll
      for (int w = 0; w < kRowWarps; ++w) {
        c += sm.u.h.cntw[w][b];
        ms += sm.u.h.massw[w][b];
      }
      sm.u.h.cnt[b] = c;
      sm.u.h.mass[b] = ms;
    }
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
  float theta = float(mk / S / 16.0);
  race_row<T>(P, sm, rp, row, c0, Sf, theta, keep);
  // the race's best is below theta with probability e^-16; each further
  // round lowers theta 16-fold, the last one races every kept id
#pragma unroll 1
  for (int r = 1; r < 4 && !(sm.ntop > 0 && sm.top[0].r >= theta); ++r) {
    theta = r < 3 ? theta * 0.0625f : 0.f;
    race_row<T>(P, sm, rp, row, c0, Sf, theta, keep);
  }
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
__device__ __forceinline__ bool small_k(const Params& P, RowSm& sm, const RowP& rp, int row, float c0, float Sf, float thr_m) {
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

// ---------------------------------------------------------------- 2. decide kernel
struct alignas(16) DecSm {
  RowP rp;
  TaskRec tr[kMaxTasks];
  int gl[kGList];                // groups expanded in the race round
  int rs[kRescanCap];            // tasks whose every group is re-bounded
  Cand wtop[kRowWarps][kTC];
  Cand top[kTC];
  int ngl, nrs, ntop;
  uint32_t red_u[kRowWarps];
  double red_d[kRowWarps][2];
  long long red_l[kRowWarps][2];
  int hash[kHashCap];            // last: allocated only for launches with a penalty history
};

__device__ __forceinline__ uint32_t dmax_u(uint32_t* red, uint32_t v) {
  v = __reduce_max_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0u;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r = max(r, red[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ uint32_t dmin_u(uint32_t* red, uint32_t v) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0xFFFFFFFFu;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) r = min(r, red[w]);
  __syncthreads();
  return r;
}
// Two doubles and two counts summed over the CTA (fixed order: deterministic).
__device__ __forceinline__ void dsum2(DecSm& sm, double& a, double& b, long long& c, long long& d) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm.red_d[w][0] = a; sm.red_d[w][1] = b;
    sm.red_l[w][0] = c; sm.red_l[w][1] = d;
  }
  __syncthreads();
  a = b = 0.0;
  c = d = 0;
#pragma unroll
  for (int i = 0; i < kRowWarps; ++i) {
    a += sm.red_d[i][0]; b += sm.red_d[i][1];
    c += sm.red_l[i][0]; d += sm.red_l[i][1];
  }
  __syncthreads();
}

// Groups of scan task t: global ids [*g0, *g0 + *ng).
__device__ __forceinline__ void task_groups(const Params& P, int t, int64_t* g0, int* ng) {
  int s = 0;
#pragma unroll 1
  while (s + 1 < kNumSlices && P.tbase[s + 1] <= t) ++s;
  const int tile0 = (t - P.tbase[s]) * P.tpw;
  *g0 = P.gbase[s] + int64_t(tile0) * 32;
  *ng = min(P.tpw, P.snt[s] - tile0) * 32;
}

// CTA-wide kTC best of every thread's Top4 (rho desc, id asc) into sm.top.
__device__ __forceinline__ void merge_top(DecSm& sm, const Top4& top) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int h = 0;
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    float r = -1.f, xx = 0.f, EE = 1.f;
    int id = INT_MAX;
#pragma unroll
    for (int k = 0; k < kTC; ++k)
      if (k == h) { r = top.r[k]; xx = top.x[k]; EE = top.E[k]; id = top.id[k]; }
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
  if (warp == 0) {
    // lane l holds candidate l of the 32 (8 warps x kTC)
    Cand c = sm.wtop[lane / kTC][lane % kTC];
    bool used = false;
    int n = 0;
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      const uint32_t kr = (!used && c.r >= 0.f) ? __float_as_uint(c.r) + 1u : 0u;
      const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
      const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(c.id) : 0xFFFFFFFFu);
      const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(c.id) == im)) - 1;
      const Cand w{__shfl_sync(0xFFFFFFFFu, c.r, src), __shfl_sync(0xFFFFFFFFu, c.x, src),
                   __shfl_sync(0xFFFFFFFFu, c.E, src), int(im)};
      if (lane == src) used = true;
      if (lane == 0) sm.top[i] = km != 0u ? w : Cand{-1.f, 0.f, 1.f, INT_MAX};
      n += km != 0u ? 1 : 0;
    }
    if (lane == 0) sm.ntop = n;
  }
  __syncthreads();
}

// Ids a race may take: all, or (retry races) only those strictly ahead of
// (x, id) in the order (x desc, id asc); every id at or after a candidate
// that is outside the kept set is outside it too.
struct Restr {
  bool on;
  float x;
  int id;
  __device__ __forceinline__ bool ok(float v, int i) const { return !on || v > x || (v == x && i < id); }
};

// One race round: every group whose noise bound can reach theta is expanded
// exactly; sm.top gets the kTC best ratios among the ids `rs_` allows,
// complete above theta.  Returns false when a capacity ran out (the row
// then takes the exact path).
template <typename T>
__device__ __forceinline__ bool race_round(const Params& P, DecSm& sm, const RowP& rp, int row, float u, float c0, float Sf,
                           float theta, const Restr& rr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntask = P.tasks_row;
  const bool cnoise = P.a.noise != nullptr;
  // bound key threshold: 2^(bk - u) / S >= theta, with a margin for the
  // approximate logs
  const float lth = lg2_approx(theta) + u + lg2_approx(Sf) - 1e-3f;
  if (tid == 0) { sm.ngl = 0; sm.nrs = 0; }
  __syncthreads();
  for (int i = tid; i < ntask; i += kRowThreads) {
    const TaskRec& tr = sm.tr[i];
    if (rr.on && tr.tmax < rr.x) continue;
    if (tr.bk0 >= lth && tr.bg0 != int(rp.s_gid)) sm.gl[min(atomicAdd(&sm.ngl, 1), kGList - 1)] = tr.bg0;
    if (tr.bk1 >= lth && tr.bg1 != int(rp.s_gid)) sm.gl[min(atomicAdd(&sm.ngl, 1), kGList - 1)] = tr.bg1;
    if (tr.bceil >= lth) {
      const int at = atomicAdd(&sm.nrs, 1);
      if (at < kRescanCap) sm.rs[at] = i;
    }
  }
  if (tid == 0 && !cnoise && rp.s_gid >= 0) sm.gl[min(atomicAdd(&sm.ngl, 1), kGList - 1)] = int(rp.s_gid);
  __syncthreads();
  const int nrs = sm.nrs;
  if (nrs > kRescanCap) return false;
  // tasks with three or more groups above the threshold: bound every group
  for (int ri = warp; ri < nrs; ri += kRowWarps) {
    const int t = sm.rs[ri];
    const TaskRec& tr = sm.tr[t];
    int64_t g0;
    int ng;
    task_groups(P, t, &g0, &ng);
    float gms[4];
    for (int j0 = 0; j0 < ng; j0 += 128) {
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        const int j = j0 + k2 * 32 + lane;
        gms[k2] = j < ng ? P.summ[size_t(row) * size_t(P.G) + size_t(g0 + j)].gmax : -INFINITY;
      }
#pragma unroll
     for (int k2 = 0; k2 < 4; ++k2) {
      const int j = j0 + k2 * 32 + lane;
      const int64_t g = g0 + j;
      const float gm = gms[k2];
      if (j >= ng || g == tr.bg0 || g == tr.bg1 || g == rp.s_gid) continue;
      if (!(gm > -INFINITY) || (rr.on && gm < rr.x)) continue;
      // the group's bound key: stored by the scan kernel in Philox mode, from
      // the group's noise minimum in caller-noise mode
      const float ev = P.emin[size_t(row) * size_t(P.G) + size_t(g)];
      const float bk = !cnoise ? ev : (ev > 0.f ? __fmul_rn(gm, rp.c1) - lg2_approx(ev) : INFINITY);
      if (bk >= lth) sm.gl[min(atomicAdd(&sm.ngl, 1), kGList - 1)] = int(g);
     }
    }
  }
  __syncthreads();
  const int ngl = sm.ngl;
  if (ngl >= kGList) return false;
  // expansion: one group per thread
  const float c1 = rp.c1;
  const float pref = __fmul_rn(__fmul_rn(theta, Sf), 1.f - 1e-5f);   // e >= pref * E needed to reach theta
  Top4 top;
  top.init();
  const unsigned char* rsrc = static_cast<const unsigned char*>(P.a.logits) + size_t(row) * size_t(P.a.ld) * P.esize;
  const float* nz = cnoise ? P.a.noise + size_t(row) * size_t(P.a.noise_ld) : nullptr;
  for (int i = tid; i < ngl; i += kRowThreads) {
    const int64_t g = sm.gl[i];
    const GrpGeo q = grp_geo(P, g);
    float x[32];
    load_members<T>(P, rsrc + size_t(q.base) * P.esize, q.lg >> 5, q.lg & 31, q.L, x);
    const int bid = group_base_id(q);
    if (rp.pen) {
#pragma unroll
      for (int m = 0; m < 32; ++m)
        if (m < q.n && in_history(sm.hash, rp, member_id(bid, m))) x[m] = pen_x(x[m], rp.rp);
    }
    const int n = q.n;
    if (cnoise) {
#pragma unroll
      for (int m = 0; m < 32; ++m) {
        if (m >= n) continue;
        const float e = qe_ex2_ftz(__fmaf_rn(x[m], c1, c0));
        const int id = member_id(bid, m);
        const float E = __ldg(nz + id);
        if (!(e >= __fmul_rn(pref, E)) || !rr.ok(x[m], id)) continue;
        top.add(__fdiv_rn(__fdiv_rn(e, Sf), E), x[m], E, id);
      }
      continue;
    }
    const bool holds = g == rp.s_gid;
    const U4 wd = philox_at(rp.key, uint32_t(g), kTagGroup);
    int am;
    float emin;
    if (holds) {
      am = rp.s_mem;
      emin = rp.e_root;
    } else {
      am = int(select_index32(wd.y, uint32_t(n)));
      const float l = neglog(uniform_open(group_min_word(rp.key, g)));
      emin = __fadd_rn(rp.e_root, n == 32 ? __fmul_rn(l, 0.03125f) : __fdiv_rn(l, float(n)));
    }
    int a2 = -1;
    float e2 = INFINITY;
    if (n >= 2) {
      e2 = __fadd_rn(emin, __fdiv_rn(neglog(uniform_open(wd.z)), float(n - 1)));
      const int i2 = int(select_index32(wd.w, uint32_t(n - 1)));
      a2 = i2 < am ? i2 : i2 + 1;
    }
    const float pre2 = __fmul_rn(pref, e2);
    // the noise-minimum and second members exactly (selected without
    // branches: the members differ from lane to lane); every other member
    // only marked when RN(p/E2) can reach theta
    float xa = -INFINITY, xb = -INFINITY;
    uint32_t need = 0u;
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      xa = m == am ? x[m] : xa;
      xb = m == a2 ? x[m] : xb;
      const bool pass = m < n && m != am && m != a2 && qe_ex2_ftz(__fmaf_rn(x[m], c1, c0)) >= pre2 &&
                        rr.ok(x[m], member_id(bid, m));
      need |= pass ? (1u << m) : 0u;
    }
    if (am < n) {
      const int id = member_id(bid, am);
      const float e = qe_ex2_ftz(__fmaf_rn(xa, c1, c0));
      if (rr.ok(xa, id) && e >= __fmul_rn(pref, emin)) top.add(__fdiv_rn(__fdiv_rn(e, Sf), emin), xa, emin, id);
    }
    if (a2 >= 0 && a2 < n) {
      const int id = member_id(bid, a2);
      const float e = qe_ex2_ftz(__fmaf_rn(xb, c1, c0));
      if (rr.ok(xb, id) && e >= pre2) top.add(__fdiv_rn(__fdiv_rn(e, Sf), e2), xb, e2, id);
    }
#pragma unroll 1
    while (need) {
      const int m = __ffs(need) - 1;
      need &= need - 1u;
      const int id = member_id(bid, m);
      float xv = load_one<T>(P, row, id);
      if (rp.pen && in_history(sm.hash, rp, id)) xv = pen_x(xv, rp.rp);
      const float p = __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xv, c1, c0)), Sf);
      if (!rbetter(__fdiv_rn(p, e2), id, top.r[kTC - 1], top.id[kTC - 1])) continue;
      const float E = __fadd_rn(e2, neglog(uniform_open(pick_word(philox_at(rp.key, uint32_t(id >> 2), kTagToken),
                                                                   uint32_t(id & 3)))));
      top.add(__fdiv_rn(p, E), xv, E, id);
    }
  }
  merge_top(sm, top);
  return true;
}

__device__ __forceinline__ void push_fin(const Params& P, int row, unsigned kind) {
  const unsigned at = atomicAdd(&P.ctl->n_fin, 1u);
  P.flist[at] = int(unsigned(row) | (kind << 28));
}

// Race and kept-set test of a sampled row whose max and normaliser are
// known.  Up to three rounds: the race (complete above 1/4, else above 1/16;
// the best ratio is below those with probability e^-4 and e^-16), then the
// test of its candidates in race order, from the task records and then the
// group records.  A candidate outside the kept set restricts the next round
// to the ids ahead of it.  Undecided candidates go to the count kernel of
// `round`; rows still open after the rounds go to the finish kernel.
template <typename T>
__device__ __forceinline__ void sample_rounds(const Params& P, DecSm& sm, const RowP& rp, int row, float u, float Sf, double S,
                              float thr_m, Restr rr, int round) {
  const int tid = threadIdx.x;
  const int ntask = P.tasks_row;
  const int64_t V = P.a.vocab;
  const float c0 = -u;
  RowState* rs = P.rstate + row;
  const double tpS = double(rp.tp) * S;
  const GroupSum* gs = P.summ + size_t(row) * size_t(P.G);
  const int G = int(P.G);
#pragma unroll 1
  for (int it = 0; it < 3; ++it) {
    // one call site of the race (complete above 1/4, else above 1/16)
    float theta = 0.25f;
    bool ok = false;
#pragma unroll 1
    for (int rnd = 0; rnd < 2; ++rnd) {
      theta = rnd == 0 ? 0.25f : 0.0625f;
      ok = race_round<T>(P, sm, rp, row, u, c0, Sf, theta, rr);
      if (!ok || (sm.ntop > 0 && sm.top[0].r >= theta)) break;
    }
    if (!ok || !(sm.ntop > 0 && sm.top[0].r >= theta)) break;
    if (!rp.filtered) {
      write_row(P, row, sm.top[0].id, 0, V);
      return;
    }
    const int ntop = sm.ntop;
    Restr nr = rr;
#pragma unroll 1
    for (int i = 0; i < ntop; ++i) {
      const Cand c = sm.top[i];
      if (!(c.r >= theta)) break;
      const float e = qe_ex2_ftz(__fmaf_rn(c.x, rp.c1, c0));
      bool in_p = true, in_k = true, out = false;
      if (rp.m_on && __fdiv_rn(e, Sf) < thr_m) {
        out = true;   // removed by min-p
      } else {
        double U = 0.0, Lm = 0.0;
        long long N = 0, Lc = 0;
        for (int t = tid; t < ntask; t += kRowThreads) {
          const TaskRec& tr = sm.tr[t];
          if (!(tr.tmax >= c.x)) continue;
          U += tr.tsum * double(qe_ex2_ftz(__fsub_rn(__fmul_rn(tr.tmax, rp.c1), u)));
          int64_t g0;
          int ng;
          task_groups(P, t, &g0, &ng);
          N += (long long)ng * 32;
        }
        dsum2(sm, U, Lm, N, Lc);
        in_p = !rp.p_on || U - double(e) <= tpS * (1.0 - 1e-6);
        in_k = !rp.k_on || N - 1 < rp.k;
        if (!(in_p && in_k)) {
          // group level: eight record loads in flight per thread
          U = 0.0; N = 0;
          for (int gb = tid; gb < G; gb += kRowThreads * 8) {
            GroupSum v[8];
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
              const int g = gb + k2 * kRowThreads;
              v[k2] = g < G ? gs[g] : GroupSum{-INFINITY, 0.f};
            }
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
              if (!(v[k2].gmax >= c.x)) continue;
              U += double(v[k2].aux) * double(qe_ex2_ftz(__fsub_rn(__fmul_rn(v[k2].gmax, rp.c1), u)));
              N += 32;
              if (v[k2].gmax > c.x) {
                Lm += double(qe_ex2_ftz(__fmaf_rn(v[k2].gmax, rp.c1, c0)));
                Lc += 1;
              }
            }
          }
          dsum2(sm, U, Lm, N, Lc);
          in_p = !rp.p_on || U - double(e) <= tpS * (1.0 - 1e-6);
          in_k = !rp.k_on || N - 1 < rp.k;
          out = (rp.p_on && Lm > tpS * (1.0 + 1e-6)) || (rp.k_on && Lc >= rp.k);
        }
      }
      if (!out && in_p && in_k) {
        write_row(P, row, c.id, 0, 0);
        return;
      }
      if (out) {
        if (!nr.on || c.x > nr.x || (c.x == nr.x && c.id < nr.id)) nr = Restr{true, c.x, c.id};
        continue;
      }
      // undecided: the count kernel counts this and every later candidate
      if (tid == 0) {
        int n = 0;
        for (int j = i; j < ntop; ++j) {
          const Cand cj = sm.top[j];
          if (!(cj.r >= theta)) break;
          rs->cand[n] = cj;
          rs->cmass[n] = 0ull;
          rs->ccnt[n] = 0ull;
          ++n;
        }
        rs->ncand = n;
        rs->done = 0u;
        rs->rx = nr.on ? nr.x : INFINITY;
        rs->rid = nr.on ? nr.id : -1;
        const unsigned at = atomicAdd(&P.ctl->n_pend[round], 1u);
        P.plist[size_t(round) * size_t(P.a.batch) + at] = row;
      }
      return;
    }
    rr = nr;   // every candidate is outside the kept set
  }
  if (tid == 0) push_fin(P, row, kFinExact);
}

// Row parameters and the noise root of `row` into sm.rp (thread 0).
__device__ __forceinline__ void load_row_params(const Params& P, DecSm& sm, int row) {
  RowP r = row_params(P, row);
  if (!P.a.noise && r.kind != kKindGreedy && r.kind != kKindArgmax) {
    const NoiseRoot rt = noise_root(r.key, P.a.vocab);
    int64_t gsd = -1;
    int rm = 0;
    token_group_p(P, rt.s, &gsd, &rm);
    r.e_root = rt.e_root;
    r.s_gid = gsd;
    r.s_mem = rm;
  }
  sm.rp = r;
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) decide_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DecSm& sm = *reinterpret_cast<DecSm*>(smem_raw);
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int64_t V = P.a.vocab;
  const int ntask = P.tasks_row;
  const TaskRec* trg = P.trec + size_t(row) * size_t(ntask);
  if (tid == 0) load_row_params(P, sm, row);   // inputs only: overlaps the scan's tail
  wait_prior_grid();
  for (int i = tid; i < ntask; i += kRowThreads) sm.tr[i] = trg[i];
  __syncthreads();
  const RowP rp = sm.rp;
  const bool idx_mode = rp.kind == kKindGreedy || rp.kind == kKindArgmax;
  uint32_t kmax = 0u;
  for (int i = tid; i < ntask; i += kRowThreads) kmax = max(kmax, nan_key(sm.tr[i].tmax));
  kmax = dmax_u(sm.red_u, kmax);
  const float xmax = kmax == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : key_to_float(kmax);
  const float u = __fmul_rn(xmax, rp.c1);
  bool fin = finite_f(xmax) && finite_f(u);
  double S = 0.0;
  if (!idx_mode && fin) {
    double a = 0.0, b = 0.0;
    long long c = 0, d = 0;
    for (int i = tid; i < ntask; i += kRowThreads) {
      const TaskRec& tr = sm.tr[i];
      const float ut = __fmul_rn(tr.tmax, rp.c1);
      if (tr.tmax > -INFINITY && finite_f(ut)) a += tr.tsum * double(qe_ex2_ftz(__fsub_rn(ut, u)));
    }
    dsum2(sm, a, b, c, d);
    S = a;
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
      const int lane = tid & 31, warp = tid >> 5;
      for (int t = warp; t < ntask; t += kRowWarps) {
        const float tm = sm.tr[t].tmax;
        if (!(xn ? tm != tm : tm == xmax)) continue;
        int64_t g0;
        int ng;
        task_groups(P, t, &g0, &ng);
        for (int j = lane; j < ng; j += 32) {
          const GroupSum sg = P.summ[size_t(row) * size_t(P.G) + size_t(g0 + j)];
          if (!(xn ? sg.gmax != sg.gmax : sg.gmax == xmax)) continue;
          const GrpGeo q = grp_geo(P, g0 + j);
          first = min(first, uint32_t(q.base + member_offset(q.lg, __float_as_int(sg.aux))));
        }
      }
      first = dmin_u(sm.red_u, first);
    } else {
      first = 0u;   // every logit is -inf: torch.argmax returns 0
    }
    const int status = rp.kind == kKindGreedy ? QE_ROW_GREEDY : (!fin ? QE_ROW_NONFINITE : 0);
    write_row(P, row, first, status, rp.kind == kKindArgmax && fin ? 1 : 0);
    return;
  }
  const float Sf = float(S);
  const float thr_m = rp.m_on ? __fmul_rn(rp.minp, __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xmax, rp.c1, -u)), Sf)) : 0.f;
  RowState* rs = P.rstate + row;
  if (tid == 0) {
    rs->xmax = xmax; rs->u = u; rs->Sf = Sf; rs->thr_m = thr_m; rs->S = S;
    rs->ncand = 0; rs->done = 0u;
  }
  if (rp.kind == kKindSmallK || rp.exact) {
    if (tid == 0) push_fin(P, row, rp.kind == kKindSmallK ? kFinSmallK : kFinExact);
    return;
  }
  if (rp.pen) hash_build(sm.hash, rp, V);
  sample_rounds<T>(P, sm, rp, row, u, Sf, S, thr_m, Restr{false, 0.f, 0}, 0);
}

// Retry round: rows whose counted candidates were all outside the kept set
// race again, restricted to the ids ahead of the best of them.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) retry_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DecSm& sm = *reinterpret_cast<DecSm*>(smem_raw);
  wait_prior_grid();
  const unsigned nr = *reinterpret_cast<volatile unsigned*>(&P.ctl->n_retry);
  const int tid = threadIdx.x;
  const int ntask = P.tasks_row;
#pragma unroll 1
  for (unsigned li = blockIdx.x; li < nr; li += gridDim.x) {
    const int row = P.rlist[li];
    const TaskRec* trg = P.trec + size_t(row) * size_t(ntask);
    for (int i = tid; i < ntask; i += kRowThreads) sm.tr[i] = trg[i];
    if (tid == 0) load_row_params(P, sm, row);
    __syncthreads();
    const RowP rp = sm.rp;
    const RowState* rs = P.rstate + row;
    const float u = rs->u, Sf = rs->Sf, thr_m = rs->thr_m;
    const double S = rs->S;
    const Restr rr{true, rs->rx, rs->rid};
    if (rp.pen) hash_build(sm.hash, rp, P.a.vocab);
    sample_rounds<T>(P, sm, rp, row, u, Sf, S, thr_m, rr, 1);
    __syncthreads();
  }
}

// ---------------------------------------------------------------- 3. count kernel
// Exact count and mass of the ids ahead of each pending candidate, one warp
// per (pending row, scan task); the warp that completes a row decides it.
// A row whose candidates are all outside the kept set goes to the retry
// round (from the first round) or to the finish kernel (from the retry round).
template <typename T>
__global__ void __launch_bounds__(kSumThreads) count_kernel(const __grid_constant__ Params P, int round) {
  __shared__ uint32_t pen_bits[kSumThreads / 32][64];
  wait_prior_grid();
  const unsigned npend = *reinterpret_cast<volatile unsigned*>(&P.ctl->n_pend[round]);
  if (npend == 0u) return;
  const int* plist = P.plist + size_t(round) * size_t(P.a.batch);
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int tiles_row = int(P.G / 32);
  const long long items = (long long)npend * tiles_row;   // one tile (32 groups, a lane each) per item
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  const KernelArgs& a = P.a;
#pragma unroll 1
  for (long long item = (long long)blockIdx.x * (blockDim.x >> 5) + wib; item < items; item += nw) {
    const int row = plist[item / tiles_row];
    const int gt = int(item % tiles_row);   // global tile index: groups [gt*32, gt*32+32)
    RowState* rs = P.rstate + row;
    const GroupSum sg = P.summ[size_t(row) * size_t(P.G) + size_t(gt) * 32 + lane];
    const int nc = rs->ncand;
    Cand cand[kTC];
    float xlo = INFINITY;
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      cand[i] = i < nc ? rs->cand[i] : Cand{-1.f, INFINITY, 1.f, -1};
      if (i < nc) xlo = fminf(xlo, cand[i].x);
    }
    const float c1 = temp_coef(a.temperatures[row]);
    const float c0 = -rs->u;
    float rpen = 1.f;
    int hl = 0;
    if (a.history && a.rep_penalties) {
      rpen = a.rep_penalties[row];
      hl = a.history_lens ? a.history_lens[row] : int(a.history_ld);
      hl = hl < 0 ? 0 : (hl > int(a.history_ld) ? int(a.history_ld) : hl);
    }
    const bool pen = hl > 0 && !(rpen == 1.f);
    int s = 0;
#pragma unroll
    for (int step = 8; step > 0; step >>= 1)
      if (s + step < kNumSlices && P.gbase[s + step] <= int64_t(gt) * 32) s += step;
    const int tile = int((int64_t(gt) * 32 - P.gbase[s]) / 32);
    const int64_t sa = P.sstart[s];
    const int L = int(P.sstart[s + 1] - sa);
    if (pen) pen_bits_build(pen_bits[wib], a.history + row * a.history_ld, hl, sa, tile, 1, L);
    // per candidate: mass (fp32 per lane, then 2^-40 fixed point) and count
    // of the ids strictly ahead of it
    float msf[kTC] = {0.f, 0.f, 0.f, 0.f};
    unsigned long long ms[kTC], ct[kTC] = {0ull, 0ull, 0ull, 0ull};
    if (sg.gmax >= xlo) {
      const unsigned char* src = static_cast<const unsigned char*>(a.logits) + (size_t(row) * size_t(a.ld) + size_t(sa)) * P.esize;
      float x[32];
      load_members<T>(P, src, tile, lane, L, x);
      const uint32_t pb = pen ? pen_bits[wib][lane] : 0u;
      if (pb) {
#pragma unroll
        for (int m = 0; m < 32; ++m)
          if ((pb >> m) & 1u) x[m] = pen_x(x[m], rpen);
      }
      const int bid = int(sa) + tile * kTile + lane * 8;
      float e[32];
#pragma unroll
      for (int m = 0; m < 32; ++m) e[m] = qe_ex2_ftz(__fmaf_rn(x[m], c1, c0));
#pragma unroll
      for (int i = 0; i < kTC; ++i) {
        if (i >= nc) break;
        const float cx = cand[i].x;
        const int cid = cand[i].id;
        float acc = 0.f;
        unsigned int cnt = 0u;
#pragma unroll
        for (int m = 0; m < 32; ++m) {
          const bool ahead = x[m] > cx || (x[m] == cx && member_id(bid, m) < cid);
          acc += ahead ? e[m] : 0.f;
          cnt += ahead ? 1u : 0u;
        }
        msf[i] = acc;
        ct[i] = cnt;
      }
    }
#pragma unroll
    for (int i = 0; i < kTC; ++i) ms[i] = __float2ull_rn(msf[i] * 1099511627776.0f);
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ms[i] += __shfl_xor_sync(0xFFFFFFFFu, ms[i], o);
        ct[i] += __shfl_xor_sync(0xFFFFFFFFu, ct[i], o);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kTC; ++i) {
        if (i < nc && ms[i]) atomicAdd(&rs->cmass[i], ms[i]);
        if (i < nc && ct[i]) atomicAdd(&rs->ccnt[i], ct[i]);
      }
      __threadfence();
      const unsigned d = atomicAdd(&rs->done, 1u);
      if (d == unsigned(tiles_row - 1)) {
        __threadfence();
        // the row's counts are complete: first candidate inside the kept set
        const float tp_ = a.top_ps ? a.top_ps[row] : 1.f;
        const bool p_on = (a.flags & QE_FLAG_USE_TOP_P) && a.top_ps && tp_ < 1.f;
        const long long kraw = a.top_ks ? (long long)a.top_ks[row] : 0;
        const bool k_on = kraw > 0 && kraw < a.vocab;
        const double S = rs->S;
        const unsigned long long tfix =
            p_on ? static_cast<unsigned long long>(floor(double(tp_) * S * 1099511627776.0)) : ~0ull;
        const float Sf = rs->Sf, thr_m = rs->thr_m;
        const bool m_on = a.min_ps && a.min_ps[row] > 0.f;
        long long win = -1;
        float bx = rs->rx;
        int bid2 = rs->rid;
        for (int i = 0; i < nc; ++i) {
          const unsigned long long mm = atomicAdd(&rs->cmass[i], 0ull);
          const unsigned long long cc = atomicAdd(&rs->ccnt[i], 0ull);
          const bool in = !(m_on && __fdiv_rn(qe_ex2_ftz(__fmaf_rn(cand[i].x, c1, c0)), Sf) < thr_m) &&
                          (!k_on || (long long)cc < kraw) && mm <= tfix;
          if (in) {
            win = cand[i].id;
            break;
          }
          // outside: the ids at and after it are outside too
          if (bid2 < 0 || cand[i].x > bx || (cand[i].x == bx && cand[i].id < bid2)) {
            bx = cand[i].x;
            bid2 = cand[i].id;
          }
        }
        if (win >= 0) {
          a.out_ids[row] = win;
          if (a.out_status) a.out_status[row] = 0;
          if (a.out_kept) a.out_kept[row] = 0;
        } else if (round == 0) {
          rs->rx = bx;
          rs->rid = bid2;
          const unsigned at = atomicAdd(&P.ctl->n_retry, 1u);
          P.rlist[at] = row;
        } else {
          push_fin(P, row, kFinExact);
        }
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- 4. finish kernel
// Rows that need the kept set itself: small top-k rows, rows whose race
// candidates all fall outside the kept set, rows whose kept-set size was
// asked for.  Persistent CTAs over the finish list.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) finish_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowSm& sm = *reinterpret_cast<RowSm*>(smem_raw);
  wait_prior_grid();
  const unsigned nfin = *reinterpret_cast<volatile unsigned*>(&P.ctl->n_fin);
  const int tid = threadIdx.x;
  const int64_t V = P.a.vocab;
#pragma unroll 1
  for (unsigned li = blockIdx.x; li < nfin; li += gridDim.x) {
    const unsigned ent = unsigned(P.flist[li]);
    const int row = int(ent & 0x0FFFFFFFu);
    const unsigned kind = ent >> 28;
    if (tid == 0) {
      RowP r = row_params(P, row);
      if (!P.a.noise) {
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
    const RowState* rs = P.rstate + row;
    const float u = rs->u, Sf = rs->Sf, thr_m = rs->thr_m;
    const double S = rs->S;
    if (rp.pen) hash_build(sm.hash, rp, V);
    if (kind == kFinSmallK) {
      if (!small_k<T>(P, sm, rp, row, -u, Sf, thr_m)) exact_path<T>(P, sm, rp, row, -u, Sf, S, thr_m, -INFINITY);
    } else {
      exact_path<T>(P, sm, rp, row, -u, Sf, S, thr_m, -INFINITY);
    }
    __syncthreads();
  }
}


// ---------------------------------------------------------------- host
struct DevInfo {
  bool ready = false;
  int sms = 0;
};
std::mutex g_mu;
DevInfo g_dev[64];

constexpr size_t kDecSmFull = sizeof(DecSm);
constexpr size_t kDecSmNoHash = offsetof(DecSm, hash);

template <typename T>
cudaError_t prepare() {
  cudaError_t e = cudaFuncSetAttribute(finish_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(RowSm)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(scan_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kScanSmem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decide_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDecSmFull));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(retry_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDecSmFull));
  return e;
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

// Launch with programmatic stream serialization (see wait_prior_grid).
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem, cudaStream_t st,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename T>
cudaError_t launch_all(const Params& P, dim3 g1, unsigned g2, size_t dec_smem, unsigned g3, unsigned g4,
                       cudaStream_t stream) {
  scan_kernel<T><<<g1, kSumThreads, kScanSmem, stream>>>(P);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = launch_dependent(decide_kernel<T>, dim3(g2), kRowThreads, dec_smem, stream, P);
  if (e == cudaSuccess) e = launch_dependent(count_kernel<T>, dim3(g3), kSumThreads, 0, stream, P, 0);
  if (e == cudaSuccess) e = launch_dependent(retry_kernel<T>, dim3(g4), kRowThreads, dec_smem, stream, P);
  if (e == cudaSuccess) e = launch_dependent(count_kernel<T>, dim3(g3), kSumThreads, 0, stream, P, 1);
  if (e == cudaSuccess) e = launch_dependent(finish_kernel<T>, dim3(g4), kRowThreads, sizeof(RowSm), stream, P);
  return e;
}

}  // namespace st

bool stream_supports(int64_t vocab) { return vocab >= 1 && vocab < (int64_t(1) << 24); }

size_t stream_workspace_bytes(int64_t batch, int64_t vocab) {
  const size_t a = st::make_layout(batch, vocab, 2).total, b = st::make_layout(batch, vocab, 4).total;
  return a > b ? a : b;
}

const void* stream_error_word(const void* workspace) {
  return static_cast<const char*>(workspace) + offsetof(st::Ctl, err);
}

int launch_stream(const KernelArgs& ka, cudaStream_t stream) {
  using namespace st;
  const int esize = ka.dtype == QE_DTYPE_F32 ? 4 : 2;
  if (ka.batch >= (int64_t(1) << 28)) return set_error(QE_ERR_UNSUPPORTED, "batch too large");
  const Layout L = make_layout(ka.batch, ka.vocab, esize);
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
  P.tpw = L.tpw;
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
  if (tb != L.tasks || gb != L.G) return set_error(QE_ERR_CUDA, "stream sampler: inconsistent layout");
  char* base = static_cast<char*>(ka.workspace);
  P.ctl = reinterpret_cast<Ctl*>(base);
  P.summ = reinterpret_cast<GroupSum*>(base + L.summ);
  P.trec = reinterpret_cast<TaskRec*>(base + L.trec);
  P.emin = reinterpret_cast<float*>(base + L.emin);
  P.rstate = reinterpret_cast<RowState*>(base + L.rstate);
  P.plist = reinterpret_cast<int*>(base + L.plist);
  P.rlist = reinterpret_cast<int*>(base + L.rlist);
  P.flist = reinterpret_cast<int*>(base + L.flist);
  // scan: one warp per task, a 2-D grid of (task blocks, rows)
  const dim3 g1(unsigned((tb + kSumThreads / 32 - 1) / (kSumThreads / 32)),
                unsigned(ka.batch < 65535 ? ka.batch : 65535));
  const unsigned g2 = unsigned(ka.batch);
  const bool pen = ka.history && ka.rep_penalties;
  const size_t dec_smem = pen ? kDecSmFull : kDecSmNoHash;
  const long long cwarps = ((long long)ka.batch * (L.G / 32) + 7) / 8;
  const unsigned g3 = unsigned(cwarps < (long long)sms * 4 ? (cwarps < 1 ? 1 : cwarps) : (long long)sms * 4);
  const unsigned g4 = unsigned(ka.batch < (int64_t)sms * 2 ? ka.batch : (int64_t)sms * 2);
  cudaError_t e;
  switch (ka.dtype) {
    case QE_DTYPE_F32: e = launch_all<float>(P, g1, g2, dec_smem, g3, g4, stream); break;
    case QE_DTYPE_BF16: e = launch_all<__nv_bfloat16>(P, g1, g2, dec_smem, g3, g4, stream); break;
    default: e = launch_all<__half>(P, g1, g2, dec_smem, g3, g4, stream); break;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("stream sampler launch: ") + cudaGetErrorString(e));
  return QE_OK;
}

}  // namespace qe
