// qe_sample_stream.cu — the default sampler path: one persistent launch that
// reads every row of logits from HBM once.
//
// Replaces BatchSampler.forward (src/compute/sampler.py:25-41) and the
// extensions of this library (top-k, min-p, repetition penalty, Philox
// noise).  The semantics of a sample are those of qe_sample_ref.cu and the
// CPU oracle: softmax of the penalised logits / T, kept set = the longest
// prefix of the order (x desc, id asc) allowed by top-k, top-p and min-p,
// token = argmax over the kept set of RN(RN(e/S)/E).
//
// Work is split into chunks (qe_stream.cuh).  Each CTA runs one producer warp
// and eight compute warps.  The producer claims work items from global
// counters and moves each chunk into one of two shared-memory buffers with a
// 1-D bulk copy (mbarrier completion); the compute warps reduce it:
//
//   pass 1   per 32-id group: NaN-propagating packed max, then the sum of
//            2^(x c1 - RN(gmax c1)) (the only per-token exponential)
//   race     lazy exponential race over the Philox noise tree: a group's best
//            ratio is bounded from its noise minimum; only groups (and then
//            tokens) whose bound reaches the running threshold get exact
//            noise.  The chunk files its best candidates and a ceiling over
//            every other token.
//   gather   small top-k rows (k <= 64) file every token at or above a lower
//            bound of the chunk's k-th largest logit instead.
//
// The CTA that files a row's last record merges the row (max, S, greedy id,
// candidates) and either writes the token or publishes a follow-up round:
// a test of the candidates' kept-set membership (mass and rank ahead of
// them), or the exact rounds (radix histogram of the kept-set boundary, tie
// counts, race over the kept set).  Follow-up items go to any CTA and re-read
// their chunk from L2.  No CTA ever waits for another; every wait is bounded.
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

using fz::bulk_g2s;
using fz::fence_proxy_async;
using fz::key_to_float;
using fz::mbar_expect_tx;
using fz::mbar_init;
using fz::mbar_wait;
using fz::ordered_key;
using fz::rbetter;
using fz::smem_u32;

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_relaxed(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Release/acquire fence at GPU scope, issued by one thread after a CTA
// barrier: it orders the whole CTA's earlier writes (cumulativity through the
// barrier) before that thread's next signal, and its later reads after it.
__device__ __forceinline__ void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void st_release(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
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
// Barrier of the compute warps only (the producer warp never joins it).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }
__device__ __forceinline__ bool csync_or(bool p) {
  int r;
  asm volatile(
      "{\n .reg .pred a, b;\n setp.ne.s32 a, %1, 0;\n bar.red.or.pred b, 1, %2, a;\n selp.s32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"(int(p)), "n"(kThreads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------- launch parameters
struct Params {
  KernelArgs a;
  int esize, tpc, cps, nc;
  int tma_ok, noise_vec, force_exact, dtype_level;
  uint32_t polls, data_polls;
  unsigned int nitems;
  int64_t sstart[kNumSlices + 1];
  int64_t gbase[kNumSlices + 1];
  int snt[kNumSlices];
  Ctl* ctl;
  RowCtl* rowctl;
  unsigned int* queue;
  ChunkRec* rec;
  float* hist;
  GItem* gather;
  RowRound* round;
  Part* part;
  HistAcc* hacc;
};

// ---------------------------------------------------------------- row parameters
struct RowP {
  int kind;
  bool p_on, k_on, m_on, filtered, pen, exact;
  float T, c1, tp, minp, rp;
  long long k;
  const int32_t* hist;
  int hlen;
};

// ---------------------------------------------------------------- shared memory
struct Q2Ent {
  uint16_t lg;
  uint8_t arg, arg2;
  float E2;   // lower bound on the group's second smallest noise
};
constexpr int kFCap = 256;   // race finalists per chunk (overflow: conservative)
constexpr int kFW = 64;      // race finalists per warp in the chunk pass (overflow: conservative)

struct alignas(128) Smem {
  unsigned char buf[kNumBuf][kBufBytes];
  uint64_t full[kNumBuf];
  uint64_t empty[kNumBuf];
  // per buffer, written by the producer before it completes `full`
  int kind[kNumBuf];            // ItemKind
  int chunk[kNumBuf];           // chunk index of a chunk or follow-up item
  int frow[kNumBuf];            // row of the item
  int bulk_elems[kNumBuf];      // elements delivered by the bulk copy
  RowP rowp[kNumBuf];           // the row's parameters
  float root_e[kNumBuf];        // the row's noise-tree root (Philox mode)
  long long root_gid[kNumBuf];
  int root_mem[kNumBuf];
  // per buffer, written by the compute warps before they release it: the row
  // whose part they filed (-1: none); the producer turns it into an arrival
  int mail[kNumBuf];
  int finq[kFinQ];              // producer-private ring of rows to finish
  long long bcast_pre;
  int nq1, nq2, nq3;
  int ngath, over;
  int red_greedy;
  float lk;
  float e_root;
  int s_mem;
  long long s_gid;
  float cceil;
  int ncand;
  Cand cand[kR];
  Cand tc[kTC];
  int ntc;
  uint32_t pen[kMaxGroups];
  float gmax[kMaxGroups];
  uint32_t red_k[kWarps];
  int red_i[kWarps];
  double red_d[kWarps];
  long long red_l[kWarps];
  Cand wl[kWarps][kR];
  float wceil[kWarps];
  Q2Ent q2[kQ2Cap];
  uint16_t fq[kFCap];           // race finalists: type << 14 | local group << 5 | member
  int nf;
  float theta;
  unsigned int ceil_bits;       // CTA ceiling (non-negative float bits, atomicMax)
  float wtop[kWarps][kR];
  // warp-local chunk pass: each warp's max (ordered key), exponent anchor,
  // sum in its own scale, and finalists
  uint32_t wr_key[kWarps];
  float wr_u[kWarps];
  double wr_S[kWarps];
  uint16_t fqw[kWarps][kFW];
  uint32_t phist[kWarps][kBins];
  float topm[kWarps][kTopM];
  GItem gl[kGCap];
  double pd[kWarps][kTC];
  long long pl[kWarps][kTC];
  RowRound rr;
  union {
    struct {
      unsigned int cnt[256];
      unsigned long long mass[256];
      unsigned int nm;
    } h;
    struct {
      uint32_t bits[kMaxGroups];
      uint32_t pre[kMaxGroups];
    } t;
    unsigned long long keys[kSortCap];
    struct {
      float rho[kSmallK];
      int keep[kSmallK];
      int id[kSmallK];
    } sk;
  } u;
};

// ---------------------------------------------------------------- geometry
struct Geo {
  int row, chunk, ntiles, len;
  int64_t start, gbase;
};
__device__ __forceinline__ Geo geo_of(const Params& P, int row, int chunk) {
  Geo g;
  g.row = row;
  g.chunk = chunk;
  const int s = chunk / P.cps, part = chunk % P.cps;
  const int t0 = part * P.tpc;
  const int nt = P.snt[s];
  const int t1 = min(nt, t0 + P.tpc);
  g.ntiles = t1 > t0 ? t1 - t0 : 0;
  g.start = P.sstart[s] + int64_t(t0) * kTile;
  const int64_t rem = P.sstart[s + 1] - g.start;
  g.len = g.ntiles > 0 ? int(rem < int64_t(g.ntiles) * kTile ? rem : int64_t(g.ntiles) * kTile) : 0;
  g.gbase = P.gbase[s] + int64_t(t0) * 32;
  return g;
}
// Offset (inside the chunk) of member m of the group in lane gl of tile `tile`.
__device__ __forceinline__ int moff(int tile, int gl, int m) {
  return tile * kTile + (m >> 3) * 256 + gl * 8 + (m & 7);
}
// Members of that group inside a chunk of `len` ids (a prefix of 0..31).
__device__ __forceinline__ int gsize(int len, int tile, int gl) {
  int n = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int c = len - (tile * kTile + b * 256 + gl * 8);
    n += c <= 0 ? 0 : (c >= 8 ? 8 : c);
  }
  return n;
}

__device__ __noinline__ RowP row_params(const Params& P, int row) {
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
  if (a.history) {
    hl = a.history_lens ? a.history_lens[row] : int(a.history_ld);
    hl = hl < 0 ? 0 : (hl > int(a.history_ld) ? int(a.history_ld) : hl);
  }
  r.hlen = hl;
  r.hist = a.history ? a.history + row * a.history_ld : nullptr;
  r.pen = hl > 0 && !(r.rp == 1.f);
  r.kind = greedy ? kKindGreedy
                  : (r.k_on && k == 1) ? kKindArgmax : (r.k_on && k <= kSmallK) ? kKindSmallK : kKindRace;
  r.exact = P.force_exact && r.filtered && !greedy;
  return r;
}

__device__ __forceinline__ NoiseKey row_key(const Params& P, int row) {
  const KernelArgs& a = P.a;
  const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
  return make_noise_key(row_seed(a, row), step, a.row_offset + row);
}

// ---------------------------------------------------------------- elements
template <typename T> struct Elt;
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float at(const unsigned char* b, int o) {
    return __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(b)[o]) << 16);
  }
  static __device__ __forceinline__ void neg_inf(unsigned char* b, int o) {
    reinterpret_cast<uint16_t*>(b)[o] = 0xFF80u;
  }
  static __device__ __forceinline__ void copy(unsigned char* b, int o, const void* src, int64_t j) {
    reinterpret_cast<uint16_t*>(b)[o] = __ldg(reinterpret_cast<const unsigned short*>(src) + j);
  }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float at(const unsigned char* b, int o) {
    return __half2float(reinterpret_cast<const __half*>(b)[o]);
  }
  static __device__ __forceinline__ void neg_inf(unsigned char* b, int o) {
    reinterpret_cast<uint16_t*>(b)[o] = 0xFC00u;
  }
  static __device__ __forceinline__ void copy(unsigned char* b, int o, const void* src, int64_t j) {
    reinterpret_cast<uint16_t*>(b)[o] = __ldg(reinterpret_cast<const unsigned short*>(src) + j);
  }
};
template <> struct Elt<float> {
  static __device__ __forceinline__ float at(const unsigned char* b, int o) {
    return reinterpret_cast<const float*>(b)[o];
  }
  static __device__ __forceinline__ void neg_inf(unsigned char* b, int o) {
    reinterpret_cast<float*>(b)[o] = -INFINITY;
  }
  static __device__ __forceinline__ void copy(unsigned char* b, int o, const void* src, int64_t j) {
    reinterpret_cast<float*>(b)[o] = __ldg(reinterpret_cast<const float*>(src) + j);
  }
};

// Penalised logit of member m of group (tile, gl).
template <typename T>
__device__ __forceinline__ float xval(const Smem& sm, const unsigned char* buf, const RowP& rp, int tile, int gl,
                                      int m) {
  float x = Elt<T>::at(buf, moff(tile, gl, m));
  if (rp.pen && ((sm.pen[tile * 32 + gl] >> m) & 1u)) x = penalise(x, rp.rp);
  return x;
}

// Tail of the chunk beyond the bulk copy (plain loads) and -inf padding up to
// the end of the last tile.
template <typename T>
__device__ void fill_chunk(const Params& P, unsigned char* buf, const Geo& g, int bulk_elems) {
  const int total = g.ntiles * kTile;
  const void* src = static_cast<const unsigned char*>(P.a.logits) +
                    (size_t(g.row) * size_t(P.a.ld) + size_t(g.start)) * size_t(P.esize);
  for (int o = bulk_elems + int(threadIdx.x); o < total; o += kThreads) {
    if (o < g.len) Elt<T>::copy(buf, o, src, o);
    else Elt<T>::neg_inf(buf, o);
  }
}

// Repetition-penalty bits of the chunk: bit m of pen[lg] marks member m of
// local group lg as a history id.
__device__ __forceinline__ void build_pen(Smem& sm, const Geo& g, const RowP& rp) {
  for (int i = threadIdx.x; i < g.ntiles * 32; i += kThreads) sm.pen[i] = 0u;
  csync();
  for (int h = threadIdx.x; h < rp.hlen; h += kThreads) {
    const int64_t o = int64_t(rp.hist[h]) - g.start;
    if (o >= 0 && o < g.len) {
      const int lg = int(o >> 10) * 32 + int((o >> 3) & 31);
      const int m = int(((o >> 8) & 3) * 8 + (o & 7));
      atomicOr(&sm.pen[lg], 1u << m);
    }
  }
  csync();
}

// ---------------------------------------------------------------- pass 1
struct G1 {
  float gmax, fsum;
};

template <typename T> struct Pack;
template <> struct Pack<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
};
template <> struct Pack<__half> {
  static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
    __half2 r = __hmax2_nan(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
};

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

// A group holding history ids: unpack, penalise, reduce in fp32.
template <typename T>
__device__ __forceinline__ G1 pass1_pen(const unsigned char* buf, const RowP& rp, int tile, int lane, uint32_t pb,
                                     bool sum) {
  G1 g;
  float x[32];
#pragma unroll
  for (int m = 0; m < 32; ++m) {
    float v = Elt<T>::at(buf, moff(tile, lane, m));
    if ((pb >> m) & 1u) v = penalise(v, rp.rp);
    x[m] = v;
  }
  float mx = x[0];
#pragma unroll
  for (int m = 1; m < 32; ++m) mx = fmax_nan(mx, x[m]);
  g.gmax = mx;
  g.fsum = 0.f;
  if (!sum || !(g.gmax > -INFINITY)) return g;
  g.fsum = group_sum(x, rp.c1, -__fmul_rn(g.gmax, rp.c1));
  return g;
}

// Group max (NaN-propagating) and, when `sum`, the group-relative sum
// fsum = sum_j 2^(x_j c1 - RN(gmax c1)).
template <typename T>
__device__ __forceinline__ G1 pass1(const Smem& sm, const unsigned char* buf, const RowP& rp, int tile, int lane,
                                    bool sum) {
  G1 g;
  const uint32_t pb = rp.pen ? sm.pen[tile * 32 + lane] : 0u;
  float x[32];
  if constexpr (sizeof(T) == 2) {
    if (pb == 0u) {
      const uint16_t* p = reinterpret_cast<const uint16_t*>(buf) + tile * kTile + lane * 8;
      uint32_t w[16];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint4 q = *reinterpret_cast<const uint4*>(p + b * 256);
        w[4 * b] = q.x;
        w[4 * b + 1] = q.y;
        w[4 * b + 2] = q.z;
        w[4 * b + 3] = q.w;
      }
      uint32_t m0 = Pack<T>::max2(Pack<T>::max2(w[0], w[1]), Pack<T>::max2(w[2], w[3]));
      uint32_t m1 = Pack<T>::max2(Pack<T>::max2(w[4], w[5]), Pack<T>::max2(w[6], w[7]));
      uint32_t m2 = Pack<T>::max2(Pack<T>::max2(w[8], w[9]), Pack<T>::max2(w[10], w[11]));
      uint32_t m3 = Pack<T>::max2(Pack<T>::max2(w[12], w[13]), Pack<T>::max2(w[14], w[15]));
      const uint32_t mm = Pack<T>::max2(Pack<T>::max2(m0, m1), Pack<T>::max2(m2, m3));
      const float lo = Pack<T>::lo(mm), hi = Pack<T>::hi(mm);
      g.gmax = (lo != lo || hi != hi) ? __int_as_float(0x7FFFFFFF) : fmaxf(lo, hi);
      g.fsum = 0.f;
      if (!sum || !(g.gmax > -INFINITY)) return g;   // no mass (all -inf) or NaN (row not finite)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        x[2 * i] = Pack<T>::lo(w[i]);
        x[2 * i + 1] = Pack<T>::hi(w[i]);
      }
      g.fsum = group_sum(x, rp.c1, -__fmul_rn(g.gmax, rp.c1));
      return g;
    }
  } else {
    if (pb == 0u) {
      const float* p = reinterpret_cast<const float*>(buf) + tile * kTile + lane * 8;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float4 q0 = *reinterpret_cast<const float4*>(p + b * 256);
        const float4 q1 = *reinterpret_cast<const float4*>(p + b * 256 + 4);
        x[8 * b] = q0.x; x[8 * b + 1] = q0.y; x[8 * b + 2] = q0.z; x[8 * b + 3] = q0.w;
        x[8 * b + 4] = q1.x; x[8 * b + 5] = q1.y; x[8 * b + 6] = q1.z; x[8 * b + 7] = q1.w;
      }
      float mx = x[0];
#pragma unroll
      for (int m = 1; m < 32; ++m) mx = fmax_nan(mx, x[m]);
      g.gmax = mx;
      g.fsum = 0.f;
      if (!sum || !(g.gmax > -INFINITY)) return g;
      g.fsum = group_sum(x, rp.c1, -__fmul_rn(g.gmax, rp.c1));
      return g;
    }
  }
  return pass1_pen<T>(buf, rp, tile, lane, pb, sum);
}

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ uint32_t nan_key(float v) { return ordered_key(v); }   // NaN above +inf

// Offer each lane's candidate (r >= 0; r < 0: none) to the warp's list wl of
// R entries in race order (r desc, id asc).  Whatever does not stay in the
// list raises the warp's ceiling.
__device__ __forceinline__ void warp_offer(Cand* wl, float* wceil, int R, float r, float x, float E, int id) {
  const int lane = threadIdx.x & 31;
  uint32_t kr = r >= 0.f ? __float_as_uint(r) + 1u : 0u;
  float ceil = 0.f;
  while (true) {
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
    if (km == 0u) break;
    const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(id) : 0xFFFFFFFFu);
    const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(id) == im)) - 1;
    const float br = __shfl_sync(0xFFFFFFFFu, r, src);
    const float bx = __shfl_sync(0xFFFFFFFFu, x, src);
    const float bE = __shfl_sync(0xFFFFFFFFu, E, src);
    const int bid = int(im);
    int entered = 0;
    if (lane == 0) {
      if (rbetter(br, bid, wl[R - 1].r, wl[R - 1].id)) {
        if (wl[R - 1].r >= 0.f) ceil = fmaxf(ceil, wl[R - 1].r);
        int i = R - 1;
        while (i > 0 && rbetter(br, bid, wl[i - 1].r, wl[i - 1].id)) {
          wl[i] = wl[i - 1];
          --i;
        }
        wl[i] = Cand{br, bx, bE, bid};
        entered = 1;
      }
    }
    entered = __shfl_sync(0xFFFFFFFFu, entered, 0);
    if (lane == src) kr = 0u;
    if (!entered) {
      // the best remaining candidate did not enter the list: neither will the rest
      const uint32_t rest = __reduce_max_sync(0xFFFFFFFFu, kr);
      if (lane == 0) {
        ceil = fmaxf(ceil, br);
        if (rest) ceil = fmaxf(ceil, __uint_as_float(rest - 1u));
      }
      break;
    }
  }
  if (lane == 0 && ceil > 0.f) *wceil = fmaxf(*wceil, ceil);
  __syncwarp();
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ void raise_ceiling(Smem& sm, float lc) {
  lc = warp_max(lc);
  if ((threadIdx.x & 31) == 0 && lc > 0.f) {
    float* w = &sm.wceil[threadIdx.x >> 5];
    *w = fmaxf(*w, lc);
  }
}
__device__ __forceinline__ float cta_theta(const Smem& sm, int R) {
  float t = -1.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t = fmaxf(t, sm.wl[w][R - 1].r);
  return t;
}

// Merge the warp lists into the CTA's R best (sm.cand, sm.ncand) and the
// ceiling over every other token (sm.cceil).  Warp 0 only.
__device__ __forceinline__ void merge_lists(Smem& sm, int R) {
  if ((threadIdx.x >> 5) != 0) return;
  const int lane = threadIdx.x & 31;
  Cand c{-1.f, 0.f, 1.f, INT_MAX};
  if (lane < kWarps * R) c = sm.wl[lane / R][lane % R];
  float cl = lane < kWarps ? sm.wceil[lane] : 0.f;
  uint32_t kr = c.r >= 0.f ? __float_as_uint(c.r) + 1u : 0u;
  int n = 0;
  for (int i = 0; i < R; ++i) {
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
    if (km == 0u) break;
    const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(c.id) : 0xFFFFFFFFu);
    const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(c.id) == im)) - 1;
    const float r = __shfl_sync(0xFFFFFFFFu, c.r, src), x = __shfl_sync(0xFFFFFFFFu, c.x, src);
    const float E = __shfl_sync(0xFFFFFFFFu, c.E, src);
    if (lane == 0) sm.cand[i] = Cand{r, x, E, int(im)};
    if (lane == src) kr = 0u;
    ++n;
  }
  if (kr) cl = fmaxf(cl, c.r);
  cl = warp_max(cl);
  if (lane == 0) {
    sm.ncand = n;
    sm.cceil = cl;
  }
  __syncwarp();
}

// ---------------------------------------------------------------- kept-set predicate
// Exact race rounds race only over the kept set: key(x) >> sh above kkey,
// or equal to it and among the first `allow` such ids of the chunk (tie
// ranks from the chunk's tie bitmap).  Everywhere else `on` is 0.
struct Keep {
  int on;
  int sh;
  uint32_t kkey;
  int ties_all;
  long long allow;
  __device__ __forceinline__ bool operator()(const Smem& sm, float x, int o) const {
    if (!on) return true;
    const uint32_t k = ordered_key(x) >> sh;
    if (k != kkey) return k > kkey;
    if (ties_all) return true;
    if (allow <= 0) return false;
    const uint32_t w = sm.u.t.bits[o >> 5];
    return (long long)(sm.u.t.pre[o >> 5] + __popc(w & ((1u << (o & 31)) - 1u))) < allow;
  }
  __device__ __forceinline__ bool group_may(float gm) const {
    return !on || (ordered_key(gm) >> sh) >= kkey;
  }
};

// ---------------------------------------------------------------- exact group noise
// Out-of-line copies of the noise arithmetic: they run for a few groups and
// tokens per chunk, and inlining them at every call site multiplies the
// kernel's code size (instruction-cache misses cost more than the calls).
__device__ __noinline__ U4 philox_nl(const NoiseKey& key, uint32_t index, uint32_t tag) {
  return philox_at(key, index, tag);
}
__device__ __noinline__ float neglog_nl(float u) { return neglog(u); }
__device__ __noinline__ float div_nl(float a, float b) { return __fdiv_rn(a, b); }
__device__ __noinline__ double exp2_nl(double d) { return exp2(d); }
__device__ __forceinline__ float emin_exact(const U4& w, int n, bool holds, float e_root) {
  if (holds) return e_root;
  const float l = neglog_nl(uniform_open(w.x));
  return __fadd_rn(e_root, n == 32 ? __fmul_rn(l, 0.03125f) : div_nl(l, float(n)));
}
__device__ __forceinline__ int arg_of(const U4& w, int n, bool holds, int s_mem) {
  return holds ? s_mem : int(select_index32(w.y, uint32_t(n)));
}
__device__ __forceinline__ float e2_exact(const U4& w, int n, float emin) {
  return __fadd_rn(emin, div_nl(neglog_nl(uniform_open(w.z)), float(n - 1)));
}
__device__ __forceinline__ int arg2_of(const U4& w, int n, int arg) {
  const int i2 = int(select_index32(w.w, uint32_t(n - 1)));
  return i2 < arg ? i2 : i2 + 1;
}

// Global group id and member index of token j (the slice table of the launch).
__device__ __forceinline__ void token_group_p(const Params& P, int64_t j, int64_t* gid, int* mem) {
  int sl = 0;
  while (sl + 1 < kNumSlices && P.sstart[sl + 1] <= j) ++sl;
  const int64_t o = j - P.sstart[sl];
  *gid = P.gbase[sl] + local_group(o);
  *mem = member_index(o);
}

// The kTC best (rho desc, id asc) that one thread has seen.
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
  __device__ __forceinline__ Cand at(int i) const {
    Cand c{-1.f, 0.f, 1.f, INT_MAX};
#pragma unroll
    for (int k = 0; k < kTC; ++k)
      if (k == i) c = Cand{r[k], x[k], E[k], id[k]};
    return c;
  }
};

// ---------------------------------------------------------------- race: Philox noise tree
// Bounds first, exact noise last.  Every group gets one Philox call; its two
// smallest noises are bracketed with the hardware log (lg2.approx, whose
// error is far inside the 3e-5 relative + 3e-5 absolute margin used here),
// giving lower and upper bounds on the ratios of its noise-minimum and
// second-minimum members and an upper bound on all its other members.  The
// R-th largest lower bound is a valid threshold; whatever can still reach it
// becomes a finalist and only finalists get the exact noise of the tree
// (oracle-identical IEEE arithmetic).  Everything else feeds the ceiling.
enum : int { kFinA = 0, kFinB = 1, kFinT = 2 };

// Exact noise of a finalist (noise minimum, second minimum or another member
// m of the group with global id gid and n members); *mem gets the member.
// Out of line with scalar arguments only.
__device__ __noinline__ float finalist_noise(NoiseKey key, long long gid, int n, long long s_gid, int s_mem,
                                             float e_root, int type, int m, long long j, int* mem) {
  const U4 w = philox_at(key, uint32_t(gid), kTagGroup);
  const bool holds = gid == s_gid;
  const int arg = arg_of(w, n, holds, s_mem);
  const float emin = emin_exact(w, n, holds, e_root);
  *mem = arg;
  if (type == kFinA) return emin;
  const float e2 = e2_exact(w, n, emin);
  if (type == kFinB) {
    *mem = arg2_of(w, n, arg);
    return e2;
  }
  *mem = m;
  const U4 wt = philox_at(key, uint32_t(j >> 2), kTagToken);
  const uint32_t word = (j & 3) == 0 ? wt.x : (j & 3) == 1 ? wt.y : (j & 3) == 2 ? wt.z : wt.w;
  return __fadd_rn(e2, neglog(uniform_open(word)));
}

// Exact candidate for a finalist.
template <typename T>
__device__ __forceinline__ Cand finalist(const Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp,
                                         const NoiseKey& key, float c0s, uint32_t code) {
  const int type = int(code >> 14), lg = int((code >> 5) & 0x1FFu), m = int(code & 31u);
  const int tile = lg >> 5, gl = lg & 31;
  int mem = 0;
  const float E = finalist_noise(key, g.gbase + lg, gsize(g.len, tile, gl), sm.s_gid, sm.s_mem, sm.e_root, type, m,
                                 g.start + moff(tile, gl, m), &mem);
  const float x = xval<T>(sm, buf, rp, tile, gl, mem);
  return Cand{div_nl(qe_ex2_ftz(__fmaf_rn(x, rp.c1, c0s)), E), x, E, int(g.start + moff(tile, gl, mem))};
}

__device__ __forceinline__ void push_finalist(Smem& sm, uint32_t code, float hi, float& lc) {
  const int f = atomicAdd(&sm.nf, 1);
  if (f < kFCap) sm.fq[f] = uint16_t(code);
  else lc = fmaxf(lc, hi);   // not evaluated: the ceiling keeps the record honest
}

// Race over the chunk in the scale c0s: leaves the R best (ratio e/E, with
// e = 2^(x c1 + c0s)) in sm.cand and a ceiling over every other (kept) token
// in sm.cceil.
template <typename T>
__device__ __forceinline__ void race_philox(const Params& P, Smem& sm, const unsigned char* buf, const Geo& g,
                                         const RowP& rp, float c0s, int R, const Keep& keep) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const NoiseKey key = row_key(P, g.row);
  const float c1 = rp.c1, e_root = sm.e_root;
  const long long s_gid = sm.s_gid;
  const int s_mem = sm.s_mem;
  if (lane == 0) {
    for (int i = 0; i < R; ++i) sm.wl[warp][i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
    sm.wceil[warp] = 0.f;
  }
  if (tid == 0) {
    sm.nq2 = 0;
    sm.nf = 0;
    sm.ceil_bits = 0u;
  }
  // A: bounds for the lane's two groups
  float alo[2], ahi[2], blo[2], bhi[2], ob[2], el2[2];
  int ag[2], ag2[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    alo[s] = ahi[s] = blo[s] = bhi[s] = ob[s] = -1.f;
    el2[s] = 1.f;
    ag[s] = ag2[s] = 0;
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles) continue;
    const int lg = tile * 32 + lane;
    const float gm = sm.gmax[lg];
    const int n = gsize(g.len, tile, lane);
    if (n <= 0 || !(gm > -INFINITY) || !keep.group_may(gm)) continue;
    const long long gid = g.gbase + lg;
    const U4 w = philox_at(key, uint32_t(gid), kTagGroup);
    const bool holds = gid == s_gid;
    const int a = arg_of(w, n, holds, s_mem);
    float lo1 = e_root, hi1 = e_root;
    if (!holds) {
      const float la = -lg2_approx(uniform_open(w.x)) * 0.6931472f;
      const float inv = 1.f / float(n);
      lo1 = (e_root + fmaxf(0.f, la * (1.f - 3e-5f) - 3e-5f) * inv) * (1.f - 2e-6f);
      hi1 = (e_root + (la * (1.f + 3e-5f) + 3e-5f) * inv) * (1.f + 2e-6f);
    }
    ag[s] = a;
    const float xa = xval<T>(sm, buf, rp, tile, lane, a);
    if (keep(sm, xa, moff(tile, lane, a))) {
      const float ea = qe_ex2_ftz(__fmaf_rn(xa, c1, c0s));
      alo[s] = __fdividef(ea, hi1) * (1.f - 1e-5f);
      ahi[s] = __fdividef(ea, lo1) * (1.f + 1e-5f);
    }
    if (n >= 2) {
      const float lz = -lg2_approx(uniform_open(w.z)) * 0.6931472f;
      const float inv1 = 1.f / float(n - 1);
      const float lo2 = (lo1 + fmaxf(0.f, lz * (1.f - 3e-5f) - 3e-5f) * inv1) * (1.f - 2e-6f);
      const float hi2 = (hi1 + (lz * (1.f + 3e-5f) + 3e-5f) * inv1) * (1.f + 2e-6f);
      const int a2 = arg2_of(w, n, a);
      ag2[s] = a2;
      el2[s] = lo2;
      const float xb = xval<T>(sm, buf, rp, tile, lane, a2);
      if (keep(sm, xb, moff(tile, lane, a2))) {
        const float eb = qe_ex2_ftz(__fmaf_rn(xb, c1, c0s));
        blo[s] = __fdividef(eb, hi2) * (1.f - 1e-5f);
        bhi[s] = __fdividef(eb, lo2) * (1.f + 1e-5f);
      }
      if (n >= 3) ob[s] = __fdividef(qe_ex2_ftz(__fmaf_rn(gm, c1, c0s)), lo2) * (1.f + 1e-5f);
    }
  }
  // the warp's R largest lower bounds
  {
    float v0 = alo[0], v1 = blo[0], v2 = alo[1], v3 = blo[1];
    for (int round = 0; round < R; ++round) {
      const float m = fmaxf(fmaxf(v0, v1), fmaxf(v2, v3));
      const float wm = warp_max(m);
      if (lane == 0) sm.wtop[warp][round] = wm;
      const unsigned bal = __ballot_sync(0xFFFFFFFFu, m == wm);
      if (lane == __ffs(bal) - 1) {
        if (v0 == wm) v0 = -1.f;
        else if (v1 == wm) v1 = -1.f;
        else if (v2 == wm) v2 = -1.f;
        else v3 = -1.f;
      }
    }
  }
  csync();
  // threshold: the R-th largest lower bound of the CTA (a valid lower bound
  // on the chunk's R-th best ratio)
  if (warp == 0) {
    const int nv = kWarps * R;
    const float a = lane < nv ? sm.wtop[lane / R][lane % R] : -2.f;
    int rank = 0;
    for (int j = 0; j < nv; ++j) {
      const float bj = __shfl_sync(0xFFFFFFFFu, a, j);
      rank += int(bj > a || (bj == a && j < lane));
    }
    if (lane < nv && rank == R - 1) sm.theta = a;
  }
  csync();
  const float theta = sm.theta;
  // B: what can still reach the threshold becomes a finalist or an expansion
  float lc = 0.f;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int lg = (warp + kWarps * s) * 32 + lane;
    if (ahi[s] >= 0.f) {
      if (ahi[s] >= theta) push_finalist(sm, uint32_t(kFinA << 14) | uint32_t(lg << 5), ahi[s], lc);
      else lc = fmaxf(lc, ahi[s]);
    }
    if (bhi[s] >= 0.f) {
      if (bhi[s] >= theta) push_finalist(sm, uint32_t(kFinB << 14) | uint32_t(lg << 5), bhi[s], lc);
      else lc = fmaxf(lc, bhi[s]);
    }
    if (ob[s] >= 0.f) {
      if (ob[s] >= theta) {
        const int q = atomicAdd(&sm.nq2, 1);
        if (q < kQ2Cap) sm.q2[q] = Q2Ent{uint16_t(lg), uint8_t(ag[s]), uint8_t(ag2[s]), el2[s]};
        else lc = fmaxf(lc, ob[s]);
      } else {
        lc = fmaxf(lc, ob[s]);
      }
    }
  }
  csync();
  // C: members of expanded groups whose bound reaches the threshold
  const int nq2 = min(sm.nq2, kQ2Cap);
#pragma unroll 1
  for (int e = warp; e < nq2; e += kWarps) {
    const Q2Ent q = sm.q2[e];
    const int tile = q.lg >> 5, gl = q.lg & 31;
    const int n = gsize(g.len, tile, gl);
    const int m = lane;
    if (m < n && m != q.arg && m != q.arg2) {
      const float xm = xval<T>(sm, buf, rp, tile, gl, m);
      if (keep(sm, xm, moff(tile, gl, m))) {
        const float bm = __fdividef(qe_ex2_ftz(__fmaf_rn(xm, c1, c0s)), q.E2) * (1.f + 1e-5f);
        if (bm >= theta) push_finalist(sm, uint32_t(kFinT << 14) | uint32_t(q.lg << 5) | uint32_t(m), bm, lc);
        else lc = fmaxf(lc, bm);
      }
    }
  }
  lc = warp_max(lc);
  if (lane == 0 && lc > 0.f) atomicMax(&sm.ceil_bits, __float_as_uint(lc));
  csync();
  // D: exact noise for the finalists, ranked in the warp lists
  const int nf = min(sm.nf, kFCap);
  for (int base = 0; base < nf; base += kThreads) {
    const int e = base + tid;
    Cand c{-1.f, 0.f, 1.f, INT_MAX};
    if (e < nf) c = finalist<T>(sm, buf, g, rp, key, c0s, sm.fq[e]);
    warp_offer(sm.wl[warp], &sm.wceil[warp], R, c.r, c.x, c.E, c.id);
  }
  csync();
  merge_lists(sm, R);
  if (tid == 0) sm.cceil = fmaxf(sm.cceil, __uint_as_float(sm.ceil_bits));
  csync();
}

// ---------------------------------------------------------------- race: caller noise (parity mode)
template <typename T>
__device__ __forceinline__ void race_noise(const Params& P, Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp,
                           float c0s, int R, const Keep& keep) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float c1 = rp.c1;
  if (lane == 0) {
    for (int i = 0; i < R; ++i) sm.wl[warp][i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
    sm.wceil[warp] = 0.f;
  }
  __syncwarp();
  // the lane's own kR best (exact ratios) and a ceiling over the rest
  Top4 best;
  best.init();
  float lc = 0.f;
  const float* nz = P.a.noise + size_t(g.row) * size_t(P.a.noise_ld) + size_t(g.start);
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles) continue;
    const float gm = sm.gmax[tile * 32 + lane];
    const int n = gsize(g.len, tile, lane);
    if (n <= 0 || !(gm > -INFINITY) || !keep.group_may(gm)) continue;
#pragma unroll 1
    for (int m = 0; m < n; ++m) {
      const int o = moff(tile, lane, m);
      const float x = xval<T>(sm, buf, rp, tile, lane, m);
      if (!keep(sm, x, o)) continue;
      const float ev = qe_ex2_ftz(__fmaf_rn(x, c1, c0s));
      const float E = __ldg(nz + o);
      const float ap = __fdividef(ev, E) * (1.f + 1e-5f);
      if (!(ap >= best.r[kTC - 1])) {
        lc = fmaxf(lc, ap);
        continue;
      }
      const float r = __fdiv_rn(ev, E);
      if (best.r[kTC - 1] >= 0.f && !rbetter(r, int(g.start + o), best.r[kTC - 1], best.id[kTC - 1])) {
        lc = fmaxf(lc, r);
        continue;
      }
      if (best.r[kTC - 1] >= 0.f) lc = fmaxf(lc, best.r[kTC - 1]);
      best.add(r, x, E, int(g.start + o));
    }
  }
#pragma unroll
  for (int i = 0; i < kTC; ++i) warp_offer(sm.wl[warp], &sm.wceil[warp], R, best.r[i], best.x[i], best.E[i], best.id[i]);
  raise_ceiling(sm, lc);
  csync();
  merge_lists(sm, R);
  csync();
}

template <typename T>
__device__ __forceinline__ void race(const Params& P, Smem& sm, const unsigned char* buf, const Geo& g,
                                     const RowP& rp, float c0s, int R, const Keep& keep) {
  if (P.a.noise) race_noise<T>(P, sm, buf, g, rp, c0s, R, keep);
  else race_philox<T>(P, sm, buf, g, rp, c0s, R, keep);
}

// ---------------------------------------------------------------- chunk max / greedy id
// Pass 1 over the chunk's groups (two per lane), the chunk max into
// red_k (as an ordered key) and sm.gmax per group.  Returns the lane's slots.
template <typename T>
__device__ void chunk_pass1(Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp, bool sum, G1 sl[2],
                            float* cmax_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t kmax = 0u;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    sl[s] = G1{-INFINITY, 0.f};
    const int tile = warp + kWarps * s;
    if (tile < g.ntiles) {
      sl[s] = pass1<T>(sm, buf, rp, tile, lane, sum);
      sm.gmax[tile * 32 + lane] = sl[s].gmax;
      kmax = max(kmax, nan_key(sl[s].gmax));
    }
  }
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  if (lane == 0) sm.red_k[warp] = kmax;
  csync();
  uint32_t k = 0u;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) k = max(k, sm.red_k[w]);
  *cmax_out = g.ntiles > 0 ? (k == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : key_to_float(k)) : -INFINITY;
}

// First id of the chunk whose value is cmax (the first NaN when cmax is NaN).
template <typename T>
__device__ __noinline__ int chunk_greedy(Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp, const G1 sl[2],
                            float cmax) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool cnan = cmax != cmax;
  int best = INT_MAX;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles) continue;
    const float gm = sl[s].gmax;
    if (!(cnan ? gm != gm : gm == cmax)) continue;
    const int n = gsize(g.len, tile, lane);
    for (int m = 0; m < n; ++m) {
      const float x = xval<T>(sm, buf, rp, tile, lane, m);
      if (cnan ? x != x : x == cmax) {
        best = min(best, int(g.start + moff(tile, lane, m)));
        break;
      }
    }
  }
  best = __reduce_min_sync(0xFFFFFFFFu, best);
  if (lane == 0) sm.red_i[warp] = best;
  csync();
  int r = INT_MAX;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) r = min(r, sm.red_i[w]);
  return r;
}

// CTA sum of a per-thread double (compute warps).
__device__ double cta_sum_d(Smem& sm, double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) sm.red_d[threadIdx.x >> 5] = v;
  csync();
  double s = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += sm.red_d[w];
  csync();
  return s;
}
__device__ long long cta_sum_l(Smem& sm, long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0) sm.red_l[threadIdx.x >> 5] = v;
  csync();
  long long s = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += sm.red_l[w];
  csync();
  return s;
}

// ---------------------------------------------------------------- small top-k gather
// Files every token of the chunk at or above lk, a lower bound on the
// chunk's k-th largest (penalised) logit: the k-th largest among each warp's
// kTopM largest group maxima (k group maxima, hence k tokens, reach it).
template <typename T>
__device__ __forceinline__ void gather_head(Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp, const G1 sl[2]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = int(rp.k);
  float v0 = warp < g.ntiles ? sl[0].gmax : -INFINITY;
  float v1 = warp + kWarps < g.ntiles ? sl[1].gmax : -INFINITY;
#pragma unroll 1
  for (int i = 0; i < kTopM; ++i) {
    const float b = fmaxf(v0, v1);
    const uint32_t kb = ordered_key(b);
    const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kb);
    const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kb == km)) - 1;
    if (lane == 0) sm.topm[warp][i] = key_to_float(km);
    if (lane == src) {
      if (v0 >= v1) v0 = -INFINITY;
      else v1 = -INFINITY;
    }
  }
  if (tid == 0) {
    sm.ngath = 0;
    sm.over = 0;
    sm.lk = -INFINITY;
  }
  csync();
  if (tid < kWarps * kTopM) {
    const float* tv = &sm.topm[0][0];
    const float a = tv[tid];
    int r = 0;
#pragma unroll 1
    for (int j = 0; j < kWarps * kTopM; ++j) {
      const float b = tv[j];
      r += int(b > a || (b == a && j < tid));
    }
    if (r == k - 1) sm.lk = a;
  }
  csync();
  const float lk = sm.lk;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles || !(sl[s].gmax >= lk)) continue;
    const int n = gsize(g.len, tile, lane);
    for (int m = 0; m < n; ++m) {
      const float x = xval<T>(sm, buf, rp, tile, lane, m);
      if (x >= lk) {
        const int i = atomicAdd(&sm.ngath, 1);
        if (i < kGCap) sm.gl[i] = GItem{x, int(g.start + moff(tile, lane, m))};
        else sm.over = 1;
      }
    }
  }
  csync();
}

// ---------------------------------------------------------------- row completion
__device__ __noinline__ void complete_row(const Params& P, int row, long long id, int status, long long kept) {
  if (threadIdx.x != 0) return;
  const KernelArgs& a = P.a;
  a.out_ids[row] = id;
  if (a.out_status) a.out_status[row] = status;
  if (a.out_kept) a.out_kept[row] = kept;
  fence_acq_rel();
  atomicAdd(&P.ctl->rows_done, 1u);
}

// Publish the round in sm.rr for `row` (thread 0; callers csync before).
__device__ __forceinline__ void publish(const Params& P, Smem& sm, int row) {
  if (threadIdx.x != 0) return;
  P.round[row] = sm.rr;
  P.rowctl[row].cnt = 0u;
  P.rowctl[row].round = unsigned(sm.rr.type);
  fence_acq_rel();
  const unsigned e = atomicAdd(&P.ctl->qentries, 1u);
  if (e < unsigned(P.a.batch) * kMaxRounds) {
    st_release(&P.queue[e], unsigned(row) + 1u);
  } else {
    // cannot happen (a row publishes at most 7 rounds); never leave the row open
    atomicOr(&P.ctl->err, 2u);
    complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
  }
}

__device__ __forceinline__ int final_level(const Params& P, const RowP& rp) {
  return rp.pen ? 3 : P.dtype_level;
}

// min-p threshold on p: RN(min_p * p_max), 0 when min-p is off.
__device__ __forceinline__ float minp_threshold(const RowP& rp, float xmax, float c0, float Sf) {
  if (!rp.m_on) return 0.f;
  return __fmul_rn(rp.minp, __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xmax, rp.c1, c0)), Sf));
}

// Start the exact rounds for a row whose candidates could not decide it.
__device__ __forceinline__ void enter_exact(const Params& P, Smem& sm, int row, const RowP& rp, float c0, float Sf, double S,
                            float thr_m) {
  HistAcc* h = P.hacc + row;
  for (int i = threadIdx.x; i < 256; i += kThreads) {
    h->cnt[i] = 0u;
    h->mass[i] = 0ull;
  }
  if (threadIdx.x == 0) {
    h->nm = 0u;
    RowRound& r = sm.rr;
    r.type = kRoundHist;
    r.level = 0;
    r.prefix = 0u;
    r.m = 0;
    r.c0 = c0;
    r.Sf = Sf;
    r.S = S;
    r.kk = rp.k;
    r.tfix = ~0ull;
    r.sfix = 0ull;
    r.acnt = 0;
    r.amass = 0ull;
    r.kkey = 0u;
    r.ties_all = 1;
    r.kties = 0;
    r.nkeep = 0;
    r.thr_m = thr_m;
  }
  csync();
  publish(P, sm, row);
}


__device__ __forceinline__ unsigned long long efix(float x, float c1, float c0) {
  return __float2ull_rn(qe_ex2_ftz(__fmaf_rn(x, c1, c0)) * 1099511627776.0f);   // 2^40 fixed point
}

// ---------------------------------------------------------------- CTA-wide best candidates
__device__ float cta_max_f(Smem& sm, float v) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sm.red_k[threadIdx.x >> 5] = __float_as_uint(v);
  csync();
  float m = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m = fmaxf(m, __uint_as_float(sm.red_k[w]));
  csync();
  return m;
}

// Sum kTC doubles and kTC counts over the compute threads; the totals land
// in every thread's arrays.
__device__ void cta_part(Smem& sm, double* ms, long long* ct) {
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
  csync();
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    double a = 0.0;
    long long b = 0;
    for (int w = 0; w < kWarps; ++w) {
      a += sm.pd[w][i];
      b += sm.pl[w][i];
    }
    ms[i] = a;
    ct[i] = b;
  }
  csync();
}

__device__ __forceinline__ bool row_timed_out(const Params& P, int row) {
  return __ldcg(&P.rowctl[row].timeout) != 0u;
}
__device__ __noinline__ void mark_timeout(const Params& P, int row) {
  if (threadIdx.x == 0) {
    atomicOr(&P.rowctl[row].timeout, 1u);
    atomicOr(&P.ctl->err, 1u);
  }
}

// Move the chunk's tail beyond the bulk copy into shared memory, pad it, and
// build the repetition-penalty bits.
template <typename T>
__device__ void load_chunk(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk, const RowP& rp) {
  fill_chunk<T>(P, buf, g, bulk);
  if (rp.pen) build_pen(sm, g, rp);
  else csync();
}

// ---------------------------------------------------------------- finish: chunk records
// The row's chunk records (and their mass histograms), staged into the
// finished chunk's buffer when they fit, else read from L2 on demand.
struct RecView {
  const ChunkRec* rec;
  const float* hist;
  bool staged;
  __device__ __forceinline__ ChunkRec get(int c) const {
    if (staged) return rec[c];
    union {
      int4 v[sizeof(ChunkRec) / 16];
      ChunkRec r;
    } u;
    const int4* src = reinterpret_cast<const int4*>(rec + c);
#pragma unroll
    for (int i = 0; i < int(sizeof(ChunkRec) / 16); ++i) u.v[i] = __ldcg(src + i);
    return u.r;
  }
  // Mass below bucket threshold B1 of chunk c (histogram bins with Bc - b < B1).
  __device__ __forceinline__ double mass_below(int c, int Bc, int B1) const {
    const float4* h = reinterpret_cast<const float4*>(hist + size_t(c) * kBins);
    double m = 0.0;
#pragma unroll
    for (int q = 0; q < kBins / 4; ++q) {
      const float4 f = staged ? h[q] : __ldcg(h + q);
      const int b = 4 * q;
      if (Bc - b < B1) m += double(f.x);
      if (Bc - b - 1 < B1) m += double(f.y);
      if (Bc - b - 2 < B1) m += double(f.z);
      if (Bc - b - 3 < B1) m += double(f.w);
    }
    return m;
  }
};

__device__ __forceinline__ RecView stage_records(const Params& P, unsigned char* scratch, int row, bool with_hist) {
  const int NC = P.nc;
  const size_t rb = size_t(NC) * sizeof(ChunkRec);
  const size_t hb = with_hist ? size_t(NC) * kBins * sizeof(float) : 0;
  const ChunkRec* grec = P.rec + size_t(row) * size_t(NC);
  const float* ghist = P.hist + size_t(row) * size_t(NC) * kBins;
  RecView v{grec, ghist, false};
  if (rb + hb <= size_t(kBufBytes)) {
    int4* d = reinterpret_cast<int4*>(scratch);
    const int4* src = reinterpret_cast<const int4*>(grec);
    for (int i = threadIdx.x; i < int(rb / 16); i += kThreads) d[i] = __ldcg(src + i);
    if (with_hist) {
      int4* dh = reinterpret_cast<int4*>(scratch + rb);
      const int4* sh = reinterpret_cast<const int4*>(ghist);
      for (int i = threadIdx.x; i < int(hb / 16); i += kThreads) dh[i] = __ldcg(sh + i);
    }
    v.rec = reinterpret_cast<const ChunkRec*>(scratch);
    v.hist = reinterpret_cast<const float*>(scratch + rb);
    v.staged = true;
  }
  csync();
  return v;
}

// The k-th largest (1-based) high word of keys[0..n), by an 8-bit radix
// select over shared memory (compute warps).
__device__ __forceinline__ uint32_t radix_kth(Smem& sm, const unsigned long long* keys, int n, int k) {
  uint32_t prefix = 0u;
  int need = k;
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int i = threadIdx.x; i < 256; i += kThreads) sm.u.h.cnt[i] = 0u;
    csync();
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint32_t v = uint32_t(keys[i] >> 32);
      if (level == 0 || (v >> (shift + 8)) == prefix) atomicAdd(&sm.u.h.cnt[(v >> shift) & 255u], 1u);
    }
    csync();
    if (threadIdx.x < 32) {
      // lane l owns bins 255 - 8l down to 248 - 8l
      const int lane = threadIdx.x;
      unsigned c[8];
      unsigned tot = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sm.u.h.cnt[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned excl = incl - tot;
      if (excl < unsigned(need) && unsigned(need) <= incl) {
        unsigned run = excl;
        int bin = -1;
        unsigned left = 0u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (bin < 0 && run + c[j] >= unsigned(need)) {
            bin = 255 - 8 * lane - j;
            left = unsigned(need) - run;
          }
          run += c[j];
        }
        sm.bcast_pre = ((long long)bin << 32) | (long long)left;
      }
    }
    csync();
    const long long bb = sm.bcast_pre;
    const uint32_t d = uint32_t(bb >> 32);
    need = int(bb & 0xFFFFFFFFll);
    prefix = level == 0 ? d : ((prefix << 8) | d);
    csync();
  }
  return prefix;
}

template <typename T>
__device__ __forceinline__ void finish_small_k(const Params& P, Smem& sm, const RecView& R, unsigned char* scratch, int row,
                               const RowP& rp, float c0, float Sf, double S, float xmax);

template <typename T>
__device__ __forceinline__ void finish_stats(const Params& P, Smem& sm, unsigned char* scratch, int row, const RowP& rp) {
  const int tid = threadIdx.x;
  const int NC = P.nc;
  const int64_t V = P.a.vocab;
  const RecView R = stage_records(P, scratch, row, rp.kind == kKindRace && rp.p_on && !rp.k_on && !rp.exact);
  // row max (NaN-aware), the first chunk with a NaN, the first chunk holding the max
  uint32_t kmax = 0u;
  int nanc = INT_MAX;
  for (int c = tid; c < NC; c += kThreads) {
    const ChunkRec rc = R.get(c);
    if (rc.flags & kFEmpty) continue;
    kmax = max(kmax, nan_key(rc.cmax));
    if (rc.flags & kFNan) nanc = min(nanc, c);
  }
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  nanc = __reduce_min_sync(0xFFFFFFFFu, nanc);
  if ((tid & 31) == 0) {
    sm.red_k[tid >> 5] = kmax;
    sm.red_i[tid >> 5] = nanc;
  }
  csync();
  kmax = 0u;
  nanc = INT_MAX;
  for (int w = 0; w < kWarps; ++w) {
    kmax = max(kmax, sm.red_k[w]);
    nanc = min(nanc, sm.red_i[w]);
  }
  csync();
  const bool rnan = nanc != INT_MAX;
  const float xmax = rnan ? __int_as_float(0x7FFFFFFF) : (kmax == 0u ? -INFINITY : key_to_float(kmax));
  const float u = __fmul_rn(xmax, rp.c1);
  // first chunk holding the max, and the sum S in the row scale
  int gc = INT_MAX;
  double part = 0.0;
  for (int c = tid; c < NC; c += kThreads) {
    const ChunkRec rc = R.get(c);
    if (rc.flags & kFEmpty) continue;
    if (!rnan && rc.cmax == xmax) gc = min(gc, c);
    if (rc.cmax > -INFINITY && rc.S > 0.0) part += rc.S * exp2_nl(double(rc.u) - double(u));
  }
  gc = __reduce_min_sync(0xFFFFFFFFu, gc);
  if ((tid & 31) == 0) sm.red_i[tid >> 5] = gc;
  const double Ssum = cta_sum_d(sm, part);   // its barriers also publish red_i
  gc = INT_MAX;
  for (int w = 0; w < kWarps; ++w) gc = min(gc, sm.red_i[w]);
  if (rnan) gc = nanc;
  const long long greedy = gc < NC ? (long long)R.get(gc).greedy : 0;
  if (row_timed_out(P, row)) {
    complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
    return;
  }
  if (rp.kind == kKindGreedy) {
    complete_row(P, row, greedy, QE_ROW_GREEDY, 0);
    return;
  }
  bool finite = !rnan && xmax > -INFINITY && xmax < INFINITY && isfinite(u);
  const double S = finite ? Ssum : 0.0;
  const float Sf = float(S);
  if (!(S > 0.0) || !(Sf < INFINITY)) finite = false;
  if (P.a.out_norm && tid == 0)
    P.a.out_norm[row] = finite ? S * exp2_nl(double(u) - double(xmax) * double(rp.c1))
                               : __longlong_as_double(0x7FF8000000000000LL);
  if (!finite) {
    complete_row(P, row, greedy, QE_ROW_NONFINITE, 0);
    return;
  }
  const float c0 = -u;
  const float thr_m = minp_threshold(rp, xmax, c0, Sf);
  if (rp.kind == kKindArgmax) {
    complete_row(P, row, greedy, 0, 1);
    return;
  }
  if (rp.exact) {
    enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  if (rp.kind == kKindSmallK) {
    finish_small_k<T>(P, sm, R, scratch, row, rp, c0, Sf, S, xmax);
    return;
  }
  // race rows: warp 0 ranks the chunks' candidates by exact row-scale ratio
  if ((tid >> 5) == 0) {
    const int lane = tid & 31;
    Top4 t;
    t.init();
    float cl = 0.f;
    for (int c = lane; c < NC; c += 32) {
      const ChunkRec rc = R.get(c);
      if (rc.flags & kFEmpty) continue;
      for (int i = 0; i < rc.ncand && i < kR; ++i) {
        const Cand cd = rc.cand[i];
        t.add(div_nl(div_nl(qe_ex2_ftz(__fmaf_rn(cd.x, rp.c1, c0)), Sf), cd.E), cd.x, cd.E, cd.id);
      }
      if (rc.ceil > 0.f) {
        // chunk-scale and row-scale exponents differ by the rounding of
        // x*c1 - u: a few ulps of |u|, plus the ratios' own rounding
        const double uc = double(rc.u);
        const double margin = 1.0 + 1.0 / 65536.0 + (fabs(uc) + fabs(double(u))) * (1.0 / 2097152.0);
        cl = fmaxf(cl, float(double(rc.ceil) * exp2_nl(uc - double(u)) / double(Sf) * margin));
      }
    }
    cl = warp_max(cl);
    int head = 0, n = 0;
#pragma unroll 1
    for (int round = 0; round < kTC; ++round) {
      const Cand h = t.at(head);
      const uint32_t kr = h.r >= 0.f ? __float_as_uint(h.r) + 1u : 0u;
      const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
      if (km == 0u) break;
      const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(h.id) : 0xFFFFFFFFu);
      const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(h.id) == im)) - 1;
      if (lane == src) {
        sm.tc[round] = h;
        ++head;
      }
      ++n;
    }
    if (lane == 0) {
      sm.ntc = n;
      sm.cceil = cl;
    }
  }
  csync();
  const float ceil_row = sm.cceil;
  Top4 top;
  top.init();
  for (int i = 0; i < sm.ntc; ++i) {
    const Cand c = sm.tc[i];
    top.add(c.r, c.x, c.E, c.id);
  }
  int ncomp = 0;
  for (int i = 0; i < kTC; ++i) {
    if (top.r[i] >= 0.f && top.r[i] > ceil_row) ncomp = i + 1;
    else break;
  }
  if (!rp.filtered) {
    if (ncomp > 0) complete_row(P, row, top.id[0], 0, V);
    else enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  // candidates below the min-p threshold are outside the kept set
  float xs[kTC];
  int ids[kTC];
  int m = 0;
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    xs[i] = 0.f;
    ids[i] = INT_MAX;
  }
#pragma unroll
  for (int i = 0; i < kTC; ++i) {
    if (i >= ncomp) break;
    if (rp.m_on && __fdiv_rn(qe_ex2_ftz(__fmaf_rn(top.x[i], rp.c1, c0)), Sf) < thr_m) continue;
#pragma unroll
    for (int j = 0; j < kTC; ++j)
      if (j == m) {
        xs[j] = top.x[i];
        ids[j] = top.id[i];
      }
    ++m;
  }
  if (m == 0) {
    enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  if (!rp.p_on && !rp.k_on) {
    complete_row(P, row, ids[0], 0, 0);
    return;
  }
  if (rp.p_on && !rp.k_on) {
    // proof from the chunks' group-mass histograms: a group whose max lies
    // below the candidate's logit is entirely behind it
    const float u1 = __fmul_rn(xs[0], rp.c1);
    const int B1 = __float2int_rd(fminf(fmaxf(2.f * u1, -1.0e9f), 1.0e9f));
    double L = 0.0;
    for (int c = tid; c < NC; c += kThreads) {
      const ChunkRec rc = R.get(c);
      if ((rc.flags & kFEmpty) || !(rc.cmax > -INFINITY)) continue;
      const int Bc = __float2int_rd(fminf(fmaxf(2.f * rc.u, -1.0e9f), 1.0e9f));
      L += R.mass_below(c, Bc, B1) * exp2_nl(double(rc.u) - double(u)) *
           (1.0 - 1e-6 - (fabs(double(rc.u)) + fabs(double(u))) * (1.0 / 2097152.0));
    }
    L = cta_sum_d(sm, L);
    const double ec = double(qe_ex2_ftz(__fmaf_rn(xs[0], rp.c1, c0)));
    if (S - ec * (1.0 - 1e-6) - L <= double(rp.tp) * S - S * (1.0 / 262144.0)) {
      complete_row(P, row, ids[0], 0, 0);
      return;
    }
  }
  // test round: mass and rank ahead of each candidate
  if (tid == 0) {
    RowRound& r = sm.rr;
    r.type = kRoundTest;
    r.level = 0;
    r.prefix = 0u;
    r.m = m;
    r.c0 = c0;
    r.Sf = Sf;
    r.S = S;
    for (int i = 0; i < kTC; ++i) {
      r.xs[i] = xs[i];
      r.ids[i] = ids[i];
    }
    r.thr_m = thr_m;
  }
  csync();
  publish(P, sm, row);
}

// Small top-k rows: the union of the chunks' gathered heads holds the row's
// k largest logits.  Sort it, apply the reference's top-p rule in sorted
// order (fp64 cumsum rounded to fp32, src/compute/sampler.py:35-37) and
// min-p element by element, then race over what is kept.
template <typename T>
__device__ __forceinline__ void finish_small_k(const Params& P, Smem& sm, const RecView& R, unsigned char* scratch, int row,
                               const RowP& rp, float c0, float Sf, double S, float xmax) {
  const int tid = threadIdx.x;
  const int NC = P.nc;
  const int64_t V = P.a.vocab;
  const float thr_m = minp_threshold(rp, xmax, c0, Sf);
  int over = 0;
  for (int c = tid; c < NC; c += kThreads)
    if (R.get(c).flags & kFOver) over = 1;
  if (tid == 0) sm.ngath = 0;
  if (csync_or(over != 0)) {
    enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  // the union of the chunks' heads (it holds the row's k largest), in the
  // chunk buffer after the staged records
  const size_t roff = R.staged ? (size_t(NC) * sizeof(ChunkRec) + 15) / 16 * 16 : 0;
  unsigned long long* uk = reinterpret_cast<unsigned long long*>(scratch + roff);
  const int ucap = int((size_t(kBufBytes) - roff) / sizeof(unsigned long long));
  const GItem* gsrc = P.gather + size_t(row) * size_t(NC) * kGCap;
  for (int c = 0; c < NC; ++c) {
    const int ng = R.get(c).ngather;
    for (int i = tid; i < ng; i += kThreads) {
      const long long raw = __ldcg(reinterpret_cast<const long long*>(gsrc + size_t(c) * kGCap + i));
      const float x = __int_as_float(int(raw & 0xFFFFFFFFll));
      const int id = int(raw >> 32);
      const int at = atomicAdd(&sm.ngath, 1);
      if (at < ucap)
        uk[at] = (static_cast<unsigned long long>(ordered_key(x)) << 32) |
                 static_cast<unsigned long long>(0xFFFFFFFFu - uint32_t(id));
    }
  }
  csync();
  const int nu = sm.ngath;
  if (nu > ucap || nu < int(rp.k)) {
    csync();
    enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  // every union key at or above the k-th largest logit
  const uint32_t tk = radix_kth(sm, uk, nu, int(rp.k));
  if (tid == 0) sm.ngath = 0;
  csync();
  for (int i = tid; i < nu; i += kThreads) {
    const unsigned long long key = uk[i];
    if (uint32_t(key >> 32) < tk) continue;
    const int at = atomicAdd(&sm.ngath, 1);
    if (at < kSortCap) sm.u.keys[at] = key;
  }
  csync();
  const int n = sm.ngath;
  if (n > kSortCap || n < 1) {
    csync();
    enter_exact(P, sm, row, rp, c0, Sf, S, thr_m);
    return;
  }
  int N = 2;
  while (N < n) N <<= 1;
  for (int i = n + tid; i < N; i += kThreads) sm.u.keys[i] = 0ull;
  csync();
  // bitonic sort, descending
  for (int k = 2; k <= N; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < N; i += kThreads) {
        const int p = i ^ j;
        if (p > i) {
          const unsigned long long a = sm.u.keys[i], b = sm.u.keys[p];
          const bool desc = (i & k) == 0;
          if (desc ? a < b : a > b) {
            sm.u.keys[i] = b;
            sm.u.keys[p] = a;
          }
        }
      }
      csync();
    }
  }
  const int nk = int(rp.k < (long long)n ? rp.k : (long long)n);
  const unsigned long long mykey = tid < nk ? sm.u.keys[tid] : 0ull;
  csync();
  const float xi = key_to_float(uint32_t(mykey >> 32));
  const int idi = int(0xFFFFFFFFu - uint32_t(mykey & 0xFFFFFFFFull));
  const float pi = tid < nk ? __fdiv_rn(qe_ex2_ftz(__fmaf_rn(xi, rp.c1, c0)), Sf) : 0.f;
  if (tid < nk) sm.u.sk.rho[tid] = pi;
  csync();
  if (tid == 0) {
    double cum = 0.0;
    int kept = 0;
    for (int i = 0; i < nk; ++i) {
      const float p = sm.u.sk.rho[i];
      cum += double(p);
      const float cs = float(cum);
      bool rem = rp.p_on && __fsub_rn(cs, p) > rp.tp;
      rem = rem || (rp.m_on && p < thr_m);
      sm.u.sk.keep[i] = rem ? 0 : 1;
      kept += rem ? 0 : 1;
    }
    sm.ngath = kept;
  }
  csync();
  // race over the kept heads
  float rho = -1.f;
  int rid = INT_MAX;
  if (tid < nk && sm.u.sk.keep[tid]) {
    float E;
    if (P.a.noise) {
      E = __ldg(P.a.noise + size_t(row) * size_t(P.a.noise_ld) + size_t(idi));
    } else {
      const NoiseKey key = row_key(P, row);
      const NoiseRoot rt = noise_root(key, V);
      int64_t gs = -1;
      int ms = 0;
      token_group(rt.s, V, &gs, &ms);
      E = tree_noise(key, rt, gs, ms, idi, V);
    }
    rho = __fdiv_rn(pi, E);
    rid = idi;
  }
  const long long kept = sm.ngath;
  const uint32_t kr = rho >= 0.f ? __float_as_uint(rho) + 1u : 0u;
  const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
  const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(rid) : 0xFFFFFFFFu);
  if ((tid & 31) == 0) {
    sm.red_k[tid >> 5] = km;
    sm.red_i[tid >> 5] = int(im);
  }
  csync();
  if (tid == 0) {
    uint32_t bk = 0u;
    int bid = INT_MAX;
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t k = sm.red_k[w];
      const int i = sm.red_i[w];
      if (k > bk || (k == bk && k != 0u && i < bid)) {
        bk = k;
        bid = i;
      }
    }
    sm.red_greedy = bk ? bid : -1;
  }
  csync();
  complete_row(P, row, sm.red_greedy, QE_ROW_GATHERED, kept);
}

// ---------------------------------------------------------------- chunk item
// Warp-level append of finalist codes to the warp's list.
__device__ __forceinline__ void wappend(uint16_t* fq, int& nf, bool pred, uint32_t code, float hi, float& lc) {
  const unsigned m = __ballot_sync(0xFFFFFFFFu, pred);
  if (pred) {
    const int pos = nf + __popc(m & ((1u << (threadIdx.x & 31)) - 1u));
    if (pos < kFW) fq[pos] = uint16_t(code);
    else lc = fmaxf(lc, hi);   // not evaluated: the ceiling keeps the record honest
  }
  nf += __popc(m);
}

// Warp-local race over the warp's two tiles (groups (tile, lane) for
// tile = warp, warp + kWarps) in the warp's own scale c0s, with the same
// bounds-first scheme as race_philox: leaves the warp's R best (ratios in
// that scale) in sm.wl[warp] and a ceiling over its other tokens in
// sm.wceil[warp].  No CTA barrier.
template <typename T>
__device__ __forceinline__ void race_warp(const Params& P, Smem& sm, const unsigned char* buf, const Geo& g,
                                          const RowP& rp, float c0s, int R, const G1 sl[2], float e_root,
                                          long long s_gid, int s_mem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const NoiseKey key = row_key(P, g.row);
  const float c1 = rp.c1;
  if (lane == 0) {
    for (int i = 0; i < R; ++i) sm.wl[warp][i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
    sm.wceil[warp] = 0.f;
  }
  // A: bounds for the lane's two groups
  float alo[2], ahi[2], blo[2], bhi[2], ob[2], el2[2];
  int ag[2], ag2[2], nn[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    alo[s] = ahi[s] = blo[s] = bhi[s] = ob[s] = -1.f;
    el2[s] = 1.f;
    ag[s] = ag2[s] = nn[s] = 0;
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles) continue;
    const int lg = tile * 32 + lane;
    const float gm = sl[s].gmax;
    const int n = gsize(g.len, tile, lane);
    nn[s] = n;
    if (n <= 0 || !(gm > -INFINITY)) continue;
    const long long gid = g.gbase + lg;
    const U4 w = philox_at(key, uint32_t(gid), kTagGroup);
    const bool holds = gid == s_gid;
    const int a = arg_of(w, n, holds, s_mem);
    float lo1 = e_root, hi1 = e_root;
    if (!holds) {
      const float la = -lg2_approx(uniform_open(w.x)) * 0.6931472f;
      const float inv = 1.f / float(n);
      lo1 = (e_root + fmaxf(0.f, la * (1.f - 3e-5f) - 3e-5f) * inv) * (1.f - 2e-6f);
      hi1 = (e_root + (la * (1.f + 3e-5f) + 3e-5f) * inv) * (1.f + 2e-6f);
    }
    ag[s] = a;
    const float ea = qe_ex2_ftz(__fmaf_rn(xval<T>(sm, buf, rp, tile, lane, a), c1, c0s));
    alo[s] = __fdividef(ea, hi1) * (1.f - 1e-5f);
    ahi[s] = __fdividef(ea, lo1) * (1.f + 1e-5f);
    if (n >= 2) {
      const float lz = -lg2_approx(uniform_open(w.z)) * 0.6931472f;
      const float inv1 = 1.f / float(n - 1);
      const float lo2 = (lo1 + fmaxf(0.f, lz * (1.f - 3e-5f) - 3e-5f) * inv1) * (1.f - 2e-6f);
      const float hi2 = (hi1 + (lz * (1.f + 3e-5f) + 3e-5f) * inv1) * (1.f + 2e-6f);
      const int a2 = arg2_of(w, n, a);
      ag2[s] = a2;
      el2[s] = lo2;
      const float eb = qe_ex2_ftz(__fmaf_rn(xval<T>(sm, buf, rp, tile, lane, a2), c1, c0s));
      blo[s] = __fdividef(eb, hi2) * (1.f - 1e-5f);
      bhi[s] = __fdividef(eb, lo2) * (1.f + 1e-5f);
      if (n >= 3) ob[s] = __fdividef(qe_ex2_ftz(__fmaf_rn(gm, c1, c0s)), lo2) * (1.f + 1e-5f);
    }
  }
  // threshold: the warp's R-th largest lower bound
  float theta = -1.f;
  {
    float v0 = alo[0], v1 = blo[0], v2 = alo[1], v3 = blo[1];
    for (int round = 0; round < R; ++round) {
      const float m = fmaxf(fmaxf(v0, v1), fmaxf(v2, v3));
      const float wm = warp_max(m);
      theta = wm;
      const unsigned bal = __ballot_sync(0xFFFFFFFFu, m == wm);
      if (lane == __ffs(bal) - 1) {
        if (v0 == wm) v0 = -1.f;
        else if (v1 == wm) v1 = -1.f;
        else if (v2 == wm) v2 = -1.f;
        else v3 = -1.f;
      }
    }
  }
  // B: finalists and expansions
  uint16_t* fq = sm.fqw[warp];
  int nf = 0;
  float lc = 0.f;
  bool ex[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const uint32_t lg = uint32_t((warp + kWarps * s) * 32 + lane);
    const bool pa = ahi[s] >= 0.f && ahi[s] >= theta, pb = bhi[s] >= 0.f && bhi[s] >= theta;
    if (ahi[s] >= 0.f && !pa) lc = fmaxf(lc, ahi[s]);
    if (bhi[s] >= 0.f && !pb) lc = fmaxf(lc, bhi[s]);
    wappend(fq, nf, pa, uint32_t(kFinA << 14) | (lg << 5), ahi[s], lc);
    wappend(fq, nf, pb, uint32_t(kFinB << 14) | (lg << 5), bhi[s], lc);
    ex[s] = ob[s] >= 0.f && ob[s] >= theta;
    if (ob[s] >= 0.f && !ex[s]) lc = fmaxf(lc, ob[s]);
  }
  // C: expansions, one group at a time, lanes over its members
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    unsigned em = __ballot_sync(0xFFFFFFFFu, ex[s]);
    while (em) {
      const int src = __ffs(em) - 1;
      em &= em - 1u;
      const int tile = warp + kWarps * s;
      const int n = __shfl_sync(0xFFFFFFFFu, nn[s], src);
      const int a = __shfl_sync(0xFFFFFFFFu, ag[s], src), a2 = __shfl_sync(0xFFFFFFFFu, ag2[s], src);
      const float e2lo = __shfl_sync(0xFFFFFFFFu, el2[s], src);
      const int m = lane;
      bool pm = false;
      float bm = 0.f;
      if (m < n && m != a && m != a2) {
        bm = __fdividef(qe_ex2_ftz(__fmaf_rn(xval<T>(sm, buf, rp, tile, src, m), c1, c0s)), e2lo) * (1.f + 1e-5f);
        pm = bm >= theta;
        if (!pm) lc = fmaxf(lc, bm);
      }
      wappend(fq, nf, pm, uint32_t(kFinT << 14) | uint32_t((tile * 32 + src) << 5) | uint32_t(m), bm, lc);
    }
  }
  __syncwarp();
  // D: exact noise for the finalists
  const int nfc = min(nf, kFW);
  for (int base = 0; base < nfc; base += 32) {
    const int e = base + lane;
    Cand c{-1.f, 0.f, 1.f, INT_MAX};
    if (e < nfc) c = finalist<T>(sm, buf, g, rp, key, c0s, fq[e]);
    warp_offer(sm.wl[warp], &sm.wceil[warp], R, c.r, c.x, c.E, c.id);
  }
  raise_ceiling(sm, lc);
}

// Caller-noise version (parity mode): dense over the warp's tokens.
template <typename T>
__device__ __forceinline__ void race_noise_warp(const Params& P, Smem& sm, const unsigned char* buf, const Geo& g,
                                                const RowP& rp, float c0s, int R, const G1 sl[2]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float c1 = rp.c1;
  if (lane == 0) {
    for (int i = 0; i < R; ++i) sm.wl[warp][i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
    sm.wceil[warp] = 0.f;
  }
  Top4 best;
  best.init();
  float lc = 0.f;
  const float* nz = P.a.noise + size_t(g.row) * size_t(P.a.noise_ld) + size_t(g.start);
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles || !(sl[s].gmax > -INFINITY)) continue;
    const int n = gsize(g.len, tile, lane);
#pragma unroll 1
    for (int m = 0; m < n; ++m) {
      const int o = moff(tile, lane, m);
      const float x = xval<T>(sm, buf, rp, tile, lane, m);
      const float ev = qe_ex2_ftz(__fmaf_rn(x, c1, c0s));
      const float E = __ldg(nz + o);
      const float ap = __fdividef(ev, E) * (1.f + 1e-5f);
      if (!(ap >= best.r[kTC - 1])) {
        lc = fmaxf(lc, ap);
        continue;
      }
      const float r = div_nl(ev, E);
      if (best.r[kTC - 1] >= 0.f && !rbetter(r, int(g.start + o), best.r[kTC - 1], best.id[kTC - 1])) {
        lc = fmaxf(lc, r);
        continue;
      }
      if (best.r[kTC - 1] >= 0.f) lc = fmaxf(lc, best.r[kTC - 1]);
      best.add(r, x, E, int(g.start + o));
    }
  }
#pragma unroll
  for (int i = 0; i < kTC; ++i) warp_offer(sm.wl[warp], &sm.wceil[warp], R, best.r[i], best.x[i], best.E[i], best.id[i]);
  raise_ceiling(sm, lc);
}

template <typename T>
__device__ __forceinline__ void do_chunk(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk,
                                         const RowP& rp, bool tmo, float e_root, long long s_gid, int s_mem) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  ChunkRec* rec = P.rec + size_t(g.row) * size_t(P.nc) + size_t(g.chunk);
  if (tmo || g.len <= 0) {
    if (tmo) mark_timeout(P, g.row);
    if (tid == 0) {
      ChunkRec r;
      r.cmax = -INFINITY;
      r.u = 0.f;
      r.greedy = INT_MAX;
      r.flags = kFEmpty;
      r.S = 0.0;
      r.ceil = 0.f;
      r.ncand = 0;
      r.lk = -INFINITY;
      r.ngather = 0;
      for (int i = 0; i < kR; ++i) r.cand[i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
      *rec = r;
    }
    return;
  }
  const bool race_row = rp.kind == kKindRace && !rp.exact;
  const bool smallk = rp.kind == kKindSmallK && !rp.exact;
  const bool sum = rp.kind != kKindGreedy;
  const int R = rp.filtered ? kR : 1;
  // tail beyond the bulk copy, padding, repetition-penalty bits
  const bool pad = bulk < g.ntiles * kTile;
  if (pad) fill_chunk<T>(P, buf, g, bulk);
  if (rp.pen) build_pen(sm, g, rp);
  else if (pad) csync();
  // pass 1 and the race, warp by warp in each warp's own scale
  G1 sl[2];
  uint32_t wkey = 0u;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    sl[s] = G1{-INFINITY, 0.f};
    const int tile = warp + kWarps * s;
    if (tile < g.ntiles) {
      sl[s] = pass1<T>(sm, buf, rp, tile, lane, sum);
      wkey = max(wkey, nan_key(sl[s].gmax));
    }
  }
  wkey = __reduce_max_sync(0xFFFFFFFFu, wkey);
  const float wmax = wkey == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : (wkey == 0u ? -INFINITY : key_to_float(wkey));
  const float uw = sum ? __fmul_rn(wmax, rp.c1) : 0.f;
  const bool wfin = sum && wmax == wmax && wmax > -INFINITY && wmax < INFINITY && isfinite(uw);
  const bool hist = race_row && rp.p_on && !rp.k_on;
  double sw = 0.0;
  if (wfin) {
    if (hist) {
      sm.phist[warp][lane] = 0u;
      sm.phist[warp][lane + 32] = 0u;
      __syncwarp();
    }
    const int Bw = __float2int_rd(fminf(fmaxf(2.f * uw, -1.0e9f), 1.0e9f));
    float part = 0.f;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (warp + kWarps * s >= g.ntiles || !(sl[s].gmax > -INFINITY)) continue;
      const float ug = __fmul_rn(sl[s].gmax, rp.c1);
      const float term = sl[s].fsum * qe_ex2_ftz(__fsub_rn(ug, uw));
      part += term;
      if (hist) {
        const int bg = __float2int_rd(fminf(fmaxf(2.f * ug, -1.0e9f), 1.0e9f));
        atomicAdd(&sm.phist[warp][min(kBins - 1, max(0, Bw - bg))], __float2uint_rd(term * 1048576.f));
      }
    }
    sw = double(part);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sw += __shfl_xor_sync(0xFFFFFFFFu, sw, o);
    if (race_row) {
      if (P.a.noise) race_noise_warp<T>(P, sm, buf, g, rp, -uw, R, sl);
      else race_warp<T>(P, sm, buf, g, rp, -uw, R, sl, e_root, s_gid, s_mem);
    }
  } else if (race_row && lane == 0) {
    for (int i = 0; i < R; ++i) sm.wl[warp][i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
    sm.wceil[warp] = 0.f;
  }
  if (lane == 0) {
    sm.wr_key[warp] = wkey;
    sm.wr_u[warp] = uw;
    sm.wr_S[warp] = wfin ? sw : 0.0;
  }
  csync();
  // chunk max, its anchor, and what needs the whole CTA
  uint32_t ckey = 0u;
  for (int w = 0; w < kWarps; ++w) ckey = max(ckey, sm.wr_key[w]);
  const float cmax = ckey == 0xFFFFFFFFu ? __int_as_float(0x7FFFFFFF) : (ckey == 0u ? -INFINITY : key_to_float(ckey));
  const float u = sum ? __fmul_rn(cmax, rp.c1) : 0.f;
  const bool fin = sum && cmax == cmax && cmax > -INFINITY && cmax < INFINITY && isfinite(u);
  int greedy = INT_MAX;
  // the first id of the chunk max matters only to greedy rows and to rows
  // that turn out not finite (a non-finite row's max chunk is not finite)
  if (!fin || rp.kind == kKindArgmax) greedy = chunk_greedy<T>(sm, buf, g, rp, sl, cmax);
  int ng = 0;
  float lk = -INFINITY;
  uint32_t flags = cmax != cmax ? kFNan : 0u;
  if (smallk && fin) {
    gather_head<T>(sm, buf, g, rp, sl);
    ng = min(sm.ngath, kGCap);
    lk = sm.lk;
    if (sm.over) flags |= kFOver;
    GItem* dst = P.gather + (size_t(g.row) * size_t(P.nc) + size_t(g.chunk)) * kGCap;
    for (int i = tid; i < ng; i += kThreads) dst[i] = sm.gl[i];
  }
  if (warp != 0) return;
  // warp 0: merge the warps into the chunk record (rescaled to the chunk's anchor)
  double S = 0.0;
  float cl = 0.f;
  int ncand = 0;
  Cand out[kR];
#pragma unroll
  for (int i = 0; i < kR; ++i) out[i] = Cand{-1.f, 0.f, 1.f, INT_MAX};
  if (fin) {
    if (lane < kWarps) {
      const float ul = sm.wr_u[lane];
      const double sl_ = sm.wr_S[lane];
      const double sc = sl_ > 0.0 ? sl_ * double(qe_ex2_ftz(__fsub_rn(ul, u))) : 0.0;
      S = sc;
      if (race_row) {
        const float wc = sm.wceil[lane];
        if (wc > 0.f) {
          const double margin = 1.0 + 1.0 / 65536.0 + (fabs(double(ul)) + fabs(double(u))) * (1.0 / 2097152.0);
          cl = float(double(wc) * double(qe_ex2_ftz(__fsub_rn(ul, u))) * margin);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xFFFFFFFFu, S, o);
    if (race_row) {
      // each warp's candidates, re-ranked by their exact chunk-scale ratio
      Cand c{-1.f, 0.f, 1.f, INT_MAX};
      if (lane < kWarps * R) {
        const Cand w = sm.wl[lane / R][lane % R];
        if (w.r >= 0.f) c = Cand{div_nl(qe_ex2_ftz(__fmaf_rn(w.x, rp.c1, -u)), w.E), w.x, w.E, w.id};
      }
      uint32_t kr = c.r >= 0.f ? __float_as_uint(c.r) + 1u : 0u;
#pragma unroll
      for (int i = 0; i < kR; ++i) {
        if (i >= R) break;
        const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
        if (km == 0u) break;
        const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(c.id) : 0xFFFFFFFFu);
        const int src = __ffs(__ballot_sync(0xFFFFFFFFu, kr == km && uint32_t(c.id) == im)) - 1;
        out[i] = Cand{__shfl_sync(0xFFFFFFFFu, c.r, src), __shfl_sync(0xFFFFFFFFu, c.x, src),
                      __shfl_sync(0xFFFFFFFFu, c.E, src), int(im)};
        if (lane == src) kr = 0u;
        ++ncand;
      }
      if (kr) cl = fmaxf(cl, c.r);
      cl = warp_max(cl);
    }
    if (hist) {
      // chunk bins from the warps' bins: shift each by its anchor difference
      // and rescale its mass to the chunk's anchor, rounding down (the bins
      // are lower bounds)
      const int Bc = __float2int_rd(fminf(fmaxf(2.f * u, -1.0e9f), 1.0e9f));
      float* hb = P.hist + (size_t(g.row) * size_t(P.nc) + size_t(g.chunk)) * kBins;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = lane + 32 * h;
        double q = 0.0;
        for (int w = 0; w < kWarps; ++w) {
          if (sm.wr_S[w] <= 0.0) continue;
          const float uwl = sm.wr_u[w];
          const int sh = Bc - __float2int_rd(fminf(fmaxf(2.f * uwl, -1.0e9f), 1.0e9f));
          unsigned long long qw = 0ull;
          if (j < kBins - 1) {
            const int b = j - sh;
            if (b >= 0) qw = sm.phist[w][b];
          } else {
            for (int b = max(0, kBins - 1 - sh); b < kBins; ++b) qw += sm.phist[w][b];
          }
          if (qw)
            q += double(qw) * double(qe_ex2_ftz(__fsub_rn(uwl, u))) *
                 (1.0 - 1.0 / 65536.0 - (fabs(double(uwl)) + fabs(double(u))) * (1.0 / 2097152.0));
        }
        hb[j] = __double2float_rd(q * (1.0 / 1048576.0));
      }
    }
  }
  if (lane == 0) {
    ChunkRec r;
    r.cmax = cmax;
    r.u = u;
    r.greedy = greedy;
    r.flags = flags;
    r.S = S;
    r.ceil = cl;
    r.ncand = ncand;
    r.lk = lk;
    r.ngather = ng;
    for (int i = 0; i < kR; ++i) r.cand[i] = out[i];
    *rec = r;
  }
}

// ---------------------------------------------------------------- test round
template <typename T>
__device__ __forceinline__ void finish_test(const Params& P, Smem& sm, int row, const RowP& rp) {
  const int NC = P.nc;
  double ms[kTC] = {0.0, 0.0, 0.0, 0.0};
  long long ct[kTC] = {0, 0, 0, 0};
  for (int c = threadIdx.x; c < NC; c += kThreads) {
    const Part* q = P.part + size_t(row) * size_t(NC) + size_t(c);
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      ms[i] += __ldcg(&q->mass[i]);
      ct[i] += __ldcg(&q->cnt[i]);
    }
  }
  cta_part(sm, ms, ct);
  if (row_timed_out(P, row)) {
    complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
    return;
  }
  const RowRound& rr = sm.rr;
  int win = -1;
  for (int i = 0; i < rr.m; ++i) {
    const bool in_k = (!rp.k_on || ct[i] < rp.k) && (!rp.p_on || ms[i] <= double(rp.tp) * rr.S);
    if (in_k) {
      win = i;
      break;
    }
  }
  if (win >= 0) complete_row(P, row, rr.ids[win], 0, 0);
  else enter_exact(P, sm, row, rp, rr.c0, rr.Sf, rr.S, rr.thr_m);
}

template <typename T>
__device__ __forceinline__ void do_test(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk, const RowP& rp,
                        bool tmo) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const RowRound& rr = sm.rr;
  double ms[kTC] = {0.0, 0.0, 0.0, 0.0};
  long long ct[kTC] = {0, 0, 0, 0};
  if (tmo) {
    mark_timeout(P, g.row);
  } else if (g.len > 0) {
    load_chunk<T>(P, sm, buf, g, bulk, rp);
    const int m = rr.m;
    float xs[kTC];
    int ids[kTC];
    float xlo = INFINITY;
#pragma unroll
    for (int i = 0; i < kTC; ++i) {
      xs[i] = i < m ? rr.xs[i] : INFINITY;
      ids[i] = i < m ? rr.ids[i] : -1;
      xlo = fminf(xlo, xs[i]);
    }
    const float c0 = rr.c0, c1 = rp.c1;
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
      const int tile = warp + kWarps * s;
      if (tile >= g.ntiles) continue;
      const G1 gg = pass1<T>(sm, buf, rp, tile, lane, false);
      if (!(gg.gmax >= xlo)) continue;
      const int n = gsize(g.len, tile, lane);
      for (int mm = 0; mm < n; ++mm) {
        const float x = xval<T>(sm, buf, rp, tile, lane, mm);
        if (!(x >= xlo)) continue;
        const double e = double(qe_ex2_ftz(__fmaf_rn(x, c1, c0)));
        const int id = int(g.start + moff(tile, lane, mm));
#pragma unroll
        for (int i = 0; i < kTC; ++i) {
          if (x > xs[i] || (x == xs[i] && id < ids[i])) {
            ms[i] += e;
            ct[i] += 1;
          }
        }
      }
    }
  }
  cta_part(sm, ms, ct);
  if (threadIdx.x == 0) {
    Part* q = P.part + size_t(g.row) * size_t(P.nc) + size_t(g.chunk);
    for (int i = 0; i < kTC; ++i) {
      q->mass[i] = ms[i];
      q->cnt[i] = ct[i];
    }
  }
}

// ---------------------------------------------------------------- exact rounds: radix histogram
template <typename T>
__device__ __forceinline__ void finish_hist(const Params& P, Smem& sm, int row, const RowP& rp) {
  const int tid = threadIdx.x;
  HistAcc* h = P.hacc + row;
  for (int i = tid; i < 256; i += kThreads) {
    sm.u.h.cnt[i] = __ldcg(&h->cnt[i]);
    sm.u.h.mass[i] = __ldcg(&h->mass[i]);
  }
  if (tid == 0) sm.u.h.nm = __ldcg(&h->nm);
  csync();
  if (row_timed_out(P, row)) {
    complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
    return;
  }
  if (tid == 0) {
    RowRound& r = sm.rr;
    const int L = r.level;
    if (L == 0) {
      unsigned long long sf = 0ull;
      for (int b = 0; b < 256; ++b) sf += sm.u.h.mass[b];
      r.sfix = sf;
      r.tfix = rp.p_on ? static_cast<unsigned long long>(floor(double(rp.tp) * double(sf))) : ~0ull;
      long long kk = rp.k;
      if (rp.m_on) kk = min(kk, (long long)sm.u.h.nm);
      r.kk = kk;
    }
    long long acnt = r.acnt;
    unsigned long long amass = r.amass;
    int d = -1;
    for (int b = 255; b >= 0; --b) {
      const long long c = sm.u.h.cnt[b];
      const unsigned long long ms = sm.u.h.mass[b];
      if (acnt + c > r.kk || amass + ms > r.tfix) {
        d = b;
        break;
      }
      acnt += c;
      amass += ms;
    }
    int next;
    if (d < 0) {   // every element is kept
      r.level = 3;
      r.kkey = 0u;
      r.ties_all = 1;
      r.kties = 0;
      r.nkeep = acnt;
      next = kRoundRace;
    } else {
      const uint32_t key_hi = L == 0 ? uint32_t(d) : ((r.prefix << 8) | uint32_t(d));
      if (L < final_level(P, rp)) {
        r.prefix = key_hi;
        r.level = L + 1;
        r.acnt = acnt;
        r.amass = amass;
        next = kRoundHist;
      } else {
        // key_hi fixes the value: its elements are ties of equal mass
        const int sh = 24 - 8 * L;
        const uint32_t hi = key_hi << sh;
        const uint32_t full = hi | ((hi & 0x80000000u) ? 0u : ((1u << sh) - 1u));
        const unsigned long long ed = efix(key_to_float(full), rp.c1, r.c0);
        long long t = min((long long)sm.u.h.cnt[d], r.kk - acnt);
        if (rp.p_on && ed > 0ull) {
          const unsigned long long q = (r.tfix - amass) / ed + 1ull;
          if (q < static_cast<unsigned long long>(t)) t = (long long)q;
        }
        if (t < 0) t = 0;
        r.kkey = key_hi;
        r.kties = t;
        r.ties_all = t == (long long)sm.u.h.cnt[d];
        r.nkeep = acnt + t;
        r.acnt = acnt;
        r.amass = amass;
        next = (r.ties_all || t == 0) ? kRoundRace : kRoundTies;
      }
    }
    r.type = next;
    sm.red_greedy = next;
  }
  csync();
  if (sm.red_greedy == kRoundHist) {
    for (int i = tid; i < 256; i += kThreads) {
      h->cnt[i] = 0u;
      h->mass[i] = 0ull;
    }
    if (tid == 0) h->nm = 0u;
  }
  csync();
  publish(P, sm, row);
}

template <typename T>
__device__ __forceinline__ void do_hist(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk, const RowP& rp,
                        bool tmo) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowRound& rr = sm.rr;
  for (int i = tid; i < 256; i += kThreads) {
    sm.u.h.cnt[i] = 0u;
    sm.u.h.mass[i] = 0ull;
  }
  if (tid == 0) sm.u.h.nm = 0u;
  csync();
  unsigned int nm = 0u;
  if (tmo) {
    mark_timeout(P, g.row);
  } else if (g.len > 0) {
    load_chunk<T>(P, sm, buf, g, bulk, rp);
    const int L = rr.level;
    const uint32_t pre = rr.prefix;
    const float c0 = rr.c0, c1 = rp.c1, thr = rr.thr_m, Sf = rr.Sf;
    const int shift = 24 - 8 * L;
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
      const int tile = warp + kWarps * s;
      if (tile >= g.ntiles) continue;
      const G1 gg = pass1<T>(sm, buf, rp, tile, lane, false);
      if (L > 0 && (ordered_key(gg.gmax) >> (32 - 8 * L)) < pre) continue;
      const int n = gsize(g.len, tile, lane);
      for (int mm = 0; mm < n; ++mm) {
        const float x = xval<T>(sm, buf, rp, tile, lane, mm);
        const uint32_t k = ordered_key(x);
        if (L > 0 && (k >> (32 - 8 * L)) != pre) continue;
        const int bin = int((k >> shift) & 255u);
        atomicAdd(&sm.u.h.cnt[bin], 1u);
        atomicAdd(&sm.u.h.mass[bin], efix(x, c1, c0));
        if (L == 0 && thr > 0.f && __fdiv_rn(qe_ex2_ftz(__fmaf_rn(x, c1, c0)), Sf) >= thr) ++nm;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nm += __shfl_xor_sync(0xFFFFFFFFu, nm, o);
  if (lane == 0 && nm) atomicAdd(&sm.u.h.nm, nm);
  csync();
  HistAcc* h = P.hacc + g.row;
  for (int i = tid; i < 256; i += kThreads) {
    const unsigned int c = sm.u.h.cnt[i];
    if (c) {
      atomicAdd(&h->cnt[i], c);
      atomicAdd(&h->mass[i], sm.u.h.mass[i]);
    }
  }
  if (tid == 0 && sm.u.h.nm) atomicAdd(&h->nm, sm.u.h.nm);
}

// ---------------------------------------------------------------- exact rounds: ties at the boundary
template <typename T>
__device__ __forceinline__ void finish_ties(const Params& P, Smem& sm, int row, const RowP& rp) {
  const int NC = P.nc;
  if (row_timed_out(P, row)) {
    complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
    return;
  }
  // chunk tie counts in id order -> how many of its ties each chunk keeps
  long long* cnt = reinterpret_cast<long long*>(sm.u.keys);
  for (int c0 = 0; c0 < NC; c0 += kSortCap) {
    for (int c = c0 + threadIdx.x; c < NC && c < c0 + kSortCap; c += kThreads)
      cnt[c - c0] = __ldcg(&P.part[size_t(row) * size_t(NC) + size_t(c)].cnt[0]);
    csync();
    if (threadIdx.x == 0) {
      long long pre = c0 == 0 ? 0 : sm.bcast_pre;
      const long long kt = sm.rr.kties;
      for (int c = c0; c < NC && c < c0 + kSortCap; ++c) {
        Part* q = P.part + size_t(row) * size_t(NC) + size_t(c);
        const long long n = cnt[c - c0];
        long long allow = kt - pre;
        allow = allow < 0 ? 0 : (allow > n ? n : allow);
        q->cnt[1] = allow;
        q->cnt[2] = n;
        pre += n;
      }
      sm.bcast_pre = pre;
    }
    csync();
  }
  if (threadIdx.x == 0) sm.rr.type = kRoundRace;
  csync();
  publish(P, sm, row);
}

template <typename T>
__device__ __forceinline__ void do_ties(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk, const RowP& rp,
                        bool tmo) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const RowRound& rr = sm.rr;
  long long cnt = 0;
  if (tmo) {
    mark_timeout(P, g.row);
  } else if (g.len > 0) {
    load_chunk<T>(P, sm, buf, g, bulk, rp);
    const int sh = 24 - 8 * rr.level;
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
      const int tile = warp + kWarps * s;
      if (tile >= g.ntiles) continue;
      const G1 gg = pass1<T>(sm, buf, rp, tile, lane, false);
      if ((ordered_key(gg.gmax) >> sh) < rr.kkey) continue;
      const int n = gsize(g.len, tile, lane);
      for (int mm = 0; mm < n; ++mm)
        if ((ordered_key(xval<T>(sm, buf, rp, tile, lane, mm)) >> sh) == rr.kkey) ++cnt;
    }
  }
  cnt = cta_sum_l(sm, cnt);
  if (threadIdx.x == 0) P.part[size_t(g.row) * size_t(P.nc) + size_t(g.chunk)].cnt[0] = cnt;
}

// Tie ranks of the chunk: bit o of bits[] marks offset o as a boundary tie;
// pre[w] counts the ties in words before w.
template <typename T>
__device__ __forceinline__ void build_ties(Smem& sm, const unsigned char* buf, const Geo& g, const RowP& rp, int sh, uint32_t kkey,
                           const G1 sl[2]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = g.ntiles * 32;
  for (int i = tid; i < nw; i += kThreads) sm.u.t.bits[i] = 0u;
  csync();
#pragma unroll 1
  for (int s = 0; s < 2; ++s) {
    const int tile = warp + kWarps * s;
    if (tile >= g.ntiles || (ordered_key(sl[s].gmax) >> sh) < kkey) continue;
    const int n = gsize(g.len, tile, lane);
    for (int mm = 0; mm < n; ++mm) {
      if ((ordered_key(xval<T>(sm, buf, rp, tile, lane, mm)) >> sh) == kkey) {
        const int o = moff(tile, lane, mm);
        atomicOr(&sm.u.t.bits[o >> 5], 1u << (o & 31));
      }
    }
  }
  csync();
  if (warp == 0) {
    const int per = (nw + 31) / 32;
    int loc = 0;
    for (int i = 0; i < per; ++i) {
      const int w = lane * per + i;
      if (w < nw) loc += __popc(sm.u.t.bits[w]);
    }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - loc;
    for (int i = 0; i < per; ++i) {
      const int w = lane * per + i;
      if (w < nw) {
        sm.u.t.pre[w] = uint32_t(run);
        run += __popc(sm.u.t.bits[w]);
      }
    }
  }
  csync();
}

// ---------------------------------------------------------------- exact rounds: race over the kept set
template <typename T>
__device__ __forceinline__ void finish_race(const Params& P, Smem& sm, int row, const RowP& rp) {
  const int tid = threadIdx.x, NC = P.nc;
  float br = -1.f;
  int bid = INT_MAX;
  for (int c = tid; c < NC; c += kThreads) {
    const Part* q = P.part + size_t(row) * size_t(NC) + size_t(c);
    const float r = float(__ldcg(&q->mass[0]));
    const int id = int(__ldcg(&q->cnt[0]));
    if (id >= 0 && r >= 0.f && rbetter(r, id, br, bid)) {
      br = r;
      bid = id;
    }
  }
  const uint32_t kr = br >= 0.f ? __float_as_uint(br) + 1u : 0u;
  const uint32_t km = __reduce_max_sync(0xFFFFFFFFu, kr);
  const uint32_t im = __reduce_min_sync(0xFFFFFFFFu, kr == km ? uint32_t(bid) : 0xFFFFFFFFu);
  if ((tid & 31) == 0) {
    sm.red_k[tid >> 5] = km;
    sm.red_i[tid >> 5] = int(im);
  }
  csync();
  if (tid == 0) {
    uint32_t bk = 0u;
    int b = INT_MAX;
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t k = sm.red_k[w];
      const int i = sm.red_i[w];
      if (k > bk || (k == bk && k != 0u && i < b)) {
        bk = k;
        b = i;
      }
    }
    sm.red_greedy = bk ? b : -1;
    if (!bk) atomicOr(&P.ctl->err, 4u);
  }
  csync();
  if (row_timed_out(P, row)) complete_row(P, row, -1, QE_ROW_TIMEOUT, 0);
  else complete_row(P, row, sm.red_greedy, QE_ROW_SLOW, sm.rr.nkeep);
}

template <typename T>
__device__ __forceinline__ void do_race_round(const Params& P, Smem& sm, unsigned char* buf, const Geo& g, int bulk, const RowP& rp,
                              bool tmo) {
  const RowRound& rr = sm.rr;
  float rho = -1.f;
  int rid = -1;
  if (tmo) {
    mark_timeout(P, g.row);
  } else if (g.len > 0) {
    load_chunk<T>(P, sm, buf, g, bulk, rp);
    Keep kp{1, 24 - 8 * rr.level, rr.kkey, rr.ties_all, 0};
    bool need_bits = false;
    if (!rr.ties_all && rr.kties > 0) {
      const Part* q = P.part + size_t(g.row) * size_t(P.nc) + size_t(g.chunk);
      const long long allow = __ldcg(&q->cnt[1]), nt = __ldcg(&q->cnt[2]);
      if (allow >= nt) {
        kp.ties_all = 1;
      } else {
        kp.allow = allow;
        need_bits = allow > 0;
      }
    }
    G1 sl[2];
    float cm;
    chunk_pass1<T>(sm, buf, g, rp, false, sl, &cm);
    if (need_bits) build_ties<T>(sm, buf, g, rp, kp.sh, kp.kkey, sl);
    race<T>(P, sm, buf, g, rp, rr.c0, 1, kp);
    if (sm.ncand > 0) {
      const Cand c = sm.cand[0];
      rho = __fdiv_rn(__fdiv_rn(qe_ex2_ftz(__fmaf_rn(c.x, rp.c1, rr.c0)), rr.Sf), c.E);
      rid = c.id;
    }
  }
  if (threadIdx.x == 0) {
    Part* q = P.part + size_t(g.row) * size_t(P.nc) + size_t(g.chunk);
    q->mass[0] = double(rho);
    q->cnt[0] = rid;
  }
}

// ---------------------------------------------------------------- work loop
__device__ __forceinline__ void copy_round(const Params& P, Smem& sm, int row) {
  static_assert(sizeof(RowRound) % 16 == 0 && sizeof(RowRound) / 16 <= kThreads, "RowRound copy");
  if (threadIdx.x < sizeof(RowRound) / 16)
    reinterpret_cast<int4*>(&sm.rr)[threadIdx.x] = __ldcg(reinterpret_cast<const int4*>(P.round + row) + threadIdx.x);
  csync();
}

// One item on the compute warps.  Returns the row whose part was filed (the
// producer turns it into an arrival), or -1.
template <typename T>
__device__ int process(const Params& P, Smem& sm, int b, int kind, bool tmo) {
  unsigned char* buf = sm.buf[b];
  const int bulk = sm.bulk_elems[b];
  const RowP& rp = sm.rowp[b];
  const int row = sm.frow[b];
  if (threadIdx.x == 0) {
    sm.e_root = sm.root_e[b];
    sm.s_gid = sm.root_gid[b];
    sm.s_mem = sm.root_mem[b];
  }
  if (kind == kItemChunk) {
    do_chunk<T>(P, sm, buf, geo_of(P, row, sm.chunk[b]), bulk, rp, tmo, sm.root_e[b], sm.root_gid[b],
                sm.root_mem[b]);
    return row;
  }
  if (kind == kItemFollow) {
    const Geo g = geo_of(P, row, sm.chunk[b]);
    copy_round(P, sm, row);
    switch (sm.rr.type) {
      case kRoundTest: do_test<T>(P, sm, buf, g, bulk, rp, tmo); break;
      case kRoundHist: do_hist<T>(P, sm, buf, g, bulk, rp, tmo); break;
      case kRoundTies: do_ties<T>(P, sm, buf, g, bulk, rp, tmo); break;
      default: do_race_round<T>(P, sm, buf, g, bulk, rp, tmo); break;
    }
    return row;
  }
  // finish the row's current round (this CTA's producer saw its last part)
  csync();
  const unsigned rt = __ldcg(&P.rowctl[row].round);
  if (rt == 0u) {
    finish_stats<T>(P, sm, buf, row, rp);
    return -1;
  }
  copy_round(P, sm, row);
  switch (sm.rr.type) {
    case kRoundTest: finish_test<T>(P, sm, row, rp); break;
    case kRoundHist: finish_hist<T>(P, sm, row, rp); break;
    case kRoundTies: finish_ties<T>(P, sm, row, rp); break;
    default: finish_race<T>(P, sm, row, rp); break;
  }
  return -1;
}

__device__ __forceinline__ unsigned int atom_add_release(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.release.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0u;
}

// Claim work: follow-up items first (they re-read chunks still in L2), then
// this CTA's next chunk item (CTA c takes chunk items c, c + grid, ...).
// Sets kind = kItemNone when there is nothing to hand out right now.
__device__ void claim(const Params& P, unsigned int& next_chunk, int& kind, int& chunk, int& row) {
  const unsigned nc = unsigned(P.nc);
  const unsigned B = unsigned(P.a.batch);
  kind = kItemNone;
  const unsigned qe = min(ld_relaxed(&P.ctl->qentries), B * unsigned(kMaxRounds));
  const unsigned long long avail = (unsigned long long)qe * nc;
  unsigned qh = ld_relaxed(&P.ctl->qhead);
  while ((unsigned long long)qh < avail) {
    const unsigned prev = atomicCAS(&P.ctl->qhead, qh, qh + 1u);
    if (prev == qh) {
      const unsigned e = qh / nc;
      unsigned v = 0u;
      for (uint32_t w = 0; w < P.polls; ++w) {
        v = ld_acquire(&P.queue[e]);
        if (v) break;
        __nanosleep(64);
      }
      if (!v) {
        atomicOr(&P.ctl->err, 1u);
        kind = kItemEnd;
        return;
      }
      kind = kItemFollow;
      row = int(v - 1u);
      chunk = int(qh % nc);
      return;
    }
    qh = prev;
  }
  if (next_chunk < P.nitems) {
    kind = kItemChunk;
    row = int(next_chunk / nc);
    chunk = int(next_chunk % nc);
    next_chunk += gridDim.x;
  }
}

// File one arrival for `row` (release) and report whether it was the last.
__device__ __forceinline__ unsigned int file_arrival(const Params& P, int row) {
  return atom_add_release(&P.rowctl[row].cnt, 1u);
}

// The producer warp (lane 0): decides each buffer's next item, prefetches
// the row's parameters and noise root, moves chunks in with bulk copies, and
// files the compute warps' parts as arrivals, so the compute warps never wait
// on a global round trip.  An arrival whose result shows the row's last part
// becomes a finish item for this CTA.
__device__ void producer(const Params& P, Smem& sm) {
  if ((threadIdx.x & 31) != 0) return;
  const unsigned nc = unsigned(P.nc);
  uint32_t eph[kNumBuf] = {0u, 0u};
  bool busy[kNumBuf] = {false, false};   // handed to the compute warps, not yet released
  int b = 0;
  unsigned int next_chunk = blockIdx.x;
  int fq_head = 0, fq_tail = 0;
  int pend_row = -1;
  unsigned int pend_old = 0u;
  uint32_t idle = 0;
  while (true) {
    // the arrival filed last round: was it the row's last part?
    if (pend_row >= 0) {
      if (pend_old == nc - 1u) {
        fence_acq_rel();
        sm.finq[fq_tail++ % kFinQ] = pend_row;
      }
      pend_row = -1;
    }
    int kind = kItemNone, chunk = 0, row = -1;
    if (fq_head != fq_tail) {
      kind = kItemFinish;
      row = sm.finq[fq_head++ % kFinQ];
    } else {
      claim(P, next_chunk, kind, chunk, row);
    }
    if (kind == kItemNone) {
      // nothing to hand out: file the parts of released buffers, then retry or end
      bool progress = false;
      for (int x = 0; x < kNumBuf; ++x) {
        if (busy[x] && mbar_test(&sm.empty[x], eph[x])) {
          eph[x] ^= 1u;
          busy[x] = false;
          const int r = sm.mail[x];
          if (r >= 0 && file_arrival(P, r) == nc - 1u) {
            fence_acq_rel();
            sm.finq[fq_tail++ % kFinQ] = r;
          }
          progress = true;
        }
      }
      if (progress || fq_head != fq_tail) continue;
      if (ld_acquire(&P.ctl->rows_done) >= unsigned(P.a.batch)) {
        kind = kItemEnd;
      } else if (++idle > P.polls) {
        atomicOr(&P.ctl->err, 1u);
        kind = kItemEnd;
      } else {
        __nanosleep(256);
        continue;
      }
    }
    idle = 0;
    // what the compute warps need, fetched before the buffer is free
    RowP rp;
    float re = 0.f;
    long long rg = -1;
    int rm = 0;
    if (kind != kItemEnd) {
      rp = row_params(P, row);
      if (!P.a.noise && kind != kItemFinish) {
        const NoiseKey key = row_key(P, row);
        const NoiseRoot rt = noise_root(key, P.a.vocab);
        re = rt.e_root;
        int64_t gs = -1;
        token_group_p(P, rt.s, &gs, &rm);
        rg = gs;
      }
    }
    if (busy[b]) {
      if (!mbar_wait(&sm.empty[b], eph[b], P.polls)) {
        atomicOr(&P.ctl->err, 1u);
        return;
      }
      eph[b] ^= 1u;
      busy[b] = false;
      const int r = sm.mail[b];
      if (r >= 0) {
        pend_old = file_arrival(P, r);   // checked next round
        pend_row = r;
      }
    }
    sm.kind[b] = kind;
    sm.chunk[b] = chunk;
    sm.frow[b] = row;
    sm.rowp[b] = rp;
    sm.root_e[b] = re;
    sm.root_gid[b] = rg;
    sm.root_mem[b] = rm;
    uint32_t bytes = 0u;
    if (kind == kItemChunk || kind == kItemFollow) {
      const Geo g = geo_of(P, row, chunk);
      if (P.tma_ok && g.len > 0) bytes = uint32_t(g.len * P.esize) & ~15u;
      sm.bulk_elems[b] = int(bytes / uint32_t(P.esize));
      if (bytes) {
        const unsigned char* src = static_cast<const unsigned char*>(P.a.logits) +
                                   (size_t(row) * size_t(P.a.ld) + size_t(g.start)) * size_t(P.esize);
        fence_proxy_async();
        mbar_expect_tx(&sm.full[b], bytes);
        bulk_g2s(sm.buf[b], src, bytes, &sm.full[b]);
      }
    } else {
      sm.bulk_elems[b] = 0;
    }
    if (!bytes) mbar_arrive(&sm.full[b]);
    if (kind == kItemEnd) return;
    busy[b] = true;
    b ^= 1;
  }
}

template <typename T>
__device__ void consumer(const Params& P, Smem& sm) {
  uint32_t fph[kNumBuf] = {0u, 0u};
  int b = 0;
  while (true) {
    bool ok = mbar_wait(&sm.full[b], fph[b], P.data_polls);
    bool tmo = !ok;
    if (!ok) ok = mbar_wait(&sm.full[b], fph[b], P.polls);   // never reuse a buffer a copy may still fill
    if (csync_or(!ok)) {
      if (threadIdx.x == 0) atomicOr(&P.ctl->err, 1u);
      return;
    }
    tmo = csync_or(tmo);
    fph[b] ^= 1u;
    const int kind = sm.kind[b];
    if (kind == kItemEnd) return;
    const int filed = process<T>(P, sm, b, kind, tmo && kind != kItemFinish);
    csync();
    if (threadIdx.x == 0) {
      sm.mail[b] = filed;
      mbar_arrive(&sm.empty[b]);
    }
    b ^= 1;
  }
}

template <typename T>
__global__ void __launch_bounds__(kCtaThreads, 2) stream_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int b = 0; b < kNumBuf; ++b) {
      mbar_init(&sm.full[b], 1);
      mbar_init(&sm.empty[b], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x >= kThreads) producer(P, sm);
  else consumer<T>(P, sm);
}

// ---------------------------------------------------------------- host
struct DevInfo {
  bool ready = false;
  int sms = 0;
  int bps[3] = {0, 0, 0};   // resident CTAs per SM, by qe_dtype
};
std::mutex g_mu;
DevInfo g_dev[64];

template <typename T>
cudaError_t prepare(int* bps) {
  cudaError_t e = cudaFuncSetAttribute(stream_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(Smem)));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(bps, stream_kernel<T>, kCtaThreads, sizeof(Smem));
}

// Per-device kernel attributes and residency, set up once per device.
int device_info(int dtype, int* sms, int* bps) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QE_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  DevInfo& d = g_dev[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = prepare<float>(&d.bps[QE_DTYPE_F32]);
    if (e == cudaSuccess) e = prepare<__nv_bfloat16>(&d.bps[QE_DTYPE_BF16]);
    if (e == cudaSuccess) e = prepare<__half>(&d.bps[QE_DTYPE_F16]);
    if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("stream sampler setup: ") + cudaGetErrorString(e));
    d.ready = true;
  }
  *sms = d.sms;
  *bps = d.bps[dtype];
  return QE_OK;
}

}  // namespace st

bool stream_supports(int64_t vocab) { return vocab >= 1 && vocab < (int64_t(1) << 24); }

size_t stream_workspace_bytes(int64_t batch, int64_t vocab) {
  return st::make_layout(batch, vocab, 4).total;   // fp32 rows use the most chunks
}

const void* stream_error_word(const void* workspace) {
  return static_cast<const char*>(workspace) + offsetof(st::Ctl, err);
}

int launch_stream(const KernelArgs& ka, cudaStream_t stream) {
  using namespace st;
  const int esize = ka.dtype == QE_DTYPE_F32 ? 4 : 2;
  const Layout L = make_layout(ka.batch, ka.vocab, esize);
  const unsigned long long nitems = (unsigned long long)ka.batch * (unsigned long long)L.nc;
  if (nitems * kMaxRounds >= (1ull << 31))
    return set_error(QE_ERR_UNSUPPORTED, "batch too large for one launch of the streaming sampler");
  int sms = 0, bps = 0;
  const int rc = device_info(ka.dtype, &sms, &bps);
  if (rc != QE_OK) return rc;
  if (bps < 1) return set_error(QE_ERR_CUDA, "streaming sampler kernel cannot be resident");
  Params P;
  std::memset(&P, 0, sizeof(P));
  P.a = ka;
  P.esize = esize;
  P.tpc = L.tpc;
  P.cps = L.cps;
  P.nc = L.nc;
  const uintptr_t lp = reinterpret_cast<uintptr_t>(ka.logits);
  P.tma_ok = (lp % 16 == 0) && ((ka.ld * esize) % 16 == 0);
  P.noise_vec = 0;
  P.force_exact = ka.out_kept != nullptr;
  P.dtype_level = ka.dtype == QE_DTYPE_BF16 ? 1 : ka.dtype == QE_DTYPE_F16 ? 2 : 3;
  P.polls = kDefaultPolls;
  P.data_polls = ka.wait_polls ? ka.wait_polls - 1u : kDefaultPolls;
  P.nitems = unsigned(nitems);
  int64_t gb = 0;
  for (int s = 0; s < kNumSlices; ++s) {
    const int64_t a0 = slice_start(s, ka.vocab), a1 = slice_start(s + 1, ka.vocab);
    P.sstart[s] = a0;
    P.gbase[s] = gb;
    P.snt[s] = int((a1 - a0 + kTile - 1) / kTile);
    gb += int64_t(P.snt[s]) * 32;
  }
  P.sstart[kNumSlices] = ka.vocab;
  P.gbase[kNumSlices] = gb;
  char* base = static_cast<char*>(ka.workspace);
  P.ctl = reinterpret_cast<Ctl*>(base);
  P.rowctl = reinterpret_cast<RowCtl*>(base + L.rowctl);
  P.queue = reinterpret_cast<unsigned int*>(base + L.queue);
  P.rec = reinterpret_cast<ChunkRec*>(base + L.rec);
  P.hist = reinterpret_cast<float*>(base + L.hist);
  P.gather = reinterpret_cast<GItem*>(base + L.gather);
  P.round = reinterpret_cast<RowRound*>(base + L.round);
  P.part = reinterpret_cast<Part*>(base + L.part);
  P.hacc = reinterpret_cast<HistAcc*>(base + L.hacc);
  cudaError_t e = cudaMemsetAsync(base, 0, L.zero_bytes, stream);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  const unsigned long long resident = (unsigned long long)sms * (unsigned long long)bps;
  const int grid = int(nitems < resident ? (nitems > 0 ? nitems : 1) : resident);
  switch (ka.dtype) {
    case QE_DTYPE_F32: stream_kernel<float><<<grid, kCtaThreads, sizeof(Smem), stream>>>(P); break;
    case QE_DTYPE_BF16: stream_kernel<__nv_bfloat16><<<grid, kCtaThreads, sizeof(Smem), stream>>>(P); break;
    default: stream_kernel<__half><<<grid, kCtaThreads, sizeof(Smem), stream>>>(P); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("stream sampler launch: ") + cudaGetErrorString(e));
  return QE_OK;
}

}  // namespace qe
