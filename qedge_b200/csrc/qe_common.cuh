// qe_common.cuh — device helpers shared by the sampler kernels.
//
// Numerics follow the reference sampler (src/compute/sampler.py:30-41):
// logits are upcast to fp32, divided by the temperature with IEEE division,
// soft-maxed in fp32 and drawn by an exponential race.  The canonical
// row reductions (slice maxima, fixed-point group sums) and the Philox noise
// tree are defined here once so every kernel (single-GPU, vocab-sharded)
// produces the same bits.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qedge_sample.h"

namespace qe {

constexpr int kNumSlices = 16;         // canonical vocab slices per row (== kSlices)
constexpr int kTile = 1024;            // ids per tile inside a slice
constexpr int kGroupLanes = 32;        // groups per tile
constexpr float kGreedyEps = 1e-5f;    // sampler.py:30 `temperatures <= 1e-5`
constexpr double kSumScale = 1099511627776.0;        // 2^40: fixed-point of group sums
constexpr double kMassScale = 4611686018427387904.0; // 2^62: fixed-point of probabilities

// ---------------------------------------------------------------- layout
// Slice g of a row covers ids [slice_start(g), slice_start(g+1)); starts are
// multiples of 8 ids so every slice begins 16-byte aligned for 2-byte types.
__host__ __device__ __forceinline__ int64_t slice_start(int g, int64_t V) {
  return g >= kNumSlices ? V : ((int64_t(g) * V) / (kNumSlices * 8)) * 8;
}
__host__ __device__ __forceinline__ int64_t slice_groups(int64_t L) {
  return ((L + kTile - 1) / kTile) * kGroupLanes;
}
// Inside a slice, offset o = t*1024 + b*256 + l*8 + i belongs to local group
// t*32 + l as member b*8 + i (members in increasing id order).
__host__ __device__ __forceinline__ int64_t local_group(int64_t o) {
  return (o >> 10) * kGroupLanes + ((o >> 3) & 31);
}
__host__ __device__ __forceinline__ int member_index(int64_t o) {
  return int(((o >> 8) & 3) * 8 + (o & 7));
}
// Offset of member m of local group lg.
__host__ __device__ __forceinline__ int64_t member_offset(int64_t lg, int m) {
  return (lg >> 5) * kTile + int64_t(m >> 3) * 256 + (lg & 31) * 8 + (m & 7);
}
// Members of local group lg in a slice of length L.
__host__ __device__ __forceinline__ int group_size(int64_t lg, int64_t L) {
  int n = 0;
  for (int b = 0; b < 4; ++b) {
    int64_t base = (lg >> 5) * kTile + int64_t(b) * 256 + (lg & 31) * 8;
    int64_t c = L - base;
    n += c <= 0 ? 0 : (c >= 8 ? 8 : int(c));
  }
  return n;
}

// ---------------------------------------------------------------- loads
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return __ldg(p); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) {
    unsigned short b = __ldg(reinterpret_cast<const unsigned short*>(p));
    return __uint_as_float(uint32_t(b) << 16);
  }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float load(const __half* p) {
    return __half2float(__ldg(p));
  }
};

// ---------------------------------------------------------------- math
// exp(d) for d <= 0 through the SFU: 2^(d*log2 e).  Relative error stays
// below ~2^-21 + |d| * 2^-24, i.e. < 5e-6 down to the fp32 underflow point.
__device__ __forceinline__ float qe_exp(float d) {
  float t = __fmul_rn(d, 1.4426950408889634f);
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}

// Repetition penalty of one logit (Hugging Face rule: x<0 ? x*rp : x/rp).
// Out-of-line IEEE division: keeps the rarely taken penalty branch small at
// every call site.
static __device__ __noinline__ float div_rn_outlined(float x, float y) { return __fdiv_rn(x, y); }
__device__ __forceinline__ float penalise(float x, float rp) {
  return x < 0.f ? __fmul_rn(x, rp) : div_rn_outlined(x, rp);
}

// Greedy comparison of torch.argmax: NaN is maximal, first index wins ties.
__device__ __forceinline__ bool argmax_better(float a, int64_t ia, float b, int64_t ib) {
  bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

// ---------------------------------------------------------------- Philox
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): multipliers and Weyl
// key increments from that paper.
struct U4 { uint32_t x, y, z, w; };
__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
enum : uint32_t { kTagRoot = 0, kTagGroup = 1, kTagToken = 2, kTagGroupMin = 3 };

// Odd multiple of 2^-24 in (0,1): exact in fp32.
__device__ __forceinline__ float uniform_open(uint32_t w) {
  return __fmul_rn(float((w >> 9) * 2u + 1u), 5.9604644775390625e-8f);
}
// floor(((hi<<32)|lo) * n / 2^64) for n < 2^24.
__device__ __forceinline__ uint32_t select_index(uint32_t hi, uint32_t lo, uint32_t n) {
  uint64_t x = (uint64_t(hi) << 32) | lo;
  return uint32_t(__umul64hi(x, uint64_t(n)));
}
// floor(w * n / 2^32) for n <= 2^24.
__device__ __forceinline__ uint32_t select_index32(uint32_t w, uint32_t n) {
  return uint32_t((uint64_t(w) * n) >> 32);
}
// -ln(u) for u in [2^-24, 1); IEEE fp32 round-to-nearest, no contraction.
// ln m = 2 atanh((m-1)/(m+1)) by its odd series after reduction to
// m in [sqrt(1/2), sqrt(2)]; ln 2 split into a 15-bit head and a tail.
__device__ __forceinline__ float neglog(float u) {
  uint32_t bits = __float_as_uint(u);
  int e = int(bits >> 23) - 127;
  float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > __uint_as_float(0x3FB504F3u)) { m = __fmul_rn(m, 0.5f); e += 1; }
  float f = __fdiv_rn(__fsub_rn(m, 1.f), __fadd_rn(m, 1.f));
  float f2 = __fmul_rn(f, f);
  float t = __fmul_rn(f2, __uint_as_float(0x3E638E39u));
  t = __fadd_rn(__uint_as_float(0x3E924925u), t);
  t = __fmul_rn(f2, t);
  t = __fadd_rn(__uint_as_float(0x3ECCCCCDu), t);
  t = __fmul_rn(f2, t);
  t = __fadd_rn(__uint_as_float(0x3F2AAAABu), t);
  float poly = __fmul_rn(f2, t);
  float lnm = __fadd_rn(__fadd_rn(f, f), __fmul_rn(f, poly));
  float ef = float(e);
  float r = __fadd_rn(__fmul_rn(ef, __uint_as_float(0x3F317200u)),
                      __fadd_rn(__fmul_rn(ef, __uint_as_float(0x35BFBE8Eu)), lnm));
  return -r;
}

// Philox stream key for (seed, step, row).
struct NoiseKey {
  uint32_t k0, k1, step_lo, hi;
  uint32_t row;
};
__device__ __forceinline__ NoiseKey make_noise_key(uint64_t seed, uint64_t step, int64_t row) {
  NoiseKey k;
  k.k0 = uint32_t(seed);
  k.k1 = uint32_t(seed >> 32);
  k.step_lo = uint32_t(step);
  k.hi = uint32_t((step >> 32) << 2);
  k.row = uint32_t(row);
  return k;
}
__device__ __forceinline__ U4 philox_at(const NoiseKey& k, uint32_t index, uint32_t tag) {
  return philox4x32_10(U4{index, k.row, k.step_lo, k.hi | tag}, k.k0, k.k1);
}

// Root of the noise tree: E_root = -ln(u)/V and the token s carrying it.
struct NoiseRoot { float e_root; int64_t s; };
__device__ __forceinline__ NoiseRoot noise_root(const NoiseKey& k, int64_t V) {
  U4 w = philox_at(k, 0u, kTagRoot);
  NoiseRoot r;
  r.e_root = __fdiv_rn(neglog(uniform_open(w.x)), float(V));
  r.s = select_index(w.y, w.z, uint32_t(V));
  return r;
}
__device__ __forceinline__ uint32_t pick_word(const U4& w, uint32_t i) {
  return i == 0u ? w.x : i == 1u ? w.y : i == 2u ? w.z : w.w;
}
// Word of group gid's noise minimum: one Philox call (tag kTagGroupMin,
// counter gid / 4) covers four consecutive groups, word gid % 4 each, so a
// kernel can bound every group's best ratio at a quarter of the cost.
__device__ __forceinline__ uint32_t group_min_word(const NoiseKey& k, int64_t gid) {
  return pick_word(philox_at(k, uint32_t(gid >> 2), kTagGroupMin), uint32_t(gid & 3));
}
// Noise of a group of n members: its minimum E_min = E_root + (-ln u)/n
// (u from group_min_word) and, from one Philox call with counter = global
// group id (tag kTagGroup), the member carrying it (word y), the gap to the
// second smallest value, E2 = E_min + (-ln u')/(n-1) (word z), and the
// member carrying that, uniform among the others (word w).  Every other
// member j has E_j = E2 + (-ln u_j).  The group holding the root token s
// takes E_min = E_root with s as its argmin.
struct GroupNoise { float e_min, e2; int arg, arg2; };
__device__ __forceinline__ GroupNoise group_noise_from(const NoiseRoot& root, U4 w, uint32_t wmin, int n,
                                                       bool holds_root, int mem_s) {
  GroupNoise g;
  if (holds_root) {
    g.e_min = root.e_root;
    g.arg = mem_s;
  } else {
    // n = 32 (every full group): the division is an exact scaling by 2^-5
    const float l = neglog(uniform_open(wmin));
    g.e_min = __fadd_rn(root.e_root, n == 32 ? __fmul_rn(l, 0.03125f) : __fdiv_rn(l, float(n)));
    g.arg = int(select_index32(w.y, uint32_t(n)));
  }
  if (n >= 2) {
    g.e2 = __fadd_rn(g.e_min, __fdiv_rn(neglog(uniform_open(w.z)), float(n - 1)));
    const int i2 = int(select_index32(w.w, uint32_t(n - 1)));
    g.arg2 = i2 < g.arg ? i2 : i2 + 1;
  } else {
    g.e2 = INFINITY;
    g.arg2 = -1;
  }
  return g;
}
__device__ __forceinline__ GroupNoise noise_group(const NoiseKey& k, const NoiseRoot& root, int64_t gid, int n,
                                                  int64_t gid_s, int mem_s) {
  return group_noise_from(root, philox_at(k, uint32_t(gid), kTagGroup), group_min_word(k, gid), n, gid == gid_s,
                          mem_s);
}
// Noise of token j (global id) that is member `mem` of group g.
__device__ __forceinline__ float noise_token(const NoiseKey& k, const GroupNoise& g, int64_t j, int mem) {
  if (mem == g.arg) return g.e_min;
  if (mem == g.arg2) return g.e2;
  return __fadd_rn(g.e2, neglog(uniform_open(pick_word(philox_at(k, uint32_t(j >> 2), kTagToken), uint32_t(j & 3)))));
}

// Global group id of token j in a row of V ids, plus its member index.
__device__ __forceinline__ void token_group(int64_t j, int64_t V, int64_t* gid, int* mem) {
  int64_t base = 0;
  for (int g = 0; g < kNumSlices; ++g) {
    int64_t a = slice_start(g, V), z = slice_start(g + 1, V);
    if (j < z) {
      int64_t o = j - a;
      *gid = base + local_group(o);
      *mem = member_index(o);
      return;
    }
    base += slice_groups(z - a);
  }
  *gid = -1;
  *mem = 0;
}
__device__ __forceinline__ int64_t slice_group_base(int g, int64_t V) {
  int64_t base = 0;
  for (int s = 0; s < g; ++s) base += slice_groups(slice_start(s + 1, V) - slice_start(s, V));
  return base;
}
// Noise of global token j under the Philox tree (any CTA can evaluate it).
__device__ __forceinline__ float tree_noise(const NoiseKey& key, const NoiseRoot& root, int64_t gid_s,
                                            int mem_s, int64_t j, int64_t V) {
  int s = 0;
  while (s + 1 < kNumSlices && slice_start(s + 1, V) <= j) ++s;
  const int64_t a = slice_start(s, V), L = slice_start(s + 1, V) - a;
  const int64_t o = j - a, lg = local_group(o);
  const GroupNoise gm = noise_group(key, root, slice_group_base(s, V) + lg, int(group_size(lg, L)), gid_s, mem_s);
  return noise_token(key, gm, j, member_index(o));
}

// ---------------------------------------------------------------- softmax numerics
// Canonical arithmetic of the sampler's softmax, shared by every kernel:
//   c1 = RN(log2(e) / T);  for a slice with max xm: c0 = -RN(xm * c1)
//   e_j = 2^fma(x_j, c1, c0)        (SFU ex2, within 2^-21 relative)
//   fsum(G) = sequential fp32 sum of e_j over a group's members in order
//   sfix(slice) = sum over groups of round(fsum(G) * 2^40)   (exact u64)
//   S = sum over slices of sfix * 2^-40 * 2^(c0_row - c0_slice)   (double, slice order)
//   p_j = RN(2^fma(x_j, c1, c0_row) / S)
// which is softmax(x / T) up to ~1e-6 relative.
__device__ __forceinline__ float qe_ex2(float a) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
// Flush-to-zero variant (one SFU instruction).  Identical to qe_ex2 except
// that results below 2^-126 become 0; the fused path uses it everywhere: such
// terms are below half an ulp of every sum they enter (each sum holds a term
// of 1) and a token with e < 2^-126 can never win the race.
__device__ __forceinline__ float qe_ex2_ftz(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ float unnorm_ftz(float x, float c1, float c0) { return qe_ex2_ftz(__fmaf_rn(x, c1, c0)); }
__device__ __forceinline__ float temp_coef(float T) { return __fdiv_rn(1.4426950408889634f, T); }
__device__ __forceinline__ float max_coef(float xm, float c1) { return -__fmul_rn(xm, c1); }
__device__ __forceinline__ float unnorm(float x, float c1, float c0) { return qe_ex2(__fmaf_rn(x, c1, c0)); }

}  // namespace qe
