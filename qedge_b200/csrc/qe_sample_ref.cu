// qe_sample_ref.cu — the multi-kernel sampler path (general sizes).
//
// Replaces BatchSampler.forward (src/compute/sampler.py:25-41).  Five
// launches per call, each a plain data-parallel pass over the logits
// (rows re-read from L2 between passes):
//   1. slice_stats   (grid 8 x B): penalty, greedy argmax, slice max of
//                     logits/T, fixed-point group sums of exp(y - m_slice)
//   2. row_reduce    (grid B):     M, S, greedy / non-finite rows resolved
//   3. threshold     (grid B):     exact kept set of top-k / top-p by a
//                     4 x 8-bit radix select on the fp32 probability bits
//   4. race          (grid 8 x B): exponential race over the kept ids
//   5. finalize      (grid B):     argmax over the 8 slice winners
// The fused cluster kernel (qe_sample_fused.cu) computes the same values
// for the common shapes; this path covers everything else and is the GPU
// yardstick for it.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "qe_common.cuh"
#include "qe_internal.h"

namespace qe {

// --------------------------------------------------------------- helpers
__device__ __forceinline__ uint64_t fix_mass(float p) {
  return __double2ull_rn(double(p) * kMassScale);
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* sm) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < NT / 32 ? sm[threadIdx.x] : -INFINITY;
    for (int o = 16; o; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) sm[0] = w;
  }
  __syncthreads();
  float r = sm[0];
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ void block_argmax(float& v, int64_t& i, float* smv, int64_t* smi) {
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (argmax_better(ov, oi, v, i)) { v = ov; i = oi; }
  }
  if ((threadIdx.x & 31) == 0) { smv[threadIdx.x >> 5] = v; smi[threadIdx.x >> 5] = i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < NT / 32; ++w)
      if (argmax_better(smv[w], smi[w], v, i)) { v = smv[w]; i = smi[w]; }
    smv[0] = v; smi[0] = i;
  }
  __syncthreads();
  v = smv[0]; i = smi[0];
  __syncthreads();
}

// Race order: larger r first, then smaller id; NaN never wins.
__device__ __forceinline__ bool race_better(float r, int64_t i, float rb, int64_t ib) {
  if (r != r) return false;
  return r > rb || (r == rb && i < ib);
}

// Penalty bitmap of ids [a, a + nbits) built from the row's history.
__device__ void build_bitmap(uint32_t* bits, int64_t nwords, const int32_t* hist, int64_t hlen,
                             int64_t a, int64_t z) {
  for (int64_t w = threadIdx.x; w < nwords; w += blockDim.x) bits[w] = 0u;
  __syncthreads();
  for (int64_t h = threadIdx.x; h < hlen; h += blockDim.x) {
    int64_t id = hist[h];
    if (id >= a && id < z) atomicOr(&bits[(id - a) >> 5], 1u << ((id - a) & 31));
  }
  __syncthreads();
}

struct RowParams {
  float T, rp;
  bool greedy, pen;
  const int32_t* hist;
  int64_t hlen;
};

__device__ __forceinline__ RowParams row_params(const KernelArgs& a, int64_t row) {
  RowParams p;
  p.T = a.temperatures[row];
  p.greedy = (a.flags & QE_FLAG_ALL_GREEDY) || !(p.T > kGreedyEps);
  p.rp = a.rep_penalties ? a.rep_penalties[row] : 1.f;
  p.hist = a.history ? a.history + row * a.history_ld : nullptr;
  p.hlen = a.history ? (a.history_lens ? a.history_lens[row] : a.history_ld) : 0;
  if (p.hlen > a.history_ld) p.hlen = a.history_ld;
  if (p.hlen < 0) p.hlen = 0;
  p.pen = p.hist && p.hlen > 0 && p.rp != 1.f;
  return p;
}

template <typename T>
__device__ __forceinline__ float load_x(const KernelArgs& a, int64_t row, int64_t j,
                                        const uint32_t* bits, int64_t base, const RowParams& rp) {
  const T* x = static_cast<const T*>(a.logits) + row * a.ld;
  float v = Elem<T>::load(x + j);
  if (rp.pen && ((bits[(j - base) >> 5] >> ((j - base) & 31)) & 1u)) v = penalise(v, rp.rp);
  return v;
}

// --------------------------------------------------------------- kernel 1
template <typename T>
__global__ void __launch_bounds__(256) slice_stats_kernel(KernelArgs a) {
  extern __shared__ uint32_t smem_bits[];
  __shared__ float smf[32];
  __shared__ int64_t smi[32];
  __shared__ unsigned long long ssum;
  __shared__ int snan;
  const int g = blockIdx.x;
  const int64_t row = blockIdx.y;
  const int64_t V = a.vocab;
  const int64_t s0 = slice_start(g, V), s1 = slice_start(g + 1, V), L = s1 - s0;
  const RowParams rp = row_params(a, row);
  if (rp.pen) build_bitmap(smem_bits, (L + 31) / 32, rp.hist, rp.hlen, s0, s1);
  if (threadIdx.x == 0) { ssum = 0ull; snan = 0; }
  __syncthreads();

  float xb = -INFINITY; int64_t ib = INT64_MAX;
  float xmax = -INFINITY; bool nan = false;
  for (int64_t j = s0 + threadIdx.x; j < s1; j += blockDim.x) {
    float x = load_x<T>(a, row, j, smem_bits, s0, rp);
    if (argmax_better(x, j, xb, ib)) { xb = x; ib = j; }
    nan |= (x != x);
    xmax = fmaxf(xmax, x);
  }
  block_argmax<256>(xb, ib, smf, smi);
  if (nan) snan = 1;
  xmax = block_max<256>(xmax, smf);
  SlicePart* part = a.ws.slices + row * kNumSlices + g;
  uint64_t total = 0;
  const float c1 = rp.greedy ? 0.f : temp_coef(rp.T);
  const float c0 = max_coef(xmax, c1);
  const bool nonfinite = snan || !(xmax > -INFINITY) || !(fabsf(c0) < INFINITY);
  if (!rp.greedy && !nonfinite) {
    // canonical group sums: relative to each group's own max
    const int64_t ng = slice_groups(L);
    GroupPart* gp = a.ws.groups + row * a.ws.groups_per_row + slice_group_base(g, V);
    for (int64_t lg = threadIdx.x; lg < ng; lg += blockDim.x) {
      float gm = -INFINITY;
      for (int m = 0; m < 32; ++m) {
        int64_t o = member_offset(lg, m);
        if (o < L) gm = fmaxf(gm, load_x<T>(a, row, s0 + o, smem_bits, s0, rp));
      }
      float fs = 0.f;
      if (gm > -INFINITY) {
        const float c0g = max_coef(gm, c1);
        for (int m = 0; m < 32; ++m) {
          int64_t o = member_offset(lg, m);
          if (o < L) fs = __fadd_rn(fs, unnorm(load_x<T>(a, row, s0 + o, smem_bits, s0, rp), c1, c0g));
        }
      }
      gp[lg] = GroupPart{gm, fs};
    }
  }
  (void)c0;
  (void)ssum;
  if (threadIdx.x == 0) {
    part->ymax = xmax;
    part->xbest = xb;
    part->xbest_idx = ib;
    part->sfix = total;
    part->flags = (snan ? 1u : 0u) | (L == 0 ? 2u : 0u);
  }
}

// --------------------------------------------------------------- kernel 2
__global__ void __launch_bounds__(256) row_reduce_kernel(KernelArgs a) {
  __shared__ unsigned long long s_sum;
  const int64_t row = blockIdx.x;
  const RowParams rp = row_params(a, row);
  const SlicePart* sp = a.ws.slices + row * kNumSlices;
  float xb = -INFINITY; int64_t ib = INT64_MAX;
  float M = -INFINITY; bool nan = false;
  for (int g = 0; g < kNumSlices; ++g) {
    if (sp[g].flags & 2u) continue;
    if (argmax_better(sp[g].xbest, sp[g].xbest_idx, xb, ib)) { xb = sp[g].xbest; ib = sp[g].xbest_idx; }
    nan |= (sp[g].flags & 1u) != 0;
    M = fmaxf(M, sp[g].ymax);
  }
  const bool nonfinite_x = nan || !(M > -INFINITY) || M == INFINITY;
  const float c1 = rp.greedy ? 0.f : temp_coef(rp.T);
  const float nM = max_coef(M, c1);
  if (threadIdx.x == 0) s_sum = 0ull;
  __syncthreads();
  if (!rp.greedy && !nonfinite_x && fabsf(nM) < INFINITY) {
    // S = sum over groups of round(2^40 * fsum * 2^(c0_row - c0_group)) * 2^-40
    const GroupPart* gp = a.ws.groups + row * a.ws.groups_per_row;
    unsigned long long acc = 0;
    for (int64_t i = threadIdx.x; i < a.ws.groups_per_row; i += blockDim.x) {
      const GroupPart g = gp[i];
      if (g.fsum > 0.f) {
        const float sc = qe_ex2(__fsub_rn(nM, max_coef(g.gmax, c1)));
        acc += __double2ull_rn(double(__fmul_rn(g.fsum, sc)) * kSumScale);
      }
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_sum, acc);
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  RowInfo* ri = a.ws.rows + row;
  uint32_t status = 0;
  ri->active = 0;
  if (rp.greedy) {
    status = QE_ROW_GREEDY;
  } else if (nonfinite_x || !(fabsf(nM) < INFINITY)) {
    status = QE_ROW_NONFINITE;
  } else {
    const double S = double(s_sum) * (1.0 / kSumScale);
    ri->M = nM;
    ri->c1 = c1;
    ri->S = float(S);
    const int64_t V = a.vocab;
    int k = a.top_ks ? a.top_ks[row] : 0;
    bool k_on = k > 0 && int64_t(k) < V;
    float tp = a.top_ps ? a.top_ps[row] : 1.f;
    bool p_on = (a.flags & QE_FLAG_USE_TOP_P) && a.top_ps && tp < 1.f;
    ri->active = (k_on || p_on) ? 1 : 0;
    ri->k_on = k_on; ri->p_on = p_on;
    if (!(ri->S > 0.f) || ri->S == INFINITY) status = QE_ROW_NONFINITE;
    if (status) ri->active = 0;
  }
  ri->status = status;
  if (status) {
    a.out_ids[row] = ib;
    ri->done = 1;
  } else {
    ri->done = 0;
  }
  if (a.out_status) a.out_status[row] = int32_t(status);
}

// --------------------------------------------------------------- kernel 3
template <typename T>
__device__ __forceinline__ float prob_at(const KernelArgs& a, int64_t row, int64_t j, const uint32_t* bits,
                                         const RowParams& rp, float c1, float M, float S) {
  return __fdiv_rn(unnorm(load_x<T>(a, row, j, bits, 0, rp), c1, M), S);
}

template <typename T>
__global__ void __launch_bounds__(1024) threshold_kernel(KernelArgs a) {
  extern __shared__ uint32_t smem_bits[];
  __shared__ uint32_t hc[256];
  __shared__ unsigned long long hm[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ long long s_cbase;
  __shared__ unsigned long long s_mbase;
  __shared__ int s_bin;
  __shared__ unsigned long long s_tie[kNumSlices];
  const int64_t row = blockIdx.x;
  RowInfo* ri = a.ws.rows + row;
  if (ri->done || !ri->active) return;
  const RowParams rp = row_params(a, row);
  const int64_t V = a.vocab;
  if (rp.pen) build_bitmap(smem_bits, (V + 31) / 32, rp.hist, rp.hlen, 0, V);
  const float M = ri->M, S = ri->S, c1 = ri->c1;
  const int k = a.top_ks ? a.top_ks[row] : 0;
  const int64_t n_k = ri->k_on ? int64_t(k) : V;
  int64_t n_keep = n_k;
  uint32_t pstar = 0;
  int64_t tie_keep = 0;
  bool have = false;

  if (ri->p_on) {
    // weighted select: last element whose exclusive mass is <= top_p
    const uint64_t Tfix = uint64_t(double(a.top_ps[row]) * kMassScale);
    if (threadIdx.x == 0) { s_prefix = 0; s_mask = 0; s_cbase = 0; s_mbase = 0; }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) { hc[b] = 0; hm[b] = 0; }
      __syncthreads();
      const uint32_t pre = s_prefix, msk = s_mask;
      for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
        float p = prob_at<T>(a, row, j, smem_bits, rp, c1, M, S);
        uint32_t key = __float_as_uint(p);
        if ((key & msk) == pre) {
          int b = (key >> shift) & 255;
          atomicAdd(&hc[b], 1u);
          atomicAdd(&hm[b], (unsigned long long)fix_mass(p));
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        long long c = s_cbase;
        unsigned long long m = s_mbase;
        int cand = -1; long long cc = c; unsigned long long cm = m;
        for (int b = 255; b >= 0; --b) {
          if (hc[b] == 0) continue;
          if (m <= Tfix) { cand = b; cc = c; cm = m; } else break;
          m += hm[b]; c += hc[b];
        }
        s_bin = cand;
        s_prefix = pre | (uint32_t(cand) << shift);
        s_mask = msk | (255u << shift);
        s_cbase = cc; s_mbase = cm;
      }
      __syncthreads();
    }
    // s_prefix is the exact key; hc[s_bin] its tie count
    const uint32_t key = s_prefix;
    const uint64_t f = fix_mass(__uint_as_float(key));
    const long long nt = hc[s_bin & 255];
    long long c = nt;
    if (f > 0) {
      unsigned long long room = Tfix - s_mbase;
      unsigned long long q = room / f + 1;
      if (q < (unsigned long long)nt) c = (long long)q;
    }
    const int64_t n_p = s_cbase + c;
    if (n_p <= n_k) { have = true; pstar = key; tie_keep = c; n_keep = n_p; }
    __syncthreads();
  }
  if (!have) {
    // count select: element at position n_keep - 1
    const long long pos = n_keep - 1;
    if (threadIdx.x == 0) { s_prefix = 0; s_mask = 0; s_cbase = 0; }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) hc[b] = 0;
      __syncthreads();
      const uint32_t pre = s_prefix, msk = s_mask;
      for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
        uint32_t key = __float_as_uint(prob_at<T>(a, row, j, smem_bits, rp, c1, M, S));
        if ((key & msk) == pre) atomicAdd(&hc[(key >> shift) & 255], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        long long c = s_cbase;
        int cand = 0;
        for (int b = 255; b >= 0; --b) {
          if (hc[b] == 0) continue;
          if (pos < c + hc[b]) { cand = b; break; }
          c += hc[b];
        }
        s_bin = cand; s_cbase = c;
        s_prefix = pre | (uint32_t(cand) << shift);
        s_mask = msk | (255u << shift);
      }
      __syncthreads();
    }
    pstar = s_prefix;
    tie_keep = pos - s_cbase + 1;
  }
  // ties per slice (for the id-order rank of tied candidates)
  if (threadIdx.x < kNumSlices) s_tie[threadIdx.x] = 0;
  __syncthreads();
  for (int g = 0; g < kNumSlices; ++g) {
    const int64_t s0 = slice_start(g, V), s1 = slice_start(g + 1, V);
    unsigned long long cnt = 0;
    for (int64_t j = s0 + threadIdx.x; j < s1; j += blockDim.x)
      cnt += __float_as_uint(prob_at<T>(a, row, j, smem_bits, rp, c1, M, S)) == pstar;
    if (cnt) atomicAdd(&s_tie[g], cnt);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ri->pstar = pstar;
    ri->tie_keep = tie_keep;
    long long acc = 0;
    for (int g = 0; g < kNumSlices; ++g) { ri->tie_prefix[g] = acc; acc += s_tie[g]; }
  }
}

// --------------------------------------------------------------- kernel 4
template <typename T>
__global__ void __launch_bounds__(256) race_kernel(KernelArgs a) {
  extern __shared__ uint32_t smem_bits[];
  __shared__ float smf[32];
  __shared__ int64_t smi[32];
  __shared__ int warp_ties[8];
  const int g = blockIdx.x;
  const int64_t row = blockIdx.y;
  const RowInfo* ri = a.ws.rows + row;
  RacePart* out = a.ws.race + row * kNumSlices + g;
  if (ri->done) return;
  const int64_t V = a.vocab;
  const int64_t s0 = slice_start(g, V), s1 = slice_start(g + 1, V), L = s1 - s0;
  const RowParams rp = row_params(a, row);
  if (rp.pen) build_bitmap(smem_bits, (L + 31) / 32, rp.hist, rp.hlen, s0, s1);
  const float M = ri->M, S = ri->S, c1 = ri->c1;
  const bool active = ri->active;
  const uint32_t pstar = ri->pstar;
  const long long tie_keep = ri->tie_keep;
  long long tie_base = ri->tie_prefix[g];
  const uint64_t step = a.step_ptr ? *a.step_ptr : a.step;
  const NoiseKey key = make_noise_key(row_seed(a, row), step, a.row_offset + row);
  NoiseRoot root{0.f, 0};
  int64_t gid_s = -1; int mem_s = 0;
  if (!a.noise) {
    root = noise_root(key, V);
    token_group(root.s, V, &gid_s, &mem_s);
  }
  const int64_t gbase = slice_group_base(g, V);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float rb = -INFINITY; int64_t ib = INT64_MAX;
  for (int64_t c0 = s0; c0 < s1; c0 += blockDim.x) {
    const int64_t j = c0 + threadIdx.x;
    const bool valid = j < s1;
    float p = 0.f;
    if (valid) {
      p = __fdiv_rn(unnorm(load_x<T>(a, row, j, smem_bits, s0, rp), c1, M), S);
      if (a.out_probs) a.out_probs[row * a.probs_ld + j] = p;
    }
    bool in = valid;
    if (active) {
      const uint32_t kb = __float_as_uint(p);
      const bool tie = valid && kb == pstar;
      const uint32_t ballot = __ballot_sync(0xffffffffu, tie);
      if (lane == 0) warp_ties[warp] = __popc(ballot);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < int(blockDim.x / 32); ++w) { if (w < warp) before += warp_ties[w]; total += warp_ties[w]; }
      const long long rank = tie_base + before + __popc(ballot & ((1u << lane) - 1u));
      in = valid && (kb > pstar || (tie && rank < tie_keep));
      tie_base += total;
      __syncthreads();
    }
    if (in) {
      float E;
      if (a.noise) {
        E = a.noise[row * a.noise_ld + j];
      } else {
        const int64_t o = j - s0;
        const int64_t gid = gbase + local_group(o);
        const int mem = member_index(o);
        const GroupNoise gm = noise_group(key, root, gid, group_size(local_group(o), L), gid_s, mem_s);
        E = noise_token(key, gm, j, mem);
      }
      const float r = __fdiv_rn(p, E);
      if (race_better(r, j, rb, ib)) { rb = r; ib = j; }
    }
  }
  // block reduction in race order
  for (int o = 16; o; o >>= 1) {
    float orr = __shfl_xor_sync(0xffffffffu, rb, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, ib, o);
    if (race_better(orr, oi, rb, ib)) { rb = orr; ib = oi; }
  }
  if (lane == 0) { smf[warp] = rb; smi[warp] = ib; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x / 32); ++w)
      if (race_better(smf[w], smi[w], rb, ib)) { rb = smf[w]; ib = smi[w]; }
    out->r = rb;
    out->id = ib;
  }
}

// --------------------------------------------------------------- kernel 5
__global__ void finalize_kernel(KernelArgs a) {
  const int64_t row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= a.batch) return;
  const RowInfo* ri = a.ws.rows + row;
  if (ri->done) return;
  const RacePart* rp = a.ws.race + row * kNumSlices;
  float rb = -INFINITY; int64_t ib = INT64_MAX;
  for (int g = 0; g < kNumSlices; ++g)
    if (race_better(rp[g].r, rp[g].id, rb, ib)) { rb = rp[g].r; ib = rp[g].id; }
  a.out_ids[row] = ib == INT64_MAX ? 0 : ib;
}

// --------------------------------------------------------------- host
template <typename T>
static int launch_typed(const KernelArgs& ka, cudaStream_t st) {
  const int64_t V = ka.vocab, B = ka.batch;
  const bool pen = ka.history && ka.rep_penalties;
  const int64_t slice_max = V / kNumSlices + 16;
  const size_t slice_bits = pen ? size_t((slice_max + 31) / 32) * 4 : 0;
  const size_t row_bits = pen ? size_t((V + 31) / 32) * 4 : 0;
  dim3 g1(kNumSlices, unsigned(B));
  slice_stats_kernel<T><<<g1, 256, slice_bits, st>>>(ka);
  row_reduce_kernel<<<unsigned(B), 256, 0, st>>>(ka);
  if (!(ka.flags & QE_FLAG_ALL_GREEDY)) {
    threshold_kernel<T><<<unsigned(B), 1024, row_bits, st>>>(ka);
    race_kernel<T><<<g1, 256, slice_bits, st>>>(ka);
    finalize_kernel<<<unsigned((B + 127) / 128), 128, 0, st>>>(ka);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  return QE_OK;
}

// Kernel attributes are per-device state: set them once per device, under a
// lock (host threads may drive several devices).
int ref_path_prepare() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QE_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return QE_OK;
  // the dynamic shared-memory bitmap of a whole row may exceed 48 KB
  const int max_bytes = 200 * 1024;
  e = cudaFuncSetAttribute(threshold_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(threshold_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(threshold_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  done[dev] = true;
  return QE_OK;
}

int launch_ref_path(const KernelArgs& ka, cudaStream_t st) {
  int rc = ref_path_prepare();
  if (rc) return rc;
  switch (ka.dtype) {
    case QE_DTYPE_F32: return launch_typed<float>(ka, st);
    case QE_DTYPE_BF16: return launch_typed<__nv_bfloat16>(ka, st);
    case QE_DTYPE_F16: return launch_typed<__half>(ka, st);
  }
  return set_error(QE_ERR_INVALID, "unknown dtype");
}

}  // namespace qe
