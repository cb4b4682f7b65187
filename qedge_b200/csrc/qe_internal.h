// qe_internal.h — host/device structures shared by the sampler translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "qedge_sample.h"

namespace qe {

constexpr int kSlices = 16;

// Per (row, slice) statistics written by the slice pass.
struct alignas(32) SlicePart {
  float ymax;               // max of the (penalised) logits over the slice
  float xbest;              // greedy candidate value (penalised logits)
  int64_t xbest_idx;        // its id (first index on ties, NaN maximal)
  unsigned long long sfix;  // sum of fp32 group sums of exp(y - ymax), fixed point 2^-40
  uint32_t flags;           // 1: NaN seen, 2: empty slice
  uint32_t pad;
};

// Per-group max and group-relative softmax sum (canonical S terms).
struct GroupPart {
  float gmax;
  float fsum;
};

// Per-row state shared between passes.
struct alignas(16) RowInfo {
  float M, S;               // M: -RN(xmax * c1) (row exponent offset); S: softmax normaliser
  float c1;                 // RN(log2(e) / T)
  uint32_t status;          // enum qe_row_status
  int32_t done;             // output already written (greedy / non-finite)
  int32_t active;           // some top-k / top-p filter removes ids
  int32_t k_on, p_on;
  uint32_t pstar;           // fp32 bits of the smallest kept probability
  long long tie_keep;       // kept ids among those with probability == pstar
  long long tie_prefix[kSlices];  // ties with p == pstar in earlier slices
};

// Per (row, slice) race winner.
struct alignas(16) RacePart {
  float r;
  int32_t pad;
  int64_t id;
};

struct Workspace {
  GroupPart* groups;        // [B, groups_per_row]
  int64_t groups_per_row;
  SlicePart* slices;
  RowInfo* rows;
  RacePart* race;
  int* err;                 // set non-zero by a kernel that hit a bounded-wait timeout
};

// Flattened, validated copy of qe_sample_args handed to the kernels.
struct KernelArgs {
  int32_t dtype;
  int64_t batch, vocab, ld;
  const void* logits;
  const float* temperatures;
  const float* top_ps;
  const int32_t* top_ks;
  const float* min_ps;
  const float* rep_penalties;
  const int32_t* history;
  const int32_t* history_lens;
  int64_t history_ld;
  const float* noise;
  int64_t noise_ld;
  uint64_t seed, step;
  const uint64_t* seeds;
  const uint64_t* step_ptr;
  int64_t row_offset;
  uint32_t flags;
  uint32_t wait_polls;
  int64_t* out_ids;
  float* out_probs;
  int64_t probs_ld;
  int32_t* out_status;
  int64_t* out_kept;
  double* out_norm;
  void* workspace;
  Workspace ws;
};

// Philox key of a row: the per-row seed when given, else the call's seed.
__host__ __device__ inline uint64_t row_seed(const KernelArgs& a, int64_t row) {
  return a.seeds ? a.seeds[row] : a.seed;
}

size_t workspace_bytes(int64_t batch, int64_t vocab);
Workspace carve_workspace(void* base, int64_t batch, int64_t vocab);
int64_t groups_per_row(int64_t vocab);

int set_error(int code, const std::string& msg);
int launch_ref_path(const KernelArgs& ka, cudaStream_t st);
// Workspace bytes of the path qe_sample takes for these arguments.
size_t call_workspace_bytes(const qe_sample_args* a);

// The streaming sampler (qe_sample_stream.cu): the default path.
bool stream_supports(int64_t vocab);
size_t stream_workspace_bytes(int64_t batch, int64_t vocab);
int launch_stream(const KernelArgs& ka, cudaStream_t st);
// Device error word of the streaming path inside a workspace.
const void* stream_error_word(const void* workspace);

}  // namespace qe
