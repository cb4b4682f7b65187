// qe_abi.cu — the exported C ABI (include/qedge_sample.h): argument
// validation, workspace layout and dispatch to the sampler paths.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "qe_common.cuh"
#include "qe_internal.h"

namespace qe {

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int64_t groups_per_row(int64_t vocab) {
  int64_t n = 0;
  for (int g = 0; g < kNumSlices; ++g) n += slice_groups(slice_start(g + 1, vocab) - slice_start(g, vocab));
  return n;
}

// Scratch of the multi-kernel path (qe_sample_ref.cu).
size_t workspace_bytes(int64_t batch, int64_t vocab) {
  size_t b = size_t(batch);
  size_t n = align_up(b * size_t(groups_per_row(vocab)) * sizeof(GroupPart), 256);
  n = align_up(n + b * kSlices * sizeof(SlicePart), 256);
  n = align_up(n + b * sizeof(RowInfo), 256);
  n = align_up(n + b * kSlices * sizeof(RacePart), 256);
  n = align_up(n + 256, 256);
  return n;
}

Workspace carve_workspace(void* base, int64_t batch, int64_t vocab) {
  char* p = static_cast<char*>(base);
  size_t b = size_t(batch), n = 0;
  Workspace w;
  w.groups = reinterpret_cast<GroupPart*>(p);
  w.groups_per_row = groups_per_row(vocab);
  n = align_up(b * size_t(w.groups_per_row) * sizeof(GroupPart), 256);
  w.slices = reinterpret_cast<SlicePart*>(p + n);
  n = align_up(n + b * kSlices * sizeof(SlicePart), 256);
  w.rows = reinterpret_cast<RowInfo*>(p + n);
  n = align_up(n + b * sizeof(RowInfo), 256);
  w.race = reinterpret_cast<RacePart*>(p + n);
  n = align_up(n + b * kSlices * sizeof(RacePart), 256);
  w.err = reinterpret_cast<int*>(p + n);
  return w;
}

// The multi-kernel path serves the debug probabilities and callers that ask
// for it; everything else runs the streaming path.
static bool uses_multi_kernel(const qe_sample_args* a) {
  return a->out_probs != nullptr || (a->flags & QE_FLAG_MULTI_KERNEL) != 0u;
}

size_t call_workspace_bytes(const qe_sample_args* a) {
  return uses_multi_kernel(a) ? workspace_bytes(a->batch, a->vocab) : stream_workspace_bytes(a->batch, a->vocab);
}

}  // namespace qe

using namespace qe;

extern "C" int qe_abi_version(void) { return QE_ABI_VERSION; }

extern "C" const char* qe_last_error(void) { return g_last_error.c_str(); }

extern "C" size_t qe_sample_workspace_size(int64_t batch, int64_t vocab) {
  if (batch <= 0 || vocab <= 0) return 0;
  const size_t a = workspace_bytes(batch, vocab), b = stream_workspace_bytes(batch, vocab);
  return a > b ? a : b;
}

extern "C" int qe_sample_errors(const void* workspace, void* stream, uint32_t* flags) {
  g_last_error.clear();
  if (!workspace || !flags) return set_error(QE_ERR_INVALID, "workspace and flags are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemcpy(flags, stream_error_word(workspace), sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("qe_sample_errors: ") + cudaGetErrorString(e));
  return QE_OK;
}

extern "C" int qe_sample(const qe_sample_args* a, void* stream) {
  g_last_error.clear();
  if (!a) return set_error(QE_ERR_INVALID, "args is NULL");
  if (a->struct_size != sizeof(qe_sample_args))
    return set_error(QE_ERR_INVALID, "struct_size mismatch (header/library version skew)");
  if (a->batch < 0) return set_error(QE_ERR_INVALID, "batch < 0");
  if (a->batch == 0) return QE_OK;
  if (a->vocab < 1 || a->vocab >= (int64_t(1) << 24))
    return set_error(QE_ERR_INVALID, "vocab must be in [1, 2^24)");
  if (a->ld < a->vocab) return set_error(QE_ERR_INVALID, "ld < vocab");
  if (a->dtype != QE_DTYPE_F32 && a->dtype != QE_DTYPE_BF16 && a->dtype != QE_DTYPE_F16)
    return set_error(QE_ERR_INVALID, "unknown dtype");
  if (!a->logits || !a->temperatures || !a->out_ids)
    return set_error(QE_ERR_INVALID, "logits, temperatures and out_ids are required");
  if (a->noise && a->noise_ld < a->vocab) return set_error(QE_ERR_INVALID, "noise_ld < vocab");
  if (a->out_probs && a->probs_ld < a->vocab) return set_error(QE_ERR_INVALID, "probs_ld < vocab");
  if (a->history && a->history_ld < 0) return set_error(QE_ERR_INVALID, "history_ld < 0");
  const bool multi = uses_multi_kernel(a);
  if (multi && (a->min_ps || a->out_kept || a->out_norm))
    return set_error(QE_ERR_UNSUPPORTED, "min_ps, out_kept and out_norm need the streaming path (no out_probs)");
  const bool pen = a->history && a->rep_penalties;
  if (multi && pen && a->vocab > 48 * 1024 * 32)
    return set_error(QE_ERR_UNSUPPORTED, "repetition penalty on the multi-kernel path supports vocab <= 1,572,864");
  const size_t need = call_workspace_bytes(a);
  if (!a->workspace || a->workspace_bytes < need)
    return set_error(QE_ERR_WORKSPACE, "workspace smaller than qe_sample_workspace_size()");
  if (reinterpret_cast<uintptr_t>(a->workspace) % 256)
    return set_error(QE_ERR_INVALID, "workspace must be 256-byte aligned");

  KernelArgs ka;
  std::memset(&ka, 0, sizeof(ka));
  ka.dtype = a->dtype;
  ka.batch = a->batch; ka.vocab = a->vocab; ka.ld = a->ld;
  ka.logits = a->logits;
  ka.temperatures = a->temperatures;
  ka.top_ps = a->top_ps;
  ka.top_ks = a->top_ks;
  ka.min_ps = a->min_ps;
  ka.rep_penalties = a->rep_penalties;
  ka.history = pen ? a->history : nullptr;
  ka.history_lens = a->history_lens;
  ka.history_ld = a->history_ld;
  ka.noise = a->noise; ka.noise_ld = a->noise_ld;
  ka.seed = a->seed; ka.seeds = a->seeds; ka.step = a->step; ka.step_ptr = a->step_ptr;
  ka.row_offset = a->row_offset;
  ka.flags = a->flags;
  ka.wait_polls = a->wait_polls;
  ka.out_ids = a->out_ids;
  ka.out_probs = a->out_probs; ka.probs_ld = a->probs_ld;
  ka.out_status = a->out_status;
  ka.out_kept = a->out_kept;
  ka.out_norm = a->out_norm;
  ka.workspace = a->workspace;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!multi) return launch_stream(ka, st);
  ka.ws = carve_workspace(a->workspace, a->batch, a->vocab);
  return launch_ref_path(ka, st);
}
