// qe_noalloc.cu — sampling for callers that cannot allocate device memory.
//
// qe_sample() takes its scratch from a caller workspace.  Some callers have
// no way to provide one: a plugin loaded into a host engine that owns every
// device allocation and exposes no allocator, a host language binding with
// no device-memory API, or code that must not grow the process's device
// footprint on the decode path.  qe_sample_noalloc() serves them with the
// same kernels, taking the scratch from a fixed array compiled into this
// library instead.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "qe_internal.h"

namespace qe {
namespace {

// Scratch for qe_sample_noalloc: fixed size, held by every GPU that uses this
// library until the process exits.  In host code `g_noalloc_scratch` is only a
// host-side stand-in for the symbol; its device address comes from
// cudaGetSymbolAddress below.
constexpr size_t kNoAllocBytes = QE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_dev_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, resolved once
// per device (the first call on a device does this set-up).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QE_ERR_CUDA, std::string("qe_sample_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(QE_ERR_UNSUPPORTED, "qe_sample_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dev_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(QE_ERR_CUDA, std::string("qe_sample_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_dev_ptr[dev] = p;
  }
  *out = g_dev_ptr[dev];
  return QE_OK;
}

}  // namespace
}  // namespace qe

extern "C" int qe_sample_noalloc(const qe_sample_args* a, void* stream) {
  using namespace qe;
  if (!a) return set_error(QE_ERR_INVALID, "args is NULL");
  if (a->struct_size != sizeof(qe_sample_args))
    return set_error(QE_ERR_INVALID, "struct_size mismatch (header/library version skew)");
  if (a->batch <= 0 || a->vocab < 1 || a->vocab >= (int64_t(1) << 24))
    return qe_sample(a, stream);  // qe_sample handles empty batches and reports bad sizes
  const size_t need = call_workspace_bytes(a);
  if (need > kNoAllocBytes)
    return set_error(QE_ERR_UNSUPPORTED,
                     "qe_sample_noalloc: " + std::to_string(a->batch) + " rows of " + std::to_string(a->vocab) +
                         " ids need " + std::to_string(need) + " bytes of scratch; the built-in scratch holds " +
                         std::to_string(kNoAllocBytes) + " bytes (split the batch, or call qe_sample with a workspace)");
  void* ws = nullptr;
  const int rc = scratch_address(&ws);
  if (rc != QE_OK) return rc;
  qe_sample_args b = *a;
  b.workspace = ws;
  b.workspace_bytes = kNoAllocBytes;
  return qe_sample(&b, stream);
}
