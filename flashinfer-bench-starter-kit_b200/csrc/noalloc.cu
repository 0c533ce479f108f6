// noalloc.cu -- the indexer for callers that must not allocate device memory.
//
// dsa_indexer_run takes a caller-provided workspace.  Some callers cannot
// provide one on demand: hosts that embed this library through a C / JNI /
// FFI boundary while another allocator (an inference server's arena, a
// framework's caching allocator) owns all device memory, and serving loops
// that forbid cudaMalloc after warm-up because it can synchronise the device
// and stall every stream.  dsa_indexer_run_noalloc serves them from one
// fixed scratch array compiled into the library instead.
#include <cuda_runtime.h>

#include <mutex>

#include "dsa_b200.h"

namespace {

// The whole scratch of one indexer call: the 256-byte status header, the
// per-request ready counters, one 2048-bin radix histogram per request and
// the fp32 score rows.  Every GPU that loads the library holds these bytes
// until the process exits; static device memory starts zero-filled, which is
// the state the ready counters must start from.
static __device__ __align__(256) unsigned char g_noalloc_scratch[DSA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
void* g_scratch_ptr[kMaxDevices];
int g_scratch_status[kMaxDevices];

}  // namespace

extern "C" int dsa_indexer_run_noalloc(const void* q_index_fp8, const void* k_index_cache_fp8,
                                       int64_t num_pages, const float* weights,
                                       const int32_t* seq_lens, const int32_t* block_table,
                                       int32_t batch, int32_t max_pages, int32_t* topk_indices,
                                       void* stream) {
  // Reject problems whose scratch does not fit before touching the device.
  if (batch > 0 && max_pages > 0 &&
      dsa_indexer_workspace_bytes(batch, max_pages) > DSA_NOALLOC_SCRATCH_BYTES)
    return DSA_ERR_WORKSPACE_TOO_SMALL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return DSA_ERR_CUDA;
  }
  // In host code g_noalloc_scratch names a host-side stand-in; the device
  // address is looked up once per device, with that device current.
  std::call_once(g_once[dev], [dev]() {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    g_scratch_ptr[dev] = e == cudaSuccess ? ptr : nullptr;
    g_scratch_status[dev] = e == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
    if (e != cudaSuccess) cudaGetLastError();
  });
  if (g_scratch_status[dev] != DSA_OK) return g_scratch_status[dev];
  // The histogram region is cleared inside dsa_indexer_run on every call,
  // the score rows are rewritten for every token they are read at, and the
  // ready counters (at fixed offsets for every request index) are left
  // consistent by every call, so the previous call's contents need no
  // clearing here.
  return dsa_indexer_run(q_index_fp8, k_index_cache_fp8, num_pages, weights, seq_lens,
                         block_table, batch, max_pages, topk_indices, g_scratch_ptr[dev],
                         DSA_NOALLOC_SCRATCH_BYTES, stream);
}
