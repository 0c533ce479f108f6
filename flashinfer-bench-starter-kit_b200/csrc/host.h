// host.h -- host-side helpers shared by the operator entry points.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace dsa {

// 256-byte header at the start of every workspace; the first uint32 is the
// sticky device status word.
constexpr size_t kWorkspaceHeader = 256;

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t max_smem_optin = 0;
};

// Properties of the current device (queried once per device, then cached).
// Returns DSA_OK or DSA_ERR_CUDA / DSA_ERR_UNSUPPORTED_DEVICE.
int current_device_info(DeviceInfo* out);

// Encodes a 2-D tiled tensor map with 128-byte swizzle.
//   inner/outer: element extents; row_pitch_bytes: stride of the outer dim;
//   box_inner/box_outer: box extents in elements.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_pitch_bytes,
                   uint32_t box_inner, uint32_t box_outer);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches the indexer's top-2048 select over `rows` score rows (one CTA
// each, programmatically after the kernel that wrote the scores): row b
// reads scores[b], hist[b], seq_lens[b] and block-table row row_req[b]
// (row_req == nullptr: row b; a negative entry yields an all -1 row).
// With per-request ready counts (`ready`), a row's wait for them gives up
// after wait_limit_ns.
int launch_topk_select(const float* scores, const unsigned int* hist, const int32_t* seq_lens,
                       const int32_t* block_table, const int32_t* row_req, int32_t* out, int rows,
                       int score_stride, int max_pages, unsigned int* status, unsigned int* ready,
                       unsigned long long wait_limit_ns, const DeviceInfo& info, cudaStream_t s);

// Arms the indexer's test fault (dsa_b200_test_inject with DSA_TEST_SKIP_READY):
// kind << 56 | wait limit in ns, or 0 to disarm.
void arm_indexer_test_fault(unsigned long long armed);

// Launches `kernel` on `stream` with programmatic stream serialization, so
// its CTAs may be scheduled while the previous kernel on the stream drains
// (the kernel synchronises with griddep_wait() before touching global
// memory).  Capturable into CUDA graphs.
template <typename... Params, typename... Args>
cudaError_t launch_programmatic(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace dsa
