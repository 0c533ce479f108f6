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

}  // namespace dsa
