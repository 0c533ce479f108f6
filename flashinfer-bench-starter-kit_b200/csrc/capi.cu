// capi.cu -- ABI-wide entry points (version, status text, device status
// word) and the host helpers shared by the operators.
#include <cudaTypedefs.h>

#include <mutex>

#include "dsa_b200.h"
#include "host.h"

namespace dsa {

namespace {

constexpr int kMaxDevices = 64;

DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

}  // namespace

int current_device_info(DeviceInfo* out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return DSA_ERR_CUDA;
  }
  std::call_once(g_info_once[dev], [dev]() {
    DeviceInfo info;
    int v = 0;
    info.device = dev;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      info.num_sms = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess)
      info.cc_major = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess)
      info.cc_minor = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
      info.max_smem_optin = static_cast<size_t>(v);
    cudaGetLastError();
    g_info[dev] = info;
  });
  *out = g_info[dev];
  if (out->num_sms <= 0) return DSA_ERR_CUDA;
  // The kernels use tcgen05 / TMEM and are built for sm_100a only.
  if (out->cc_major != 10 || out->cc_minor != 0) return DSA_ERR_UNSUPPORTED_DEVICE;
  return DSA_OK;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner,
                   uint32_t box_outer) {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    cudaGetLastError();
  });
  if (g_encode == nullptr) return DSA_ERR_TENSOR_MAP;
  if (!aligned16(base) || (row_pitch_bytes & 15u) != 0) return DSA_ERR_MISALIGNED;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSA_OK : DSA_ERR_TENSOR_MAP;
}

}  // namespace dsa

extern "C" {

int dsa_b200_abi_version(void) { return 1; }

const char* dsa_b200_status_string(int status) {
  switch (status) {
    case DSA_OK: return "ok";
    case DSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DSA_ERR_MISALIGNED: return "pointer or stride not 16-byte aligned";
    case DSA_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case DSA_ERR_CUDA: return "CUDA runtime error";
    case DSA_ERR_UNSUPPORTED_DEVICE: return "device is not sm_100 (B200)";
    case DSA_ERR_TENSOR_MAP: return "tensor map encoding failed";
    default: return "unknown status";
  }
}

int dsa_read_device_status(void* workspace, uint32_t* status_out, int clear, void* stream) {
  if (workspace == nullptr || status_out == nullptr) return DSA_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t host = 0;
  if (cudaMemcpyAsync(&host, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) !=
      cudaSuccess)
    return DSA_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return DSA_ERR_CUDA;
  *status_out = host;
  if (clear && cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s) != cudaSuccess)
    return DSA_ERR_CUDA;
  return DSA_OK;
}

}  // extern "C"
