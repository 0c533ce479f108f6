// cache_write.cu -- quantise new indexer keys into the paged FP8 K cache.
//
// The step before the indexer in a serving loop: each new token's 128-dim
// indexer key (bf16) is quantised to float8_e4m3fn with one fp32 scale per
// token and stored at its slot of the 8448-byte page layout the indexer reads
// (dsa_indexer/solution/triton/kernel.py:80,120-124: 64 x 128 fp8 bytes, then
// 64 fp32 scales).  The arithmetic is the published per-token quantisation
// of the vLLM indexer cache writer (indexer_k_quant_and_cache):
//   amax  = max_d |k_d|
//   scale = max(1e-4, amax) / 448        (optionally rounded up to a power
//                                          of two: the "ue8m0" scale format)
//   q_d   = e4m3(k_d / scale), round to nearest even
// Slots < 0 are padding and skipped; slots beyond the cache set a status bit.
//
// One warp per token: a lane loads 4 bf16 (8 bytes, coalesced 256 B per
// warp), the warp max-reduces |k| with shuffles, and each lane writes its 4
// fp8 bytes; lane 0 writes the scale.  HBM-bound: 256 B read + 132 B written
// per token.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "dsa_b200.h"
#include "host.h"

namespace dsa {
namespace kc {

constexpr int kDim = DSA_INDEX_DIM;                 // 128
constexpr int kPage = DSA_PAGE_SIZE;                // 64
constexpr int kPageBytes = DSA_INDEX_PAGE_BYTES;    // 8448
constexpr int kWarpsPerBlock = 8;

// 2^ceil(log2(s)) for a positive normal float, exactly: s itself when its
// mantissa is zero, else the next power of two.
__device__ __forceinline__ float pow2_ceil(float s) {
  const uint32_t u = __float_as_uint(s);
  if ((u & 0x007FFFFFu) == 0u) return s;
  return __uint_as_float((u & 0x7F800000u) + 0x00800000u);
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock)
index_cache_write_kernel(const __nv_bfloat16* __restrict__ k, const int64_t* __restrict__ slots,
                         int num_tokens, uint8_t* __restrict__ cache, int64_t num_slots,
                         int ue8m0, unsigned int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  const int64_t slot = __ldg(slots + t);
  if (slot < 0) return;  // padding
  if (slot >= num_slots) {
    if (lane == 0 && status != nullptr) atomicOr(status, DSA_DEV_BAD_INDEX);
    return;
  }
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(k + t * kDim) + lane);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale = fmaxf(1e-4f, amax) / 448.0f;
  if (ue8m0) scale = pow2_ceil(scale);
  const float v[4] = {a.x / scale, a.y / scale, b.x / scale, b.y / scale};
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v[i], __NV_SATFINITE, __NV_E4M3);
    packed |= static_cast<uint32_t>(q) << (8 * i);
  }
  uint8_t* page = cache + (slot / kPage) * kPageBytes;
  const int tok = static_cast<int>(slot % kPage);
  *reinterpret_cast<uint32_t*>(page + tok * kDim + 4 * lane) = packed;
  if (lane == 0) *reinterpret_cast<float*>(page + kPage * kDim + 4 * tok) = scale;
}

}  // namespace kc
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_index_cache_write(const void* k, const int64_t* slot_mapping, int32_t num_tokens,
                                     void* k_index_cache_fp8, int64_t num_pages, int32_t ue8m0,
                                     uint32_t* status, void* stream) {
  if (num_tokens < 0 || num_pages < 0) return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;
  if (!k || !slot_mapping || !k_index_cache_fp8) return DSA_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(k) & 7u) || (reinterpret_cast<uintptr_t>(slot_mapping) & 7u) ||
      (reinterpret_cast<uintptr_t>(k_index_cache_fp8) & 15u) ||
      (reinterpret_cast<uintptr_t>(status) & 3u))
    return DSA_ERR_MISALIGNED;
  DeviceInfo info;
  const int st = current_device_info(&info);
  if (st != DSA_OK) return st;
  const int blocks = (num_tokens + kc::kWarpsPerBlock - 1) / kc::kWarpsPerBlock;
  kc::index_cache_write_kernel<<<blocks, 32 * kc::kWarpsPerBlock, 0,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(k), slot_mapping, num_tokens,
      static_cast<uint8_t*>(k_index_cache_fp8), num_pages * kc::kPage, ue8m0 != 0,
      reinterpret_cast<unsigned int*>(status));
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}
