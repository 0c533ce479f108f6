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
// One warp per group of kTokPerWarp consecutive tokens: a lane loads 4 bf16
// (8 bytes, coalesced 256 B per warp) of every token of the group before it
// uses any, so a warp keeps 2 KB of keys in flight (80 KB per SM at the 40
// resident warps of five blocks, 48 registers a thread: 5 % faster than four
// blocks, while six spill; one token per warp left 16 KB per SM in flight);
// the warp max-reduces |k| of all the group's tokens, and each lane writes
// its 4 fp8 bytes of every token.  256 B of key + 8 B of slot read and 132 B
// written per token.  The maxima are reduce-scattered so that the lanes of
// token i (lanes 4i..4i+3) end with its maximum and compute its scale and
// reciprocal, resolve its slot (row address, validity) and, the first of
// them, store its scale: per lane one division, one reciprocal and one slot,
// not one per token.
//
// Instruction issue, not memory latency, bounded the first versions (a
// persistent kernel streaming the keys through shared memory with bulk
// copies, 128 KB in flight per SM, ran slower), and IEEE division was most
// of a token's instructions; with the steps below the kernel runs at the
// HBM bound.  k / scale is therefore computed as one correctly rounded
// reciprocal per token (__frcp_rn) and, per value, Markstein's FMA-corrected
// quotient (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
//   q0 = RN(x * r),  e = x - q0 * scale (exact, one FMA),  q = RN(q0 + e * r)
// which, with r = RN(1 / scale) and no overflow or underflow of the
// quotient, equals RN(x / scale).  Here |x / scale| <= 448 (scale >= amax/448)
// and a quotient small enough to be subnormal rounds to an fp8 zero of the
// same sign either way; the GPU tests check every byte against IEEE
// division over half a million tokens spanning 40 decades of magnitude.
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
// 8 tokens per warp at 5 blocks per SM measured fastest: 16 tokens per warp
// (3 blocks, 80 registers) was 3 % slower.
constexpr int kTokPerWarp = 8;
constexpr int kBlocksPerSm = 5;
constexpr int kLanesPerTok = 32 / kTokPerWarp;
static_assert(kTokPerWarp >= 1 && kTokPerWarp <= 32 && (kTokPerWarp & (kTokPerWarp - 1)) == 0,
              "tokens per warp: a power of two up to 32");
constexpr int kTokPerBlock = kWarpsPerBlock * kTokPerWarp;

// 2^ceil(log2(s)) for a positive normal float, exactly: s itself when its
// mantissa is zero, else the next power of two.
__device__ __forceinline__ float pow2_ceil(float s) {
  const uint32_t u = __float_as_uint(s);
  if ((u & 0x007FFFFFu) == 0u) return s;
  return __uint_as_float((u & 0x7F800000u) + 0x00800000u);
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock, kBlocksPerSm)
index_cache_write_kernel(const __nv_bfloat16* __restrict__ k, const int64_t* __restrict__ slots,
                         int num_tokens, uint8_t* __restrict__ cache, int64_t num_slots,
                         int ue8m0, unsigned int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t0 =
      (static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5)) * kTokPerWarp;
  if (t0 >= num_tokens) return;
  const int n = num_tokens - t0 < kTokPerWarp ? static_cast<int>(num_tokens - t0) : kTokPerWarp;
  // Lane l holds the slot of token t0 + l / kLanesPerTok (the lanes of one
  // token load the same word).
  const int my_tok = lane / kLanesPerTok;
  const int64_t my_slot = my_tok < n ? __ldg(slots + t0 + my_tok) : -1;
  uint2 raw[kTokPerWarp];
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i)
    raw[i] = i < n ? __ldg(reinterpret_cast<const uint2*>(k + (t0 + i) * kDim) + lane)
                   : make_uint2(0u, 0u);
  float amax[kTokPerWarp];
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].y));
    amax[i] = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
  }
  // Reduce-scatter of the kTokPerWarp maxima: at each step xor o (o = 16, 8,
  // ...) while a lane holds more than one partial maximum it keeps half of
  // them (chosen by its lane bit o) and sends the other half to its partner;
  // then plain butterfly steps finish it.  Afterwards lane l holds the
  // maximum over the warp of token l / kLanesPerTok.  max is exact and
  // order-independent.
  float cur[kTokPerWarp];
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) cur[i] = amax[i];
#pragma unroll
  for (int o = 16, half = kTokPerWarp / 2; o > 0; o >>= 1, half >>= 1) {
    const bool bit = (lane & o) != 0;
    if (half >= 1) {
#pragma unroll
      for (int j = 0; j < half; ++j) {
        const float send = bit ? cur[j] : cur[j + half];
        cur[j] = fmaxf(bit ? cur[j + half] : cur[j], __shfl_xor_sync(0xffffffffu, send, o));
      }
    } else {
      cur[0] = fmaxf(cur[0], __shfl_xor_sync(0xffffffffu, cur[0], o));
    }
  }
  const float a1 = cur[0];
  // Scale and its correctly rounded reciprocal of token lane / kLanesPerTok,
  // once per lane instead of once per lane and token.
  float my_scale = fmaxf(1e-4f, a1) / 448.0f;
  if (ue8m0) my_scale = pow2_ceil(my_scale);
  const float my_rcp = __frcp_rn(my_scale);
  // The token's slot is resolved once, by its lanes: validity (negative =
  // padding, skipped; beyond the cache = reported, skipped), its row address,
  // and the scale, which the token's first lane stores.
  const bool lead = (lane % kLanesPerTok) == 0;
  const bool valid = my_slot >= 0 && my_slot < num_slots;
  if (lead && my_slot >= num_slots && status != nullptr) atomicOr(status, DSA_DEV_BAD_INDEX);
  const int64_t my_page = valid ? my_slot / kPage : 0;
  const int my_row = valid ? static_cast<int>(my_slot % kPage) : 0;
  uint8_t* page = cache + my_page * kPageBytes;
  if (lead && valid) *reinterpret_cast<float*>(page + kPage * kDim + 4 * my_row) = my_scale;
  const unsigned long long my_rowp = reinterpret_cast<unsigned long long>(page + my_row * kDim);
  const unsigned int vmask = __ballot_sync(0xffffffffu, valid);
#pragma unroll
  for (int i = 0; i < kTokPerWarp; ++i) {
    const int src = kLanesPerTok * i;
    const float scale = __shfl_sync(0xffffffffu, my_scale, src);
    const float r = __shfl_sync(0xffffffffu, my_rcp, src);
    const unsigned long long rowp = __shfl_sync(0xffffffffu, my_rowp, src);
    if (!((vmask >> src) & 1u)) continue;  // past the end, padding or out of range
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].y));
    const float x[4] = {a.x, a.y, b.x, b.y};
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float q0 = __fmul_rn(x[j], r);
      v[j] = __fmaf_rn(__fmaf_rn(-q0, scale, x[j]), r, q0);
    }
    // Pairs convert in one instruction (round to nearest even, saturating;
    // the first element lands in the low byte).
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3);
    reinterpret_cast<uint32_t*>(rowp)[lane] = lo | (hi << 16);
  }
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
  const int64_t blocks = (static_cast<int64_t>(num_tokens) + kc::kTokPerBlock - 1) / kc::kTokPerBlock;
  kc::index_cache_write_kernel<<<static_cast<unsigned int>(blocks), 32 * kc::kWarpsPerBlock, 0,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(k), slot_mapping, num_tokens,
      static_cast<uint8_t*>(k_index_cache_fp8), num_pages * kc::kPage, ue8m0 != 0,
      reinterpret_cast<unsigned int*>(status));
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}
