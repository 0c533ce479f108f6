// attention.cu -- DSA sparse MLA attention (decode) for sm_100a.
//
// Replaces dsa_sparse_attention / run() of dsa_attention/solution/triton/kernel.py.
// The reference gathers the selected bf16 rows into an fp32 [T, 2048, 576]
// HBM buffer and runs two cuBLAS fp32 batched GEMMs around a softmax kernel
// (kernel.py:184-217).  Here each gathered row crosses HBM exactly once, as
// bf16, straight into shared memory:
//
//   attention_kernel (persistent, one CTA per SM).  The work list is
//   T x 32 tiles of 64 selected rows; CTA c takes the contiguous slice
//   [c*U/G, (c+1)*U/G) ("stream-K"), so every SM streams the same number of
//   rows whatever T is.  Roles:
//     warps 4-11 producers, two groups of four, one per stage of a 2-deep
//                ring: read the tile's 64 slot ids (one tile ahead) and copy
//                the rows' ckv (8 x 128-byte chunks) and kpe (1 chunk) with
//                16-byte cp.async into the 128-byte-swizzled K-major layout.
//                The group owning a token's first tile also loads q_nope /
//                q_pe by 2-D TMA.
//     warps 12-15 MMA issuers (tcgen05, bf16, fp32 accumulators in TMEM),
//                each issuing logits and PV in whatever order their inputs
//                become ready:
//                  S^T[64 rows, 16 heads]  = K[64, 576] . Q[16, 576]^T
//                  (M = 64, N = 16, 36 x K16; warp 12+r issues the K16 steps
//                  k = r (mod 4) into partial accumulator r), then after the
//                  softmax
//                  O^T[512, 16] += V^T[512, 64] . P^T[64, 16]
//                  (M = 128, N = 16, 4 x K16 for V^T block r); V^T is the
//                  same shared memory as the ckv chunks, read MN-major.  One
//                  thread hands tcgen05.mma to the tensor core only every
//                  ~135 cycles, so a tile's 52 MMAs are split four ways.
//     warps 0-3  online softmax in base 2 with lazy rescaling (the running
//                max is only moved when a tile exceeds it by more than 8,
//                so O in TMEM is rarely touched), P^T written as bf16.
//   A token fully covered by one CTA is normalised and written directly.
//   Otherwise each covering CTA takes a ticket from the token's arrival
//   counter when its segment ends.  Every CTA but the last to arrive writes
//   its partial (O in fp32, m, l) and then bumps the token's publication
//   counter; the last one waits until the others have published -- they
//   have all arrived already, so the wait is short and cannot depend on a
//   CTA that is not running -- and, once its own tiles are done, merges
//   them with all of its threads, its own part read straight from TMEM
//   when the token is its last segment:
//   lse = log2 L + M with L = sum_i l_i 2^(m_i - M),
//   out = sum_i O_i 2^(m_i - M) / L.
//   The counters sit at the end of the workspace; the merging CTA resets its
//   token's counters, so they are zero between calls (no memset).
#include <cuda_bf16.h>

#include <atomic>
#include <cmath>
#include <mutex>

#include "host.h"
#include "ptx.cuh"

namespace dsa {
namespace attn {

constexpr int kHeads = DSA_ATTN_HEADS;           // 16
constexpr int kCkv = DSA_CKV_DIM;                // 512
constexpr int kKpe = DSA_KPE_DIM;                // 64
constexpr int kTopK = DSA_TOPK;                  // 2048
constexpr int kRows = 64;                        // selected rows per tile
constexpr int kTilesPerTok = kTopK / kRows;      // 32
constexpr int kChunks = 9;                       // 8 ckv + 1 kpe chunks of 128 B
constexpr int kChunkBytes = kRows * 128;         // 8192
constexpr int kStageBytes = kChunks * kChunkBytes;  // 73728
constexpr int kQChunkBytes = kHeads * 128;       // 2048
constexpr int kQBytes = kChunks * kQChunkBytes;  // 18432
constexpr int kPBytes = kHeads * kRows * 2;      // 2048
constexpr int kSoftWarp0 = 0;                    // warps 0-3: online softmax
constexpr int kProdWarp0 = 4;                    // warps 4-11: gather producers
constexpr int kProdWarps = 8;
constexpr int kMmaWarp0 = 12;                    // warps 12-15: MMA issuers (12 owns TMEM)
constexpr int kMmaWarps = 4;
constexpr int kThreads = 512;
constexpr int kTmemCols = 256;
constexpr uint32_t kColO = 0;    // O^T buffers at [0,64) and [64,128): 4 blocks x 16 heads
constexpr uint32_t kColS = 128;  // S^T buffers at [128,192) and [192,256): 4 partial sums x 16 heads
constexpr float kRescaleThreshold = 8.0f;  // log2 units: factor 256
constexpr unsigned long long kSecondTileDelayNs = 1000;
constexpr int kMaxTokens = (1 << 30) / (kTopK / kRows) / kHeads;
// Most parts a token can have (its 32 tiles meet at most 33 CTA slices); the
// merge scratch holds the parts' per-head weights ([kMaxParts][16] floats)
// and record indices.
constexpr int kMaxParts = 48;
// A partial record: the part's O^T in fp32 as float4s of 4 heads,
// [4 column blocks mb][4 head quads q][128 dims][4 heads]: thread e of the
// softmax warps (dims 128 mb + e, all heads) writes float4 (mb, q, e), and
// consecutive threads touch consecutive 16 bytes, both when a part is
// published and when it is merged.
constexpr int kPartFloats = 4 * 128 * kHeads;  // 8192 floats = 32 KiB
__device__ __forceinline__ int part_index(int mb, int q, int dim_in_block) {
  return (mb * 4 + q) * 128 + dim_in_block;  // float4 index inside a record
}
// Only a CTA's first and last token segments can be partial: two records
// per CTA, slot 0 for its first segment and slot 1 for its last.
constexpr int kRecsPerCta = 2;
// Parts whose records one merging thread loads at once (16 floats each)
// when they do not fit the landing area.
constexpr int kMergeBatch = 2;
// Parts that land in the idle K/V stage ring (32 KiB each) during a merge.
constexpr int kLandParts = 4;
static_assert(kLandParts * kPartFloats * 4 <= 2 * kStageBytes, "landing area");
// Merge scratch in shared memory: per part and head the max m and sum l
// (then the weight), and a flag.
constexpr int kMergeScratchBytes = 2 * (kMaxParts * kHeads * 4) + 16;
// Parts of the CTA's first (slot 0) and last (slot 1) token, the only ones
// it can merge: per slot the first covering CTA, the part count and each
// part's record index, computed while the first tile is in flight.
struct MergeParts {
  int c_lo[2];
  int nparts[2];
  int64_t rec[2][kMaxParts];
};

// bf16 x bf16 -> f32.  Logits: A = K rows (K-major), B = Q (K-major), M64 N16.
constexpr uint32_t kIdescS = idesc_make(1, 1, false, false, 64, 16);
// PV: A = V^T (MN-major view of the ckv chunks), B = P^T (K-major), M128 N16.
constexpr uint32_t kIdescO = idesc_make(1, 1, true, false, 128, 16);

constexpr int kOffStage = 0;
constexpr int kOffQ = kOffStage + 2 * kStageBytes;   // 147456
constexpr int kOffP = kOffQ + 2 * kQBytes;           // 184320
constexpr int kOffSx = kOffP + 2 * kPBytes;          // 188416
constexpr int kOffBar = kOffSx + kHeads * kRows * 4; // 192512
constexpr int kOffMisc = kOffBar + 256;
constexpr int kOffParts = kOffMisc + 256;
constexpr int kSmemBytes = 1024 + kOffParts + static_cast<int>(sizeof(MergeParts));
static_assert((18 + kMmaWarps + 2) * 8 <= 256, "barrier area");
static_assert(kOffSx == kOffP + 2 * kPBytes && 2 * kPBytes + kHeads * kRows * 4 >= kMergeScratchBytes,
              "the P and Sx buffers, contiguous, hold the merge scratch");

// Test-only fault injection (dsa_b200_test_inject): the producer group of
// each CTA's second tile issues no copy and no arrival for it, so the MMA
// issuers' wait on that tile runs out and the CTA aborts.
constexpr int kInjectNone = 0;
constexpr int kInjectSkipArrival = DSA_TEST_SKIP_ARRIVAL;

struct Params {
  const int32_t* indices;
  const uint8_t* ckv;      // [num_slots][512] bf16
  const uint8_t* kpe;      // [num_slots][64] bf16
  __nv_bfloat16* out;
  float* lse;
  float* part_o;   // [grid * 2][kPartFloats]: a part's O^T (not normalised)
  float* part_ml;  // [grid * 2][16][2]: the part's (m, l)
  int* tok_arrive;  // [num_tokens] tickets taken; zero between calls (the merging CTA resets it)
  int* tok_pub;     // [num_tokens] partials published; likewise
  unsigned int* status;
  int64_t num_slots;
  int num_tokens;
  float scale_log2;
  unsigned long long wait_limit_ns;  // kWaitLimitNs unless a test shortened it
  int inject;                        // kInjectNone unless a test asked for a fault
};

// Which tokens / records a CTA covers, shared by both kernels.
// floor(total * c / grid) in double precision: total * c < 2^53 is exact and
// a non-integral quotient lies at least 1/grid from an integer, far above the
// rounding error, so the floor is exact -- and much cheaper on the GPU than
// a 64-bit integer division.
__host__ __device__ inline int64_t unit_start(int64_t total, int c, int grid) {
  return static_cast<int64_t>(static_cast<double>(total) * c / grid);
}

// CTAs c whose unit range [start(c), start(c+1)) meets token t's units.
__device__ __forceinline__ void covering_ctas(int t, int64_t total, int grid, int& c_lo, int& c_hi) {
  // The CTA holding unit x is the largest c with start(c) <= x, i.e.
  // floor(((x + 1) * grid - 1) / total) (every CTA holds >= 1 unit); exact
  // in double precision like unit_start.
  const int64_t a = static_cast<int64_t>(t) * kTilesPerTok, z = a + kTilesPerTok;
  const double dt = static_cast<double>(total);
  c_lo = static_cast<int>(static_cast<double>((a + 1) * grid - 1) / dt);
  c_hi = static_cast<int>(static_cast<double>(z * grid - 1) / dt);
  if (c_hi > grid - 1) c_hi = grid - 1;
}

__device__ __forceinline__ int parts_of(int t, int64_t total, int grid) {
  int lo, hi;
  covering_ctas(t, total, grid, lo, hi);
  return hi - lo + 1;
}

// Record of CTA c's part of token t: slot 0 if t is c's first token
// segment, else slot 1 (its last).
__device__ __forceinline__ int64_t part_record(int t, int c, int64_t total, int grid) {
  const int tf = static_cast<int>(unit_start(total, c, grid) / kTilesPerTok);
  return static_cast<int64_t>(c) * kRecsPerCta + (t == tf ? 0 : 1);
}

// Writes 16 heads of output dim `dim` of token t (bf16).
__device__ __forceinline__ void store_out_column(const Params& p, int t, int dim, const float (&acc)[16]) {
  __nv_bfloat16* out = p.out + static_cast<int64_t>(t) * kHeads * kCkv + dim;
#pragma unroll
  for (int hh = 0; hh < kHeads; ++hh) out[hh * kCkv] = __float2bfloat16_rn(acc[hh]);
}

// Merges split token t once this CTA's own work is done, with all kThreads
// threads.  Parts are the covering CTAs c_lo..c_hi in order; every part's
// O^T and (m, l) come from its record, except this CTA's own part when
// `own_obuf` names the TMEM columns of its last segment's O^T accumulator
// (own_ml: its (m, l) per head), in which case it never left the SM.  Waits
// (bounded) until the other parts have published.  The weights
// w_i = 2^(m_i - M) / L per head and the weighted sums run in part order,
// so the result does not depend on which CTA merges:
//   lse = M + log2 L, L = sum_i l_i 2^(m_i - M), out = sum_i w_i O_i.
// Up to kLandParts parts' records are brought into `landing` (the idle K/V
// stage ring) by one bulk copy each (thread 0), completing on `land_bar`
// (phase `land_parity`), while warps 2-3 load the weights' (m, l); more
// parts (small token counts) are read from L2 kMergeBatch parts at a time.
// The parts' record indices come precomputed in `parts` (slot `slot`).
// Thread -> warp w reads TMEM sub-partition w & 3 (dims 32 (w & 3) + lane of
// each 128-dim block) and block mb = w >> 2: one output dim, 16 heads.
// Returns whether the landing barrier was used (its phase then advanced).
__device__ bool merge_at_end(const Params& p, int t, const MergeParts& parts, int slot, int own_obuf,
                             const float* own_ml, uint32_t tmem_base, uint8_t* scratch, uint8_t* landing,
                             uint64_t* land_bar, uint32_t land_parity) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nparts = parts.nparts[slot];
  float* wm = reinterpret_cast<float*>(scratch);          // [kMaxParts][16] m, then weights
  float* wl = wm + kMaxParts * kHeads;                     // [kMaxParts][16] l
  int* flag = reinterpret_cast<int*>(wl + kMaxParts * kHeads);
  if (nparts > kMaxParts) {  // cannot happen for grids of <= 2^20 CTAs; never read past scratch
    if (tid == 0) atomicOr(p.status, DSA_DEV_BAD_INDEX);
    return false;
  }
  const bool own_tmem = own_obuf >= 0;
  // Part i's record index, or -1 for this CTA's own part kept in TMEM.
  const int own_i = own_tmem ? static_cast<int>(blockIdx.x) - parts.c_lo[slot] : -1;
  auto rec = [&](int i) -> int64_t { return i == own_i ? -1 : parts.rec[slot][i]; };
  const bool land = nparts <= kLandParts;
  if (tid == 0) {
    const bool ok = wait_counter_at_least(p.tok_pub + t, own_tmem ? nparts - 1 : nparts, p.status,
                                          2 * p.wait_limit_ns);
    *flag = ok ? 1 : 0;
    if (land && !ok) mbar_arrive_expect_tx(land_bar, 0);  // completes the phase at once
  }
  __syncthreads();  // flag
  if (land && tid == 0 && *flag) {
    // The acquire above made the records visible to this thread; the proxy
    // fence extends that to its bulk copies.
    fence_proxy_async_global();
    uint32_t bytes = 0;
    for (int i = 0; i < nparts; ++i) bytes += rec(i) >= 0 ? kPartFloats * 4 : 0;
    mbar_arrive_expect_tx(land_bar, bytes);  // completes the phase at once when nothing is copied
    for (int i = 0; i < nparts; ++i)
      if (rec(i) >= 0)
        bulk_load(landing + i * kPartFloats * 4, p.part_o + rec(i) * kPartFloats, kPartFloats * 4, land_bar);
  }
  const int sp = warp & 3, mb = warp >> 2;
  const int de = 32 * sp + lane;  // dim inside the 128-dim block
  if (*flag && tid >= 64 && tid < 64 + kHeads) {
    // (m, l) of every part, eight parts' loads in flight at a time (warps
    // 2-3, beside thread 0's bulk copies).
    const int e = tid - 64;
    float M = -INFINITY;
    for (int i0 = 0; i0 < nparts; i0 += 8) {
      float mv[8], lv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k;
        mv[k] = -INFINITY;
        lv[k] = 0.f;
        if (i < nparts) {
          const int64_t r = rec(i);
          if (r < 0) {
            mv[k] = own_ml[2 * e];
            lv[k] = own_ml[2 * e + 1];
          } else {
            mv[k] = __ldcg(p.part_ml + r * 2 * kHeads + 2 * e);
            lv[k] = __ldcg(p.part_ml + r * 2 * kHeads + 2 * e + 1);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (i0 + k < nparts) {
          wm[(i0 + k) * kHeads + e] = mv[k];
          wl[(i0 + k) * kHeads + e] = lv[k];
          M = fmaxf(M, mv[k]);
        }
      }
    }
    float L = 0.f;
    for (int i = 0; i < nparts; ++i) {
      const float m = wm[i * kHeads + e];
      const float w = m == -INFINITY ? 0.f : exp2f(m - M);
      L += wl[i * kHeads + e] * w;
      wm[i * kHeads + e] = w;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int i = 0; i < nparts; ++i) wm[i * kHeads + e] *= inv;
    p.lse[static_cast<int64_t>(t) * kHeads + e] = L > 0.f ? M + log2f(L) : -INFINITY;
  }
  // Every thread waits for the landing (bounded; a copy cannot hang, this
  // only guards the bookkeeping) before the weights barrier.
  if (land) mbar_drain(land_bar, land_parity, p.status);
  __syncthreads();  // weights
  if (*flag) {
    float own[16];
    if (own_tmem) {
      tc_fence_after();
      tmem_ld16(tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + own_obuf + 16 * mb, own);
      tmem_wait_ld();
    }
    float acc[16];
#pragma unroll
    for (int hh = 0; hh < kHeads; ++hh) acc[hh] = 0.f;
    auto add = [&](const float4 (&v)[4], int i) {
      const float4* wv = reinterpret_cast<const float4*>(wm + i * kHeads);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w = wv[q];
        acc[4 * q] = fmaf(v[q].x, w.x, acc[4 * q]);
        acc[4 * q + 1] = fmaf(v[q].y, w.y, acc[4 * q + 1]);
        acc[4 * q + 2] = fmaf(v[q].z, w.z, acc[4 * q + 2]);
        acc[4 * q + 3] = fmaf(v[q].w, w.w, acc[4 * q + 3]);
      }
    };
    if (land) {
      for (int i = 0; i < nparts; ++i) {
        float4 v[4];
        if (rec(i) < 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = make_float4(own[4 * q], own[4 * q + 1], own[4 * q + 2], own[4 * q + 3]);
        } else {
          const float4* f = reinterpret_cast<const float4*>(landing + i * kPartFloats * 4);
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q] = f[part_index(mb, q, de)];
        }
        add(v, i);
      }
    } else {
      for (int i0 = 0; i0 < nparts; i0 += kMergeBatch) {
        float4 v[kMergeBatch][4];
#pragma unroll
        for (int k = 0; k < kMergeBatch; ++k) {
          const int i = i0 + k;
          if (i < nparts && rec(i) >= 0) {
            const float4* src = reinterpret_cast<const float4*>(p.part_o + rec(i) * kPartFloats);
#pragma unroll
            for (int q = 0; q < 4; ++q) v[k][q] = __ldcg(src + part_index(mb, q, de));
          } else if (i < nparts) {
#pragma unroll
            for (int q = 0; q < 4; ++q) v[k][q] = make_float4(own[4 * q], own[4 * q + 1], own[4 * q + 2], own[4 * q + 3]);
          }
        }
#pragma unroll
        for (int k = 0; k < kMergeBatch; ++k)
          if (i0 + k < nparts) add(v[k], i0 + k);
      }
    }
    store_out_column(p, t, 128 * mb + de, acc);
  }
  if (tid == 0) {  // the token's counters are zero again for the next call
    p.tok_arrive[t] = 0;
    p.tok_pub[t] = 0;
  }
  return land;
}

__device__ __forceinline__ int sanitize_slot(int v, int64_t num_slots, unsigned int* status) {
  if (v < 0 || v >= num_slots) {
    if (v != -1) atomicOr(status, DSA_DEV_BAD_INDEX);
    return 0;
  }
  return v;
}

__global__ void __launch_bounds__(kThreads, 1)
attention_kernel(const __grid_constant__ CUtensorMap ckv_map,
                 const __grid_constant__ CUtensorMap kpe_map,
                 const __grid_constant__ CUtensorMap qn_map,
                 const __grid_constant__ CUtensorMap qp_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stage_mem = smem + kOffStage;
  uint8_t* q_mem = smem + kOffQ;
  uint8_t* p_mem = smem + kOffP;
  float* sx = reinterpret_cast<float*>(smem + kOffSx);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 2;
  uint64_t* q_full = bars + 4;
  uint64_t* q_empty = bars + 6;
  uint64_t* s_full = bars + 8;
  uint64_t* s_empty = bars + 10;
  uint64_t* p_full = bars + 12;
  uint64_t* p_empty = bars + 14;
  uint64_t* o_empty = bars + 16;
  uint64_t* drain = bars + 18;  // one per MMA warp
  // Single-use: completes when the CTA's first tile has landed (group 0).
  uint64_t* first_full = bars + 18 + kMmaWarps;
  // Merges: the bulk copies of other parts' records into the stage ring.
  uint64_t* land_bar = bars + 19 + kMmaWarps;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + kOffMisc + 4);
  int* ticket_smem = reinterpret_cast<int*>(smem + kOffMisc + 8);
  // count, then <= 2 (token, TMEM column of the own part's O^T or -1) pairs
  int* merge_list = reinterpret_cast<int*>(smem + kOffMisc + 12);
  int* q_last = reinterpret_cast<int*>(smem + kOffMisc + 32);      // last segment loaded per Q slot
  float* alpha_smem = reinterpret_cast<float*>(smem + kOffMisc + 64);   // 16
  float* ml_smem = reinterpret_cast<float*>(smem + kOffMisc + 128);     // 16 x (m, l)
  MergeParts* mparts = reinterpret_cast<MergeParts*>(smem + kOffParts);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 32 * kProdWarps / 2); mbar_init(&kv_empty[s], kMmaWarps);
      mbar_init(&q_full[s], 1);  mbar_init(&q_empty[s], kMmaWarps);
      mbar_init(&s_full[s], kMmaWarps);  mbar_init(&s_empty[s], 128);
      mbar_init(&p_full[s], 128);  mbar_init(&p_empty[s], kMmaWarps);
      mbar_init(&o_empty[s], 1);
    }
    for (int w = 0; w < kMmaWarps; ++w) mbar_init(&drain[w], 1);
    mbar_init(first_full, 32 * kProdWarps / 2);
    mbar_init(land_bar, 1);
    *abort_flag = 0;
    merge_list[0] = 0;
    q_last[0] = q_last[1] = -1;
    fence_mbar_init();
  }
  if (warp == kProdWarp0 && lane == 0) {
    prefetch_tensor_map(&ckv_map); prefetch_tensor_map(&kpe_map);
    prefetch_tensor_map(&qn_map);  prefetch_tensor_map(&qp_map);
  }
  if (warp == kMmaWarp0) tmem_alloc(tmem_base_smem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched programmatically after the indexer's select kernel: global
  // memory is touched only once the previous grid has completed.
  griddep_wait();

  const uint32_t tmem_base = *tmem_base_smem;
  const int64_t total = static_cast<int64_t>(p.num_tokens) * kTilesPerTok;
  const int64_t u0 = unit_start(total, blockIdx.x, gridDim.x);
  const int64_t u1 = unit_start(total, blockIdx.x + 1, gridDim.x);
  const int n = static_cast<int>(u1 - u0);
  const int t_first = static_cast<int>(u0 / kTilesPerTok);
  const WaitCtx wctx{abort_flag, p.status, p.wait_limit_ns};

  if (warp >= kProdWarp0 && warp < kProdWarp0 + kProdWarps) {
    // ------------------------------------------------------ producer warps
    // Two groups of four warps; group g fills stage g with the rows of tiles
    // i = g, g+2, ... by 16-byte cp.async straight into the 128-byte-swizzled
    // K-major layout the MMAs read (piece j of row r lands at
    // r*128 + ((j ^ (r & 7)) << 4) of its chunk).  Thread (warp wl of the
    // group, lane l) copies piece l & 7 of rows 16*wl + 4*q + (l >> 3),
    // q = 0..3, in all 9 chunks: 36 copies, each warp instruction moving
    // four 128-byte row pieces.  These are ordinary load/store-unit
    // instructions, so a tile's copies are issued in a few hundred cycles
    // (a thread hands TMA gather4 ops over only every ~100 cycles).  The
    // thread then waits for its copies, makes them visible to the tensor
    // core's async proxy and arrives on the stage's barrier.  The warp with
    // wl == 0 of the group that owns a token segment's first tile also
    // loads that token's q_nope / q_pe by 2-D TMA.
    const int w = warp - kProdWarp0;
    const int g = w >> 2;
    const int wl = w & 3;
    const int j = lane & 7;
    const int rsub = lane >> 3;
    const uint64_t policy = make_policy_evict_first();
    const uint32_t st_s = smem_u32(stage_mem + g * kStageBytes);
    auto load_idx = [&](int i, int (&v)[4]) {
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = 0;
      if (i < n) {
        const int64_t u = u0 + i;
        const int32_t* r = p.indices + (u / kTilesPerTok) * kTopK + (u % kTilesPerTok) * kRows + 16 * wl + rsub;
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = __ldg(r + 4 * q);
      }
    };
    int v[4];
    load_idx(g, v);
    int i = g;
    for (; i < n; i += 2) {
      const int64_t u = u0 + i;
      const int t = static_cast<int>(u / kTilesPerTok);
      const int tile = static_cast<int>(u % kTilesPerTok);
      int nv[4];
      load_idx(i + 2, nv);  // this group's next tile's slot ids, in flight meanwhile
      if (wl == 0 && (i == 0 || tile == 0)) {
        const int seg = t - t_first;
        const int slot = seg & 1;
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(&q_empty[slot], ((seg >> 1) & 1) ^ 1, wctx);
          if (ok) {
            mbar_arrive_expect_tx(&q_full[slot], kQBytes);
            uint8_t* q = q_mem + slot * kQBytes;
            for (int c = 0; c < 8; ++c)
              tma_load_2d(q + c * kQChunkBytes, &qn_map, &q_full[slot], c * 64, t * kHeads);
            tma_load_2d(q + 8 * kQChunkBytes, &qp_map, &q_full[slot], 0, t * kHeads);
            atomicMax(&q_last[slot], seg);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      const int s = g;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[s], ((i >> 1) & 1) ^ 1, wctx))) break;
      // With every SM starting at once, the first tile lands sooner when
      // the second one's rows are requested a little later: give the first
      // tile a head start of up to kSecondTileDelayNs (an ordering hint;
      // running out is not an error).
      if (i == 1) mbar_wait_at_most(first_full, 0, kSecondTileDelayNs);
      // Test only: the second tile is neither copied nor announced.
      if (!(i == 1 && p.inject == kInjectSkipArrival)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int row = 16 * wl + 4 * q + rsub;
          const int64_t slotid = sanitize_slot(v[q], p.num_slots, p.status);
          const uint8_t* ck = p.ckv + slotid * (kCkv * 2) + 16 * j;
          const uint32_t dst = st_s + row * 128 + ((j ^ (row & 7)) << 4);
#pragma unroll
          for (int c = 0; c < 8; ++c) cp_async16(dst + c * kChunkBytes, ck + 128 * c, policy);
          cp_async16(dst + 8 * kChunkBytes, p.kpe + slotid * (kKpe * 2) + 16 * j, policy);
        }
        cp_async_wait_all();
        fence_proxy_async_smem();
        mbar_arrive(&kv_full[s]);
        if (i == 0) mbar_arrive(first_full);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = nv[q];
    }
    cp_async_wait_all();  // copies of an aborted tile land before the CTA can exit
  } else if (warp >= kMmaWarp0) {
    // ------------------------------------------------------ MMA issuers
    // Logits of tile i need its gathered rows, its token's Q and a free S
    // buffer; PV of tile i needs P(i) (and, at a segment start, a drained O
    // buffer).  Both are polled and issued as soon as ready (PV first), so
    // PV(i) never waits behind the next tile's gather or logits.  Warp 12+r issues the logits K16
    // steps k = r (mod 4) (partial accumulator r) and the PV of V^T block r.
    const int r = warp - kMmaWarp0;
    if (lane == 0 && n > 0) {
      // Descriptors of stage / Q / P buffer 0; buffer 1 is a fixed byte offset away.
      const uint64_t st_desc0 = sdesc_sw128(smem_u32(stage_mem), 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(stage_mem), kChunkBytes, 1024);
      const uint64_t q_desc0 = sdesc_sw128(smem_u32(q_mem), 16, 1024);
      const uint64_t p_desc0 = sdesc_sw128(smem_u32(p_mem), 16, 1024);
      int nl = 0, np = 0;
      unsigned long long t_idle = 0;
      while (np < n) {
        bool progressed = false;
        // PV first: it frees the K/V stage the gather of tile np + 2 waits for.
        if (np < nl) {
          const int64_t u = u0 + np;
          const int tile = static_cast<int>(u % kTilesPerTok);
          const int seg = static_cast<int>(u / kTilesPerTok) - t_first;
          const bool seg_start = (np == 0 || tile == 0);
          const int s = np & 1;
          if (mbar_test(&p_full[s], (np >> 1) & 1) &&
              (!seg_start || mbar_test(&o_empty[seg & 1], ((seg >> 1) & 1) ^ 1))) {
            tc_fence_after();
            const uint32_t obuf = tmem_base + kColO + 64u * (seg & 1);
#pragma unroll
            for (int kk = 0; kk < kRows / 16; ++kk) {
              // V^T block r: chunks 2r, 2r+1; K16 step = 16 rows = 2048 bytes
              umma_bf16(obuf + 16 * r,
                        v_desc0 + s * (kStageBytes >> 4) + r * (2 * kChunkBytes >> 4) + kk * (2048 >> 4),
                        p_desc0 + s * (kPBytes >> 4) + kk * 2, kIdescO, (seg_start && kk == 0) ? 0u : 1u);
            }
            umma_commit(&kv_empty[s]);
            umma_commit(&p_empty[s]);
            ++np;
            progressed = true;
          }
        }
        if (nl < n) {
          const int64_t u = u0 + nl;
          const int tile = static_cast<int>(u % kTilesPerTok);
          const int seg = static_cast<int>(u / kTilesPerTok) - t_first;
          const bool seg_start = (nl == 0 || tile == 0);
          const bool seg_end = (nl == n - 1 || tile == kTilesPerTok - 1);
          const int s = nl & 1;
          if ((!seg_start || mbar_test(&q_full[seg & 1], (seg >> 1) & 1)) &&
              mbar_test(&kv_full[s], (nl >> 1) & 1) &&
              mbar_test(&s_empty[s], ((nl >> 1) & 1) ^ 1)) {
            tc_fence_after();
            const uint64_t ad = st_desc0 + s * (kStageBytes >> 4);
            const uint64_t bd = q_desc0 + (seg & 1) * (kQBytes >> 4);
            const uint32_t d = tmem_base + kColS + 64u * s;
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
              // K16 step k = 4c + r -> partial accumulator r.  Descriptor
              // offsets: +8192 bytes per 64-column chunk, +32 bytes per K16
              // step (>> 4).
              umma_bf16(d + 16 * r, ad + c * (kChunkBytes >> 4) + r * 2,
                        bd + c * (kQChunkBytes >> 4) + r * 2, kIdescS, c > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[s]);
            if (seg_end) umma_commit(&q_empty[seg & 1]);
            ++nl;
            progressed = true;
          }
        }
        if (progressed) {
          t_idle = 0;
        } else {
          if (*abort_flag) break;
          const unsigned long long now = global_timer_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > p.wait_limit_ns) {
            *abort_flag = 1;
            atomicOr(p.status, DSA_DEV_WAIT_TIMEOUT);
            break;
          }
        }
      }
      umma_commit(&drain[r]);
      mbar_drain(&drain[r], 0, p.status);
    }
  } else {
    // ------------------------------------------------------ softmax warps
    // Thread (warp sp, lane) reads S^T row 16 sp + (lane & 15) (the M = 64
    // accumulator occupies TMEM lanes 0-15 of each sub-partition) straight
    // from TMEM -- no shared-memory transpose and, in the common case, one
    // barrier per tile; lane L < 16 weights heads 0-7 of its row and lane
    // L + 16 heads 8-15 of the same row.  The running max m_run[h] is the same in
    // every thread; it moves only when some row of the tile exceeds it by more
    // than kRescaleThreshold (always at a segment's first tile), which the
    // threads learn from one OR-reduction barrier; only then is the tile's
    // per-head max reduced across the rows.  The softmax denominators are
    // kept per row (l_row[h]) and summed over the rows once per segment.
    // Every bounded wait's result joins the tile's reduction barrier, so the
    // 128 threads always meet the same barriers and leave the loop together if
    // a wait gave up.
    const int sp = warp & 3;
    const int e = tid - 32 * kSoftWarp0; // 0..127
    const bool row_lane = lane < 16;
    const uint32_t lane_base = static_cast<uint32_t>(sp * 32) << 16;
    const int srow = 16 * sp + (lane & 15);  // S^T row held by this thread (lane < 16)
    float* red = sx;  // reduction scratch: tile maxima [2][4 warps][16 heads], row sums [4][16]
    const int h0 = (lane >> 4) * 8;           // first of this lane's 8 heads
    {
      // Record indices of the parts of this CTA's first and last tokens,
      // worked out while the first tile is on its way (the merges at the
      // end then start at once).  Read after the CTA's closing barrier.
      const int slot = e >> 6, ip = e & 63;
      const int tt = static_cast<int>((slot == 0 ? u0 : u0 + n - 1) / kTilesPerTok);
      int c_lo, c_hi;
      covering_ctas(tt, total, gridDim.x, c_lo, c_hi);
      const int np = c_hi - c_lo + 1;
      if (ip == 0) {
        mparts->c_lo[slot] = c_lo;
        mparts->nparts[slot] = np;
      }
      if (ip < np && ip < kMaxParts) mparts->rec[slot][ip] = part_record(tt, c_lo + ip, total, gridDim.x);
    }
    float m_run[kHeads], l_row[8];
    int sg = -1, seg_first_tile = 0;
    int owed_t = -1, owed_tk = 0;  // (thread 0) a ticket taken whose part is not settled yet
    // A part written at a segment end whose publication waits for the next
    // tile's first barrier: by then its stores have long completed, so the
    // fence that orders them before the count no longer stalls the group.
    int pub_t = -1;
    bool ok = true;
    int i = 0;
    for (; i < n; ++i) {
      const int64_t u = u0 + i;
      const int t = static_cast<int>(u / kTilesPerTok);
      const int tile = static_cast<int>(u % kTilesPerTok);
      const bool seg_start = (i == 0 || tile == 0);
      const bool seg_end = (i == n - 1 || tile == kTilesPerTok - 1);
      if (seg_start) {
        ++sg;
        seg_first_tile = tile;
#pragma unroll
        for (int hh = 0; hh < kHeads; ++hh) m_run[hh] = -INFINITY;
#pragma unroll
        for (int k = 0; k < 8; ++k) l_row[k] = 0.f;
      }
      const int s = i & 1;
      const int idx = __ldg(p.indices + static_cast<int64_t>(t) * kTopK + tile * kRows + srow);
      const bool valid = row_lane && idx >= 0 && idx < p.num_slots;

      ok = mbar_wait(&s_full[s], (i >> 1) & 1, wctx) && ok;
      tc_fence_after();
      float x[kHeads];
      {
        float lo[32], hi[32];
        tmem_ld32(tmem_base + lane_base + kColS + 64u * s, lo);
        tmem_ld32(tmem_base + lane_base + kColS + 64u * s + 32, hi);
        tmem_wait_ld();
#pragma unroll
        for (int hh = 0; hh < kHeads; ++hh)
          x[hh] = valid ? ((lo[hh] + lo[16 + hh]) + (hi[hh] + hi[16 + hh])) * p.scale_log2 : -INFINITY;
      }
      tc_fence_before();
      mbar_arrive(&s_empty[s]);
      bool need = false;
#pragma unroll
      for (int hh = 0; hh < kHeads; ++hh) need |= x[hh] > m_run[hh] + kRescaleThreshold;
      if (pub_t >= 0) __threadfence();
      const bool slow = named_barrier_or(1, 128, need || !ok);
      if (pub_t >= 0) {
        if (e == 0) atomicAdd(p.tok_pub + pub_t, 1);
        pub_t = -1;
      }
      if (slow) {
        // ---- slow path: a wait gave up, or the running max moves.
        if (!named_barrier_and(1, 128, ok)) break;
        // Per-head tile max: a warp max (redux on order-preserving keys),
        // then the four warps' maxima through shared memory.  The scratch
        // half alternates with the tile, so the next slow path cannot
        // overwrite it before every thread has read it.
        float* rmax = red + 64 * (i & 1);
#pragma unroll
        for (int hh = 0; hh < kHeads; ++hh) {
          const uint32_t k = __reduce_max_sync(0xffffffffu, float_order_key(x[hh]));
          if (lane == 0) rmax[sp * kHeads + hh] = float_from_order_key(k);
        }
        named_barrier_sync(1, 128);
        bool any_alpha = false;
        float alpha[kHeads];
#pragma unroll
        for (int hh = 0; hh < kHeads; ++hh) {
          const float mt = fmaxf(fmaxf(rmax[hh], rmax[kHeads + hh]), fmaxf(rmax[2 * kHeads + hh], rmax[3 * kHeads + hh]));
          alpha[hh] = 1.f;
          if (mt > m_run[hh] + kRescaleThreshold) {
            alpha[hh] = exp2f(m_run[hh] - mt);  // 0 when m_run == -inf
            m_run[hh] = mt;
            any_alpha = true;
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) l_row[k] *= lane < 16 ? alpha[k] : alpha[8 + k];
        if (any_alpha && !seg_start) {
          // O must hold PV(i-1) before it is rescaled (same segment: i >= 1).
          ok = mbar_wait(&p_empty[(i - 1) & 1], ((i - 1) >> 1) & 1, wctx) && ok;
          tc_fence_after();
          const uint32_t obuf = tmem_base + lane_base + kColO + 64u * (sg & 1);
#pragma unroll
          for (int mb = 0; mb < 4; ++mb) {
            float o[16];
            tmem_ld16(obuf + 16 * mb, o);
            tmem_wait_ld();
#pragma unroll
            for (int hh = 0; hh < kHeads; ++hh) o[hh] *= alpha[hh];
            tmem_st16(obuf + 16 * mb, o);
          }
          tmem_wait_st();
        }
      }
      // P buffer s was last read by the PV of tile i-2.
      if (i >= 2) ok = mbar_wait(&p_empty[s], ((i - 2) >> 1) & 1, wctx) && ok;
      {
        // Lane L + 16 takes heads 8-15 of lane L's row.
        float xs[8], ms[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float hi = __shfl_sync(0xffffffffu, x[8 + k], lane & 15);
          xs[k] = lane < 16 ? x[k] : hi;
          ms[k] = lane < 16 ? m_run[k] : m_run[8 + k];
        }
        // P^T, K-major 128-byte swizzled: head h's 64 rows are 128 bytes,
        // 16-byte piece g holds rows 8g .. 8g + 7.
        uint8_t* pb = p_mem + s * kPBytes + (h0 >> 3) * 1024 + (srow & 7) * 2;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float pr = ms[k] == -INFINITY ? 0.f : ex2_approx(xs[k] - ms[k]);
          l_row[k] += pr;
          *reinterpret_cast<__nv_bfloat16*>(pb + k * 128 + (((srow >> 3) ^ k) << 4)) = __float2bfloat16_rn(pr);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[s]);

      if (seg_end) {
        // ---- finalise the segment.  A split token's ticket is requested
        // before the wait for the segment's last PV, so the atomic's round
        // trip overlaps it.
        const bool whole = (seg_first_tile == 0 && tile == kTilesPerTok - 1);
        int ticket = 0;
        if (!whole && e == 0) {
          ticket = atomicAdd(p.tok_arrive + t, 1);
          owed_t = t;
          owed_tk = ticket;
        }
        ok = mbar_wait(&p_empty[s], (i >> 1) & 1, wctx) && ok;
        tc_fence_after();
        // Per-head denominators: the row sums added over the 64 rows (lanes
        // 0-15 hold heads 0-7, lanes 16-31 heads 8-15).
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float v = l_row[k];
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          if ((lane & 15) == 0) red[128 + sp * kHeads + h0 + k] = v;
        }
        if (e == 0) {
          *ticket_smem = ticket;
#pragma unroll
          for (int hh = 0; hh < kHeads; ++hh) ml_smem[2 * hh] = m_run[hh];
        }
        if (!named_barrier_and(1, 128, ok)) break;
        if (e < kHeads)
          ml_smem[2 * e + 1] = (red[128 + e] + red[128 + kHeads + e]) + (red[128 + 2 * kHeads + e] + red[128 + 3 * kHeads + e]);
        named_barrier_sync(1, 128);
        const int col = 32 * sp + lane;  // == e: this thread's dims are 128 mb + col
        const uint32_t obuf = tmem_base + lane_base + kColO + 64u * (sg & 1);
        if (whole) {
          if (e < kHeads) {  // 1 / l per head, for every thread
            const float l = ml_smem[2 * e + 1];
            alpha_smem[e] = l > 0.f ? 1.f / l : 0.f;
          }
          named_barrier_sync(1, 128);
#pragma unroll 1
          for (int mb = 0; mb < 4; ++mb) {
            float o[16];
            tmem_ld16(obuf + 16 * mb, o);
            tmem_wait_ld();
#pragma unroll
            for (int hh = 0; hh < kHeads; ++hh) o[hh] *= alpha_smem[hh];
            store_out_column(p, t, 128 * mb + col, o);
          }
          if (e < kHeads) {
            const float l = ml_smem[2 * e + 1];
            p.lse[static_cast<int64_t>(t) * kHeads + e] = l > 0.f ? ml_smem[2 * e] + log2f(l) : -INFINITY;
          }
        } else {
          const int slot = t == static_cast<int>(u0 / kTilesPerTok) ? 0 : 1;
          const int parts = mparts->nparts[slot];
          const int own = static_cast<int>(blockIdx.x) - mparts->c_lo[slot];
          const int tk = *ticket_smem;
          if (tk >= parts) {
            // The counter was not zero on entry.  This kernel leaves every
            // counter at zero, even after an abort, so the workspace was
            // changed from outside (another workspace size, overlapping
            // calls): report it.  The counter is left as it is, so every
            // later call reports it too until the caller zero-fills the
            // workspace; resetting it here could pair this call's
            // publications with another call's tickets unnoticed.
            if (e == 0) atomicOr(p.status, DSA_DEV_STALE_WORKSPACE);
          } else if (tk < parts - 1 || i != n - 1) {
            // Publish this part: O^T in fp32 as this thread holds it, then
            // (m, l); a fence orders them before the publication count.
            const int64_t rec = own < kMaxParts ? mparts->rec[slot][own] : part_record(t, blockIdx.x, total, gridDim.x);
            float4* po = reinterpret_cast<float4*>(p.part_o + rec * kPartFloats);
#pragma unroll
            for (int mb = 0; mb < 4; ++mb) {
              float o[16];
              tmem_ld16(obuf + 16 * mb, o);
              tmem_wait_ld();
#pragma unroll
              for (int q = 0; q < 4; ++q)
                po[part_index(mb, q, col)] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
            }
            if (e < kHeads) {
              p.part_ml[rec * 2 * kHeads + 2 * e] = ml_smem[2 * e];
              p.part_ml[rec * 2 * kHeads + 2 * e + 1] = ml_smem[2 * e + 1];
            }
            if (i == n - 1) {  // nothing follows: publish now
              __threadfence();
              named_barrier_sync(1, 128);
              if (e == 0) atomicAdd(p.tok_pub + t, 1);
            } else {
              pub_t = t;
            }
            // The last arriver at its first segment (its O buffer is reused
            // later) merges from records once its work is done.
            if (e == 0 && tk == parts - 1) {
              merge_list[1 + 2 * merge_list[0]] = t;
              merge_list[2 + 2 * merge_list[0]] = -1;
              ++merge_list[0];
            }
          } else if (e == 0) {
            // The last arriver at its last segment: its part stays in TMEM
            // and the merge runs once every role is done, with all threads.
            merge_list[1 + 2 * merge_list[0]] = t;
            merge_list[2 + 2 * merge_list[0]] = static_cast<int>(kColO + 64u * (sg & 1));
            ++merge_list[0];
          }
        }
        owed_t = -1;
        // Every TMEM read of the O buffer has completed, and ml_smem, sx and
        // the merge scratch are free for the next segment.
        tc_fence_before();
        named_barrier_sync(1, 128);
        if (e == 0) mbar_arrive(&o_empty[sg & 1]);
      }
    }
    if (pub_t >= 0) {
      // The loop stopped before the deferred publication: publish now.
      __threadfence();
      named_barrier_sync(1, 128);
      if (e == 0) atomicAdd(p.tok_pub + pub_t, 1);
    }
    if (i < n && e == 0) {
      // The CTA aborted at tile i.  Its output is void (the status word says
      // so), but the merge counters must still end at zero for later calls:
      // settle every split token it had not finished, from tile i's on, as
      // if its part had been published -- take the ticket (unless taken
      // already), then publish, or, holding the last ticket, wait for the
      // others and zero the counters.
      const int t_end = static_cast<int>((u0 + n - 1) / kTilesPerTok);
      for (int tt = static_cast<int>((u0 + i) / kTilesPerTok); tt <= t_end; ++tt) {
        const int64_t a = static_cast<int64_t>(tt) * kTilesPerTok;
        if (a >= u0 && a + kTilesPerTok <= u0 + n) continue;  // whole in this CTA: no counters
        const int parts = parts_of(tt, total, gridDim.x);
        const int tk = tt == owed_t ? owed_tk : atomicAdd(p.tok_arrive + tt, 1);
        if (tk < parts - 1) {
          atomicAdd(p.tok_pub + tt, 1);
        } else if (tk == parts - 1) {
          wait_counter_at_least(p.tok_pub + tt, parts - 1, p.status, 2 * p.wait_limit_ns);
          p.tok_arrive[tt] = 0;
          p.tok_pub[tt] = 0;
        } else {
          atomicOr(p.status, DSA_DEV_STALE_WORKSPACE);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProdWarp0 && lane == 0) {
    // A Q load still in flight (only after an abort) must land before exit.
    // Only the last load of each slot can be: loading segment s + 2 waits
    // until segment s was consumed.  Its phase parity is unambiguous because
    // nothing reloads the slot afterwards; an older segment's parity would
    // read as pending again once the slot has been refilled twice.
    for (int k = 0; k < 2; ++k)
      if (q_last[k] >= 0) mbar_drain(&q_full[k], (q_last[k] >> 1) & 1, p.status);
  }
  // Split tokens this CTA merges (at most its first and last segments).
  const int nmerge = merge_list[0];
  uint32_t land_parity = 0;
  for (int k = 0; k < nmerge && k < 2; ++k) {
    if (k > 0) __syncthreads();  // the merge scratch (P and Sx buffers, free now) and landing are reused
    const int t = merge_list[1 + 2 * k];
    if (merge_at_end(p, t, *mparts, t == t_first ? 0 : 1, merge_list[2 + 2 * k], ml_smem, tmem_base,
                     p_mem, stage_mem, land_bar, land_parity))
      land_parity ^= 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

inline int grid_for(int num_tokens, int num_sms) {
  const int64_t units = static_cast<int64_t>(num_tokens) * kTilesPerTok;
  return static_cast<int>(units < num_sms ? units : num_sms);
}

// Workspace: header, [records][16][2] (m, l), [records][kPartFloats] O^T,
// ..., [num_tokens] publication counters, [num_tokens] arrival counters at
// the very end.
inline size_t records_for(int num_tokens, int num_sms) {
  return static_cast<size_t>(grid_for(num_tokens, num_sms)) * kRecsPerCta;
}

inline size_t workspace_for(int num_tokens, int num_sms) {
  if (num_tokens <= 0) return kWorkspaceHeader;
  return kWorkspaceHeader + records_for(num_tokens, num_sms) * (2 * kHeads + kPartFloats) * sizeof(float) +
         2 * sizeof(int) * static_cast<size_t>(num_tokens);
}

std::once_flag g_attr_once[64];
int g_attr_status[64];

// One armed test fault (dsa_b200_test_inject), consumed by the next launch.
std::atomic<unsigned long long> g_inject{0};  // kind << 56 | wait limit (ns), 0 = none

}  // namespace attn
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_b200_test_inject(int kind, uint64_t wait_limit_ns) {
  if (kind == DSA_TEST_NONE) {
    attn::g_inject.store(0);
    arm_indexer_test_fault(0);
    return DSA_OK;
  }
  if ((kind != DSA_TEST_SKIP_ARRIVAL && kind != DSA_TEST_SKIP_READY) || wait_limit_ns == 0 ||
      wait_limit_ns >= (1ull << 56))
    return DSA_ERR_INVALID_ARGUMENT;
  const unsigned long long armed = (static_cast<unsigned long long>(kind) << 56) | wait_limit_ns;
  if (kind == DSA_TEST_SKIP_READY)
    arm_indexer_test_fault(armed);  // consumed by the next dsa_indexer_run
  else
    attn::g_inject.store(armed);    // consumed by the next dsa_attention_run
  return DSA_OK;
}

extern "C" size_t dsa_attention_workspace_bytes(int32_t num_tokens) {
  DeviceInfo info;
  // Without a usable device, size for the largest SM count of the family.
  const int sms = current_device_info(&info) == DSA_OK ? info.num_sms : 160;
  return attn::workspace_for(num_tokens, sms);
}

extern "C" int dsa_attention_run(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                 const void* kpe_cache, int64_t num_slots,
                                 const int32_t* sparse_indices, int32_t num_tokens,
                                 float sm_scale, void* output, float* lse, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (num_tokens < 0 || num_tokens > attn::kMaxTokens) return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;
  if (!q_nope || !q_pe || !ckv_cache || !kpe_cache || !sparse_indices || !output || !lse ||
      !workspace)
    return DSA_ERR_INVALID_ARGUMENT;
  if (num_slots < 1 || num_slots > 0x7FFFFFFF) return DSA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_nope) || !aligned16(q_pe) || !aligned16(ckv_cache) || !aligned16(kpe_cache) ||
      !aligned16(output) || !aligned16(workspace))
    return DSA_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(sparse_indices) | reinterpret_cast<uintptr_t>(lse)) & 3u)
    return DSA_ERR_MISALIGNED;

  DeviceInfo info;
  int st = current_device_info(&info);
  if (st != DSA_OK) return st;
  if (static_cast<size_t>(attn::kSmemBytes) > info.max_smem_optin) return DSA_ERR_UNSUPPORTED_DEVICE;
  if (workspace_bytes < attn::workspace_for(num_tokens, info.num_sms))
    return DSA_ERR_WORKSPACE_TOO_SMALL;
  std::call_once(attn::g_attr_once[info.device], [&]() {
    attn::g_attr_status[info.device] =
        cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn::kSmemBytes) == cudaSuccess
            ? DSA_OK
            : DSA_ERR_CUDA;
  });
  if (attn::g_attr_status[info.device] != DSA_OK) return attn::g_attr_status[info.device];

  CUtensorMap ckv_map, kpe_map, qn_map, qp_map;
  const uint64_t rows_q = static_cast<uint64_t>(num_tokens) * attn::kHeads;
  if ((st = encode_tmap_2d(&ckv_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ckv_cache, attn::kCkv,
                           static_cast<uint64_t>(num_slots), attn::kCkv * 2, 64, 1)) != DSA_OK)
    return st;
  if ((st = encode_tmap_2d(&kpe_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kpe_cache, attn::kKpe,
                           static_cast<uint64_t>(num_slots), attn::kKpe * 2, 64, 1)) != DSA_OK)
    return st;
  if ((st = encode_tmap_2d(&qn_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q_nope, attn::kCkv, rows_q,
                           attn::kCkv * 2, 64, attn::kHeads)) != DSA_OK)
    return st;
  if ((st = encode_tmap_2d(&qp_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q_pe, attn::kKpe, rows_q,
                           attn::kKpe * 2, 64, attn::kHeads)) != DSA_OK)
    return st;

  const int grid = attn::grid_for(num_tokens, info.num_sms);
  const size_t recs = attn::records_for(num_tokens, info.num_sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  attn::Params prm;
  prm.indices = sparse_indices;
  prm.ckv = static_cast<const uint8_t*>(ckv_cache);
  prm.kpe = static_cast<const uint8_t*>(kpe_cache);
  prm.out = static_cast<__nv_bfloat16*>(output);
  prm.lse = lse;
  prm.part_ml = reinterpret_cast<float*>(ws + kWorkspaceHeader);
  prm.part_o = prm.part_ml + recs * attn::kHeads * 2;
  // The counters sit at the end of the buffer: every call leaves them at
  // zero, and no call with another token count puts partial records there
  // (records grow from the front, and workspace_for(T) >= records(T) +
  // counters(T) with records(T) non-decreasing in T), so they need no
  // clearing as long as every call passes the same workspace_bytes.
  const size_t cnt_off = (workspace_bytes - 2 * sizeof(int) * static_cast<size_t>(num_tokens)) & ~static_cast<size_t>(3);
  prm.tok_pub = reinterpret_cast<int*>(ws + cnt_off);
  prm.tok_arrive = prm.tok_pub + num_tokens;
  prm.status = reinterpret_cast<unsigned int*>(ws);
  prm.num_slots = num_slots;
  prm.num_tokens = num_tokens;
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  prm.wait_limit_ns = kWaitLimitNs;
  prm.inject = attn::kInjectNone;
  if (attn::g_inject.load(std::memory_order_relaxed) != 0) {
    const unsigned long long armed = attn::g_inject.exchange(0);
    if (armed != 0) {
      prm.inject = static_cast<int>(armed >> 56);
      prm.wait_limit_ns = armed & ((1ull << 56) - 1);
    }
  }

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (launch_programmatic(attn::attention_kernel, dim3(grid), dim3(attn::kThreads), attn::kSmemBytes,
                          s, ckv_map, kpe_map, qn_map, qp_map, prm) != cudaSuccess)
    return DSA_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}
