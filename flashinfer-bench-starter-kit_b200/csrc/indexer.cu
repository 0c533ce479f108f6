// indexer.cu -- DSA lightning indexer (decode) for sm_100a.
//
// Replaces dsa_topk_run_ms / run() of dsa_indexer/solution/triton/kernel.py.
// Two kernels, both launched on the caller's stream with no host sync:
//
// 1. indexer_score_kernel (persistent, one CTA per SM).  The work list is the
//    concatenation over requests of 128-token tiles (two 64-token pages);
//    CTA c takes the contiguous slice [c*U/G, (c+1)*U/G) of the U tiles, so
//    load balance does not depend on how seq_lens are distributed.  Roles:
//      warps 8,9   TMA producers, each owning every 2nd tile: raw FP8 pages
//                  (64 rows x 128 B, 128-byte swizzle) into an 8-deep
//                  shared-memory ring and each page's 64 fp32 scales (bulk
//                  copy) into a 12-slot scale ring that outlives the K stage
//                  until the epilogue has used it.  Block-table entries are
//                  resolved 32 tiles at a time, one group ahead, so no load
//                  latency sits between two copy issues.  Nothing is dequantised in HBM
//                  (the reference writes an fp32 copy of K, kernel.py:108-135).
//      warps 10-13 MMA issuers (warp 10+r takes the tiles n with n % 4 == r;
//                  warp 10 also loads q[b], 64 heads x 128 B, when the
//                  request changes): tcgen05.mma kind::f8f6f4,
//                  M = 128 tokens, N = 64 heads, K = 128 (4 x K32), fp32
//                  accumulator in TMEM, 4 accumulator stages; the K stage is
//                  freed as soon as the MMAs complete.
//      warps 0-7   epilogue, two sets of four (even / odd tiles): each
//                  thread owns one token row of the TMEM accumulator (64
//                  head columns) and computes sum_h w_h * relu(scale_tok *
//                  acc_h) in registers -- no cross-thread reduction -- then
//                  stores one fp32 score.
//    Scores go to a [batch, max_pages*64] fp32 workspace (L2-resident at
//    decode sizes); per-head scores never exist in memory (the reference
//    materialises [64, L] fp32, kernel.py:293-300).
//
// 2. topk_select_kernel (one CTA per request).  Exact top-min(L, 2048) by
//    radix select on the 64-bit key (order(score) << 32 | ~token), which
//    encodes "score descending, then lower token index first" as one total
//    order.  The score kernel's epilogue already histograms the top 11 key
//    bits per request (per-warp shared-memory histograms, summed by the
//    CTA's eight epilogue warps together and added into a global
//    [batch, 2048] table, cleared at each call by a small kernel that the
//    score kernel overlaps through programmatic launch);
//    one pass over the L scores then moves the winners of higher bins to the
//    output and the boundary bin to a shared-memory candidate list, which
//    later passes refine.  The 2048 winners are bucket-sorted on an 11-bit
//    digit of their score (an in-warp bitonic + merge-path sort when the
//    keys crowd into few buckets) and translated to global slot ids through
//    the block table (kernel.py:156-169), then -1 padded (kernel.py:206).
#include <algorithm>
#include <atomic>
#include <mutex>

#include "host.h"
#include "ptx.cuh"

namespace dsa {
namespace ix {

constexpr int kPage = DSA_PAGE_SIZE;                      // 64 tokens per page
constexpr int kHeads = DSA_INDEX_HEADS;                   // 64
constexpr int kDim = DSA_INDEX_DIM;                       // 128 fp8 per token
constexpr int kPageBytes = DSA_INDEX_PAGE_BYTES;          // 8448
constexpr int kPageRows = kPageBytes / 128;               // page = 66 rows of 128 B
constexpr int kPageDataBytes = kPage * kDim;              // 8192
constexpr int kScaleBytes = kPage * 4;                    // 256
constexpr int kTileTok = 2 * kPage;                       // 128 tokens per tile
constexpr int kStageData = 2 * kPageDataBytes;            // 16384: two pages of FP8 rows
constexpr int kStageStride = kStageData;                  // 1 KiB aligned (128-byte swizzle atoms)
constexpr int kStages = 8;
constexpr int kAccStages = 4;
constexpr int kTmemCols = kAccStages * kHeads;            // 256
// Token-scale ring: tile n's 2 x 64 fp32 scales go to slot n % kScaleSlots.
// The producer of tile n waited for the MMAs of tile n - kStages, which
// waited for the epilogue of tile n - kStages - kAccStages to release its
// accumulator (after reading its scales), so that slot is free again.
constexpr int kScaleSlots = kStages + kAccStages;
constexpr int kEpiWarps = 8;                              // warps 0-7: epilogue, two sets of 4
constexpr int kProdWarp0 = kEpiWarps;                     // warps 8-9: producers
constexpr int kProdWarps = 2;
constexpr int kMmaWarp0 = kProdWarp0 + kProdWarps;        // warps 10-13: MMA issuers
constexpr int kMmaWarps = 4;
constexpr int kThreads = 32 * (kMmaWarp0 + kMmaWarps);    // 14 warps
constexpr int kBins = 2048;                               // radix bins: top 11 key bits
// Each epilogue warp keeps its own histogram of 16-bit counters, two per
// word; the eight are flushed together at least every kFlushSpan slice
// positions, i.e. every kFlushSpan / 2 tiles of a warp: 32 lanes x 128 tiles
// < 65536, so a counter never carries into its neighbour.  (The span also
// makes the periodic flush happen in slices of ordinary size.)
constexpr int kFlushSpan = 256;
static_assert(32 * (kFlushSpan / 2) < 65536, "16-bit histogram counters");
constexpr int kMaxBatch = 4096;
// Per-request ready counters at the front of the workspace, at fixed offsets
// for every request index a call can have, so that a later call (of any
// batch) never takes histogram or score bytes for counters.  They are never
// reset: the score kernel adds each request's (tile, epilogue warp) pairs to
// [2 b] as they are scored, and the select, which waits until [2 b] - [2 b + 1]
// reaches the request's count, advances [2 b + 1] by that count.  A zero-filled
// workspace starts them consistent.
constexpr size_t kReadyBytes = sizeof(unsigned int) * 2 * kMaxBatch;
constexpr int kMaxPagesPerSeq = 1 << 20;
constexpr int64_t kMaxPool = (int64_t(1) << 31) / kPageRows - 1;

// e4m3 x e4m3 -> f32, A (tokens) and B (heads) K-major, M = 128, N = 64.
constexpr uint32_t kIdesc = idesc_make(0, 0, false, false, 128, 64);

constexpr int kOffStage = 0;
constexpr int kOffQ = kOffStage + kStages * kStageStride;         // 131072
constexpr int kOffHist = kOffQ + 2 * kPageDataBytes;              // 147456
constexpr int kOffScale = kOffHist + kEpiWarps * kBins * 2;       // 180224: scale ring
constexpr int kOffBar = kOffScale + kScaleSlots * 2 * kScaleBytes; // 186368
constexpr int kNumBars = 2 * kStages + 4 + 2 * kAccStages + kMmaWarps;
constexpr int kOffMisc = kOffBar + 256;
constexpr int kOffInfo = kOffMisc + 128;                          // producer warps x 32 tiles
// Weights and lengths of the first kWtReqs requests of a CTA's slice, staged
// by the epilogue warps at the start: a request change then reads them from
// shared memory instead of waiting on global loads with the pipeline behind it.
constexpr int kWtReqs = 16;
constexpr int kOffWts = kOffInfo + kProdWarps * 32 * 5 * 4;
constexpr int kOffLens = kOffWts + kWtReqs * kHeads * 4;
constexpr int kOffTiles = kOffLens + kWtReqs * 4;
static_assert(kNumBars * 8 <= 256, "barrier area");
static_assert(kStages % kProdWarps == 0 && kScaleSlots % kProdWarps == 0, "producer stride");
static_assert(16 + 4 * (kThreads / 32) <= 128, "misc area");
static_assert(kAccStages % 2 == 0, "epilogue sets take alternate accumulator stages");
static_assert((kMmaWarps & (kMmaWarps - 1)) == 0, "MMA issuers split tiles by n % kMmaWarps");

inline size_t score_smem_bytes(int batch) {
  return 1024 + kOffTiles + sizeof(int) * static_cast<size_t>(batch + 1);
}

struct ScoreParams {
  const uint8_t* k_cache;
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* scores;          // [batch][score_stride]
  unsigned int* hist;     // [batch][kBins], cleared by hist_clear_kernel at every call
  unsigned int* status;
  // [kMaxBatch][2]: per request, the count of scored (tile, epilogue warp)
  // pairs and the count the select has consumed; never reset (see
  // kReadyBytes).
  unsigned int* ready;
  int64_t num_pages;
  int batch;
  int skip_ready_req;     // test hook: a request whose ready count is never published; -1 none
  int max_pages;
  int score_stride;       // = max_pages * 64
};

__device__ __forceinline__ int clamp_len(int L, int max_len, unsigned int* status) {
  if (L < 0 || L > max_len) {
    atomicOr(status, DSA_DEV_BAD_SEQ_LEN);
    L = L < 0 ? 0 : max_len;
  }
  return L;
}


// Locates tile u of the work list: request b = the one with
// tile_off[b] <= u < tile_off[b+1], tile j = u - tile_off[b].
__device__ __forceinline__ void locate(const int* tile_off, int batch, int64_t u, int& b, int& j) {
  int lo = 0, hi = batch;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (tile_off[mid + 1] <= u) lo = mid + 1; else hi = mid;
  }
  b = lo;
  j = static_cast<int>(u - tile_off[b]);
}

// What the producer needs to know about one tile; each lane of the producer
// warp resolves one tile of a 32-tile group so the block-table loads of a
// whole group are in flight together (and one group ahead).
struct TileInfo {
  int b, j, npg, p0, p1;
};

// Tile u's request, tile index and page ids in two steps: tile_info issues
// the loads (the request's length and both block-table entries, independent
// of each other, so one round trip) and uses none of their values;
// finish_tile_info, called once the values are needed (a group of tiles
// later in the producer), checks them and settles the page count.  The
// producer thus never waits for the next group's loads before issuing the
// current group's copies.
__device__ __forceinline__ TileInfo tile_info(const ScoreParams& p, const int* tile_off,
                                              int64_t u, int64_t u1) {
  TileInfo t{-1, 0, 0, 0, 0};
  if (u < u1) {
    locate(tile_off, p.batch, u, t.b, t.j);
    const int32_t* row = p.block_table + static_cast<int64_t>(t.b) * p.max_pages;
    t.npg = __ldg(p.seq_lens + t.b);  // the raw length until finish_tile_info
    t.p0 = __ldg(row + 2 * t.j);
    t.p1 = 2 * t.j + 1 < p.max_pages ? __ldg(row + 2 * t.j + 1) : 0;
  }
  return t;
}
__device__ __forceinline__ TileInfo finish_tile_info(const ScoreParams& p, TileInfo t, int max_len) {
  if (t.b >= 0) {
    const int L = clamp_len(t.npg, max_len, p.status);
    const int req_pages = (L + kPage - 1) / kPage;
    t.npg = (2 * t.j + 1 < req_pages) ? 2 : 1;
    if (t.p0 < 0 || t.p0 >= p.num_pages) {
      atomicOr(p.status, DSA_DEV_BAD_PAGE);
      t.p0 = 0;
    }
    if (t.npg == 1) {
      t.p1 = 0;  // past the request's last page: the entry is not used or checked
    } else if (t.p1 < 0 || t.p1 >= p.num_pages) {
      atomicOr(p.status, DSA_DEV_BAD_PAGE);
      t.p1 = 0;
    }
  }
  return t;
}

// Zeroes n 16-byte words of the histogram rows.  The score kernel is
// launched programmatically after it and only its epilogue warps wait for it
// (griddep_wait), so the clearing overlaps the score kernel's start; the
// lines it writes are in L2 when the epilogue's atomics reach them.
__global__ void __launch_bounds__(256) hist_clear_kernel(uint4* p, int64_t n) {
  griddep_launch_dependents();
  for (int64_t i = blockIdx.x * 256 + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * 256)
    p[i] = make_uint4(0u, 0u, 0u, 0u);
}

__global__ void __launch_bounds__(kThreads, 1)
indexer_score_kernel(const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap qmap, const ScoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  // Pointer arithmetic on the shared array (not an integer round trip) keeps
  // the shared address space visible to the compiler: plain LDS/STS/ATOMS.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_mem = smem + kOffStage;
  uint8_t* q_mem = smem + kOffQ;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + kOffHist);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* qfull = bars + 2 * kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* accfull = qempty + 2;
  uint64_t* accempty = accfull + kAccStages;
  uint64_t* drain = accempty + kAccStages;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + kOffMisc + 4);
  int* warp_sums = reinterpret_cast<int*>(smem + kOffMisc + 16);  // one int per warp
  int* tile_off = reinterpret_cast<int*>(smem + kOffTiles);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int max_len = p.max_pages * kPage;
  // The select kernel may start launching now: it reads a row's scores and
  // histogram only once its request's ready count (released after the
  // stores and atomics it covers) shows every tile of the request scored.
  griddep_launch_dependents();

  if (tid == 0) {
    // full: the owning producer warp's arrive.expect_tx.  accempty: the four
    // epilogue warps of the set that owns the stage.  empty: the MMA
    // commit.  qempty: one commit from each MMA issuer.  accfull: the MMA
    // commit plus the issuer's arrive, which publishes the scale-ring entry.
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(&qfull[s], 1); mbar_init(&qempty[s], kMmaWarps); }
    for (int s = 0; s < kAccStages; ++s) { mbar_init(&accfull[s], 2); mbar_init(&accempty[s], 4); }
    for (int w = 0; w < kMmaWarps; ++w) mbar_init(&drain[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProdWarp0 && lane == 0) { prefetch_tensor_map(&kmap); prefetch_tensor_map(&qmap); }
  if (warp == kMmaWarp0) tmem_alloc(tmem_base_smem, kTmemCols);
  if (warp < kEpiWarps) {  // zero the shared-memory histograms
    for (int i = tid; i < kEpiWarps * kBins / 2; i += 32 * kEpiWarps) hist_all[i] = 0;
  }

  // Tile prefix sums over requests (each CTA recomputes them: seq_lens stay
  // on the device and B is small).
  {
    const int chunk = (p.batch + kThreads - 1) / kThreads;
    const int lo = min(p.batch, tid * chunk), hi = min(p.batch, lo + chunk);
    int local = 0;
    for (int b = lo; b < hi; ++b) {
      int L = clamp_len(__ldg(p.seq_lens + b), max_len, p.status);
      local += (L + kTileTok - 1) / kTileTok;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_sums[w];
    int run = base + incl - local;
    for (int b = lo; b < hi; ++b) {
      tile_off[b] = run;
      int L = clamp_len(__ldg(p.seq_lens + b), max_len, p.status);
      run += (L + kTileTok - 1) / kTileTok;
    }
    if (tid == kThreads - 1) tile_off[p.batch] = base + incl;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = *tmem_base_smem;
  const int64_t total = tile_off[p.batch];
  const int u0 = static_cast<int>(total * blockIdx.x / gridDim.x);
  const int u1 = static_cast<int>(total * (blockIdx.x + 1) / gridDim.x);
  const int nt = u1 - u0;  // tiles of this CTA
  const WaitCtx wctx{abort_flag, p.status, kWaitLimitNs};

  if (warp >= kProdWarp0 && warp < kProdWarp0 + kProdWarps) {
    // ------------------------------------------------------ producer warps
    // Warp 8+k owns tiles n = k, k+2, k+4, ... of this CTA's slice and issues
    // both of their FP8 page boxes and both 256-byte scale copies.  One thread
    // issues copies at a fixed rate, so two producer warps keep the ring
    // full.  Each warp resolves the block-table entries of its next 32 tiles
    // at once, one group ahead, and stages them in shared memory.
    const int k = warp - kProdWarp0;
    TileInfo* info = reinterpret_cast<TileInfo*>(smem + kOffInfo) + 32 * k;
    const uint64_t policy = make_policy_evict_first();
    const int mine = nt > k ? (nt - k + kProdWarps - 1) / kProdWarps : 0;
    int m = 0;  // tiles issued by this warp
    int ok = 1;
    // Stage, its phase and the scale slot of this warp's next tile
    // n = k + kProdWarps * m, advanced incrementally.
    int s = k, sslot = k;
    uint32_t ph = 0;
    TileInfo nxt = tile_info(p, tile_off, u0 + k + kProdWarps * lane, u1);
    for (int g0 = 0; g0 < mine && ok; g0 += 32) {
      info[lane] = finish_tile_info(p, nxt, max_len);
      nxt = tile_info(p, tile_off, u0 + k + kProdWarps * (g0 + 32 + lane), u1);
      __syncwarp();
      const int cnt = mine - g0 < 32 ? mine - g0 : 32;
      if (lane == 0) {
        for (int t = 0; t < cnt; ++t, ++m) {
          const TileInfo ti = info[t];
          if (!mbar_wait(&empty[s], ph ^ 1, wctx)) { ok = 0; break; }
          uint8_t* st = stage_mem + s * kStageStride;
          uint8_t* sc = smem + kOffScale + sslot * 2 * kScaleBytes;
          mbar_arrive_expect_tx(&full[s], ti.npg * (kPageDataBytes + kScaleBytes));
          tma_load_2d_hint(st, &kmap, &full[s], 0, ti.p0 * kPageRows, policy);
          bulk_load(sc, p.k_cache + static_cast<int64_t>(ti.p0) * kPageBytes + kPageDataBytes,
                    kScaleBytes, &full[s]);
          if (ti.npg == 2) {
            tma_load_2d_hint(st + kPageDataBytes, &kmap, &full[s], 0, ti.p1 * kPageRows, policy);
            bulk_load(sc + kScaleBytes, p.k_cache + static_cast<int64_t>(ti.p1) * kPageBytes + kPageDataBytes,
                      kScaleBytes, &full[s]);
          }
          if ((s += kProdWarps) >= kStages) { s -= kStages; ph ^= 1; }
          if ((sslot += kProdWarps) >= kScaleSlots) sslot -= kScaleSlots;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      __syncwarp();
    }
    if (lane == 0) {  // let every copy this thread issued land before the CTA can exit
      for (int j = (m > 2 ? m - 2 : 0); j < m; ++j) {
        const int n = k + kProdWarps * j;
        mbar_drain(&full[n % kStages], static_cast<uint32_t>((n / kStages) & 1), p.status);
      }
    }
  } else if (warp >= kMmaWarp0) {
    // ------------------------------------------------------ MMA issuers
    // Warp 10+r takes the tiles n with n % 4 == r.  A thread can hand
    // tcgen05 and bulk-copy instructions to the asynchronous units only at a
    // fixed rate (about 135-180 cycles per instruction, paid by its next
    // shared-memory access), so a tile's 4 MMAs + 2 commits from one thread
    // take longer than the tile's HBM time; four issuing warps share the
    // load.  The whole loop runs in lane 0; the other lanes wait at the final
    // __syncwarp.
    const int parity = warp - kMmaWarp0;
    if (lane == 0 && nt > 0) {
      int b = 0, j = 0;
      locate(tile_off, p.batch, u0, b, j);
      int ntb = tile_off[b + 1] - tile_off[b];  // tiles of request b
      int nq = 0, slot = 0;
      int s = 0, a = 0;          // stage and accumulator of tile n
      uint32_t ph = 0, aph = 0;  // and their phase parities
      bool ok = true, new_req = true;
      for (int n = 0; n < nt && ok; ++n) {
        if (new_req) {
          new_req = false;
          if (nq > 0) umma_commit(&qempty[(nq - 1) & 1]);
          if (parity == 0) {  // warp 10 loads q[b] once all issuers released the slot
            ok = mbar_wait(&qempty[nq & 1], ((nq >> 1) & 1) ^ 1, wctx);
            if (ok) {
              mbar_arrive_expect_tx(&qfull[nq & 1], kPageDataBytes);
              tma_load_2d(q_mem + (nq & 1) * kPageDataBytes, &qmap, &qfull[nq & 1], 0, b * kHeads);
            }
          }
          ok = ok && mbar_wait(&qfull[nq & 1], (nq >> 1) & 1, wctx);
          slot = nq & 1;
          ++nq;
          if (!ok) break;
        }
        if ((n & (kMmaWarps - 1)) == parity) {
          ok = mbar_wait(&full[s], ph, wctx) && mbar_wait(&accempty[a], aph ^ 1, wctx);
          if (!ok) break;
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(stage_mem + s * kStageStride), 16, 1024);
          const uint64_t bd = sdesc_sw128(smem_u32(q_mem + slot * kPageDataBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < kDim / 32; ++k)  // +32 bytes along K per step (start address >> 4)
            umma_f8(tmem_base + a * kHeads, ad + 2 * k, bd + 2 * k, kIdesc, k > 0 ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&accfull[a]);
          // Release after this thread's acquire of full[s]: makes the
          // tile's bulk-copied token scales visible to the epilogue.
          mbar_arrive(&accfull[a]);
        }
        if (++s == kStages) { s = 0; ph ^= 1; }
        if (++a == kAccStages) { a = 0; aph ^= 1; }
        if (++j == ntb) {
          j = 0;
          do { ++b; } while (b < p.batch && tile_off[b + 1] == tile_off[b]);
          if (b < p.batch) ntb = tile_off[b + 1] - tile_off[b];
          new_req = true;
        }
      }
      umma_commit(&drain[parity]);
      mbar_drain(&drain[parity], 0, p.status);
      if (parity == 0)  // a q load still in flight must land before exit
        for (int j = (nq > 2 ? nq - 2 : 0); j < nq; ++j) mbar_drain(&qfull[j & 1], (j >> 1) & 1, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ epilogue warps
    // Two sets of four warps take the even and the odd tiles (so the even and
    // odd accumulator stages), which gives every scheduler two epilogue warps
    // to interleave.  Warp w reads TMEM sub-partition w & 3, token rows
    // 32*(w&3) .. +31, and steps straight from one of its tiles to the next.
    const int set = warp >> 2;
    const int sp = warp & 3;          // TMEM sub-partition this warp may access
    const int row = sp * 32 + lane;   // token row of the 128-token tile
    uint32_t* hist = hist_all + warp * (kBins / 2);
    // The score kernel is launched programmatically after the kernel that
    // clears the global histograms; only these warps touch them.
    griddep_wait();
    float* w_smem = reinterpret_cast<float*>(smem + kOffWts);
    int b_first = 0;
    if (nt > 0) {
      int j0 = 0;
      locate(tile_off, p.batch, u0, b_first, j0);
      const int nr = min(kWtReqs, p.batch - b_first);
      for (int i = tid; i < nr * kHeads; i += 32 * kEpiWarps) w_smem[i] = __ldg(p.weights + b_first * kHeads + i);
      if (tid < nr) reinterpret_cast<int*>(smem + kOffLens)[tid] = __ldg(p.seq_lens + b_first + tid);
    }
    named_barrier_sync(1, 32 * kEpiWarps);
    // Histogram flushes are done by the eight epilogue warps together: at a
    // flush event they meet at a named barrier, each thread sums four words
    // of the eight warps' shared-memory histograms (32-bit sums of the packed
    // 16-bit counts) and adds the non-zero ones to the global histogram --
    // at most 2048 global atomics per event instead of one per non-zero word
    // of every warp (flushing separately measured 2.5 us per warp).  Events
    // are positions of the slice: every request end inside it, every
    // kFlushSpan positions (a warp scores at most kFlushSpan / 2 tiles
    // between two flushes, so no 16-bit count overflows) and the slice end.  A warp
    // flushes every event at or before its next tile's position before it
    // scores that tile, and all remaining ones at the end, so all eight warps
    // meet the same events in the same order, whatever tiles they hold or if
    // they stopped early.
    //
    // A request's ready count (4 per tile scored in this slice) is added by
    // one thread after every epilogue thread has fenced its score stores and
    // histogram atomics (release).  A request finished in mid-slice waits
    // for the next such fence (the next request end or the slice end): a
    // fence at every end stalls the epilogue for the acknowledgement of
    // every store in flight, and the slice's first request is finished by the
    // previous CTA at the end of its slice anyway.  Nothing is added after an
    // abort, so the select reports a timeout instead of reading a partial row.
    if (nt > 0) {
      int fpos = 0, fr = b_first, pend = -1;  // flushed up to position fpos; its request
      auto cta_flush = [&](int r) {
        named_barrier_sync(2, 32 * kEpiWarps);
        unsigned int* g = p.hist + static_cast<int64_t>(r) * kBins;
        for (int i = tid; i < kBins / 2; i += 32 * kEpiWarps) {
          uint32_t lo = 0, hi = 0;
#pragma unroll
          for (int w = 0; w < kEpiWarps; ++w) {
            const uint32_t x = hist_all[w * (kBins / 2) + i];
            lo += x & 0xFFFFu;
            hi += x >> 16;
            hist_all[w * (kBins / 2) + i] = 0;
          }
          if (lo) atomicAdd(g + 2 * i, lo);
          if (hi) atomicAdd(g + 2 * i + 1, hi);
        }
        named_barrier_sync(2, 32 * kEpiWarps);
      };
      auto publish = [&](int r) {  // after a fence by every epilogue thread and a barrier
        if (tid == 0 && r != p.skip_ready_req && !*static_cast<volatile int*>(abort_flag)) {
          const int cnt = min(tile_off[r + 1], u1) - max(tile_off[r], u0);
          if (cnt > 0) atomicAdd(p.ready + 2 * r, 4u * static_cast<unsigned int>(cnt));
        }
      };
      // Flushes every event at or before position P (the slice end included
      // when P == nt).
      auto flush_events = [&](int P) {
        while (fpos < nt) {
          const int er = tile_off[fr + 1] - u0;  // end of request fr in the slice
          int e = min(er, nt);
          e = min(e, (fpos / kFlushSpan + 1) * kFlushSpan);
          if (e > P) break;
          cta_flush(fr);
          fpos = e;
          if (e == nt) {
            __threadfence();
            named_barrier_sync(2, 32 * kEpiWarps);
            if (pend >= 0) publish(pend);
            publish(fr);
          } else if (e == er) {
            if (pend >= 0) {
              __threadfence();
              named_barrier_sync(2, 32 * kEpiWarps);
              publish(pend);
            }
            pend = fr;
            // The next request with tiles (position e < nt lies in one).
            do { ++fr; } while (tile_off[fr + 1] == tile_off[fr]);
          }
        }
      };
      if (set < nt) {
        int b = 0, j = 0;
        locate(tile_off, p.batch, u0 + set, b, j);
        int ntb = tile_off[b + 1] - tile_off[b];
        int L = 0;
        float* srow = nullptr;
        float wt[kHeads];
        auto enter = [&]() {  // request b becomes current
          const bool staged = b - b_first < kWtReqs;
          L = clamp_len(staged ? reinterpret_cast<const int*>(smem + kOffLens)[b - b_first] : __ldg(p.seq_lens + b),
                        max_len, p.status);
          srow = p.scores + static_cast<int64_t>(b) * p.score_stride;
          if (staged) {
            const float4* w4 = reinterpret_cast<const float4*>(w_smem + (b - b_first) * kHeads);
#pragma unroll
            for (int h = 0; h < kHeads / 4; ++h) {
              const float4 x = w4[h];
              wt[4 * h] = x.x; wt[4 * h + 1] = x.y; wt[4 * h + 2] = x.z; wt[4 * h + 3] = x.w;
            }
          } else {
#pragma unroll
            for (int h = 0; h < kHeads; ++h) wt[h] = __ldg(p.weights + b * kHeads + h);
          }
        };
        enter();
        int a = set, slot = set;  // accumulator, scale slot of tile n
        uint32_t aph = 0;
        for (int n = set; n < nt; n += 2) {
          flush_events(n);
          const int tok = j * kTileTok + row;
          if (!__all_sync(0xffffffffu, mbar_wait(&accfull[a], aph, wctx))) break;
          tc_fence_after();
          const float scale = *reinterpret_cast<const float*>(smem + kOffScale + slot * 2 * kScaleBytes + row * 4);
          // relu(scale * v) = scale * relu(v) for scale > 0: one max
          // (NaN-propagating, like the reference's v <= 0 ? 0 : v) and one fma
          // per head; other scales (zero, negative, NaN) take relu(scale * v)
          // term by term as the reference writes it.  Two 32-column halves keep
          // the register footprint small enough for 14 warps.
          const bool pos = scale > 0.f;
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + a * kHeads;
          float f0 = 0.f, f1 = 0.f, g0 = 0.f;
          float v[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tmem_ld32_wait(taddr + 32 * half, v);
            if (half == 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&accempty[a]);
            }
            if (pos) {
#pragma unroll
              for (int h = 0; h < 32; h += 2) {
                f0 = fmaf(relu_nan(v[h]), wt[32 * half + h], f0);
                f1 = fmaf(relu_nan(v[h + 1]), wt[32 * half + h + 1], f1);
              }
            } else {
#pragma unroll
              for (int h = 0; h < 32; ++h) {
                const float x = v[h] * scale;
                g0 += (x <= 0.f ? 0.f : x) * wt[32 * half + h];
              }
            }
          }
          if (tok < L) {
            const float sc = pos ? scale * (f0 + f1) : g0;
            srow[tok] = sc;
            const uint32_t bin = score_key(sc) >> 21;
            atomicAdd(&hist[bin >> 1], 1u << ((bin & 1u) << 4));
          }
          // Step to tile n + 2.
          if ((a += 2) >= kAccStages) { a -= kAccStages; aph ^= 1; }
          if ((slot += 2) >= kScaleSlots) slot -= kScaleSlots;
          if (n + 2 < nt && (j += 2) >= ntb) {
            do { j -= ntb; ++b; ntb = tile_off[b + 1] - tile_off[b]; } while (j >= ntb);
            enter();
          }
        }
      }
      flush_events(nt);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------ top-k select
// The select runs with T = 1024 threads per CTA (one CTA per SM: a batch
// that fits the SMs in one wave is latency-bound) or T = 512 (two CTAs per
// SM, for batches of more rows than SMs, where the select is throughput-bound).
constexpr int kTopK = DSA_TOPK;
constexpr int kStageCap = 512;                        // staged keys per warp
constexpr int kMergeOut = 4;                          // merge sort: outputs per thread per level
template <int T>
constexpr size_t sel_smem() {
  return sizeof(uint64_t) * (kTopK + (T / 32) * kStageCap) + sizeof(uint32_t) * 2 * kBins +
         sizeof(int) * (32 + 8 + T / 32);
}

struct SelectParams {
  const float* scores;
  const int32_t* row_req;  // block-table row of each score row; nullptr: the row itself
  unsigned int* status;
  const unsigned int* hist;
  const int32_t* seq_lens;
  const int32_t* block_table;
  int32_t* out;
  // The score kernel's per-request ready counts ([2 b] scored, [2 b + 1]
  // consumed), or nullptr: wait for the whole score grid instead.
  unsigned int* ready;
  unsigned long long wait_limit_ns;  // of the ready wait: kWaitLimitNs unless a test shortened it
  int score_stride;
  int max_pages;
};

__device__ __forceinline__ uint64_t composite(float s, int tok) {
  return (static_cast<uint64_t>(score_key(s)) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(tok));
}

// Inclusive prefix sum over the T threads of the block; total receives the
// block's sum.  One barrier: every warp scans the T / 32 warp totals itself.
// warp_tot (32 ints) must not be written again until every thread has passed
// a later barrier (each caller below has one before its next scan).
template <int T>
__device__ __forceinline__ int block_scan_incl(int v, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  const int wt = lane < T / 32 ? warp_tot[lane] : 0;
  int ti = wt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int u = __shfl_up_sync(0xffffffffu, ti, o);
    if (lane >= o) ti += u;
  }
  total = __shfl_sync(0xffffffffu, ti, 31);
  return v + __shfl_sync(0xffffffffu, ti - wt, warp);
}

// Finds the bin d (scanning from the highest bin down) that holds the
// need-th largest element; res = {d, count strictly above d, hist[d]}.
// Thread t holds the kBins / T bins kBins - 1 - (kBins / T) t - k, k = 0, 1, ...
template <int T>
__device__ __forceinline__ void find_bin(const uint32_t* hist, int need, int* warp_tot, int* res) {
  constexpr int kPer = kBins / T;
  const int t = threadIdx.x;
  // Defined even if the histogram holds fewer than `need` keys (it cannot
  // when it matches the scores; the output stage checks every token).
  if (t == 0) { res[0] = 0; res[1] = 0; res[2] = 0; }
  const int top = kBins - 1 - kPer * t;
  int c[kPer];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    c[k] = static_cast<int>(hist[top - k]);
    sum += c[k];
  }
  int total;
  int excl = block_scan_incl<T>(sum, warp_tot, total) - sum;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    if (excl < need && need <= excl + c[k]) { res[0] = top - k; res[1] = excl; res[2] = c[k]; }
    excl += c[k];
  }
  __syncthreads();
}

// Appends v to buf when pred holds; one shared atomic per warp.  Used only on
// the fallback path, where a degenerate score distribution overflows the
// per-warp staging areas.
__device__ __forceinline__ void warp_append(bool pred, uint64_t v, uint64_t* buf, int* counter,
                                            int cap) {
  const unsigned m = __ballot_sync(0xffffffffu, pred);
  if (m == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(counter, __popc(m));
  base = __shfl_sync(0xffffffffu, base, leader);
  const int pos = base + __popc(m & ((1u << lane) - 1u));
  if (pred && pos < cap) buf[pos] = v;
}

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), m);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// Descending sort of the 2048 keys in buf (tmp: 2048 more slots), for any
// key distribution.  Each warp sorts runs of 64 keys in registers (bitonic,
// 2 per lane; kTopK / (2 T) runs per warp); then five merge-path levels merge
// runs of 64, 128, ... 1024 keys with 512 threads.  Every thread of the block
// must call it; returns the buffer that holds the result.
template <int T>
__device__ uint64_t* sort_desc_2048_merge(uint64_t* buf, uint64_t* tmp) {
  const int t = threadIdx.x;
  const int lane = t & 31;
#pragma unroll 1
  for (int half = 0; half < kTopK / (2 * T); ++half) {
  uint64_t* run = buf + half * 2 * T;
  uint64_t x0 = run[2 * t], x1 = run[2 * t + 1];
#pragma unroll
  for (int kk = 1; kk <= 6; ++kk) {
    const int k = 1 << kk;
#pragma unroll
    for (int jj = kk - 1; jj >= 0; --jj) {
      const int j = 1 << jj;
      const int i0 = 2 * lane;                       // position inside the warp's 64
      const bool desc = k == 64 || (i0 & k) == 0;    // the last stage sorts all descending
      if (j == 1) {
        if (desc ? (x0 < x1) : (x0 > x1)) { const uint64_t tt = x0; x0 = x1; x1 = tt; }
      } else {
        const uint64_t y0 = shfl_xor64(x0, j >> 1), y1 = shfl_xor64(x1, j >> 1);
        const bool keep_max = ((i0 & j) == 0) == desc;
        x0 = keep_max ? (x0 > y0 ? x0 : y0) : (x0 < y0 ? x0 : y0);
        x1 = keep_max ? (x1 > y1 ? x1 : y1) : (x1 < y1 ? x1 : y1);
      }
    }
  }
  *reinterpret_cast<ulonglong2*>(run + 2 * t) = make_ulonglong2(x0, x1);
  }
  uint64_t* src = buf;
  uint64_t* dst = tmp;
  __syncthreads();
  // Merge levels: kMergeOut consecutive outputs per thread, so one binary
  // search (merge-path split) per kMergeOut outputs.
#pragma unroll 1
  for (int R = 64; R < kTopK; R <<= 1) {
    if (t < kTopK / kMergeOut) {
      const int o = kMergeOut * t;         // first of this thread's outputs
      const int pair = o / (2 * R);
      const int d = o - pair * 2 * R;      // diagonal inside the pair
      const uint64_t* A = src + pair * 2 * R;
      const uint64_t* B = A + R;
      // number of A keys among the d largest of A u B
      int lo = d > R ? d - R : 0, hi = d < R ? d : R;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (A[mid] > B[d - 1 - mid]) lo = mid + 1; else hi = mid;
      }
      int ia = lo, ib = d - lo;
      uint64_t a = ia < R ? A[ia] : 0ull, bb = ib < R ? B[ib] : 0ull;
      uint64_t r[kMergeOut];
#pragma unroll
      for (int k = 0; k < kMergeOut; ++k) {
        const bool take_a = ib >= R || (ia < R && a > bb);
        r[k] = take_a ? a : bb;
        if (take_a) { ++ia; a = ia < R ? A[ia] : 0ull; }
        else { ++ib; bb = ib < R ? B[ib] : 0ull; }
      }
#pragma unroll
      for (int k = 0; k < kMergeOut; k += 2)
        *reinterpret_cast<ulonglong2*>(dst + o + k) = make_ulonglong2(r[k], r[k + 1]);
    }
    __syncthreads();
    uint64_t* sw = src; src = dst; dst = sw;
  }
  return src;
}

// Descending sort of the 2048 keys in buf: the non-zero keys first (all
// distinct: they carry their token index), then the zero padding keys of a
// row shorter than 2048, which stay where the caller put them (at the end).
// Bucket sort: an 11-bit digit of the score word (key >> 32) over the
// non-zero keys' own range of score words gives 2048 buckets in descending
// key order; shared-memory atomics count them, a block scan places them, and
// each key's position inside its bucket is the number of the bucket's keys
// greater than it (full 64-bit compare, so equal scores order by token).  If
// the keys crowd into a few buckets (a bucket above kBucketCap keys), the
// merge sort above runs instead.  tmp: 2048 keys; cnt: 2048 counters;
// scratch: 64 words; flag: one int, zero on entry.  Every thread of the block
// must call it; returns the buffer that holds the result.
constexpr int kBucketCap = 48;

template <int T>
__device__ uint64_t* sort_desc_2048(uint64_t* buf, uint64_t* tmp, uint32_t* cnt, int* warp_tot,
                                    uint32_t* scratch, int* flag) {
  constexpr int K = kTopK / T;  // keys per thread (consecutive), and buckets per thread
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int warp = t >> 5;
  uint64_t x[K];
  bool v[K];
#pragma unroll
  for (int k = 0; k < K; k += 2) {
    const ulonglong2 xx = *reinterpret_cast<const ulonglong2*>(buf + K * t + k);
    x[k] = xx.x;
    x[k + 1] = xx.y;
  }
  uint32_t hmax = 0u, hmin = 0xFFFFFFFFu;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    v[k] = x[k] != 0;
    const uint32_t h = static_cast<uint32_t>(x[k] >> 32);
    hmax = max(hmax, v[k] ? h : 0u);
    hmin = min(hmin, v[k] ? h : 0xFFFFFFFFu);
  }
  uint32_t mx = __reduce_max_sync(0xffffffffu, hmax);
  uint32_t mn = __reduce_min_sync(0xffffffffu, hmin);
  if (lane == 0) { scratch[warp] = mx; scratch[32 + warp] = mn; }
  for (int i = t; i < kTopK; i += T) cnt[i] = 0;
  __syncthreads();
  mx = __reduce_max_sync(0xffffffffu, lane < T / 32 ? scratch[lane] : 0u);
  mn = __reduce_min_sync(0xffffffffu, lane < T / 32 ? scratch[32 + lane] : 0xFFFFFFFFu);
  if (mx < mn) return buf;  // no non-zero keys
  const uint32_t span = mx - mn;
  const int shift = span < 2048 ? 0 : 32 - __clz(static_cast<int>(span)) - 11;
  int bk[K], sl[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    bk[k] = v[k] ? 2047 - static_cast<int>((static_cast<uint32_t>(x[k] >> 32) - mn) >> shift) : 0;
    sl[k] = v[k] ? static_cast<int>(atomicAdd(&cnt[bk[k]], 1u)) : 0;
  }
  __syncthreads();
  // Thread t owns buckets K t .. K t + K - 1: counts -> exclusive starts.
  int c[K];
  int sum = 0;
  bool over = false;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    c[k] = static_cast<int>(cnt[K * t + k]);
    sum += c[k];
    over = over || c[k] > kBucketCap;
  }
  if (over) atomicOr(flag, 1);
  int nvalid;
  int run = block_scan_incl<T>(sum, warp_tot, nvalid) - sum;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    cnt[K * t + k] = run;
    run += c[k];
  }
  __syncthreads();  // also orders the flag's atomics before its read
  if (*flag) return sort_desc_2048_merge<T>(buf, tmp);
#pragma unroll
  for (int k = 0; k < K; ++k)
    if (v[k]) tmp[cnt[bk[k]] + sl[k]] = x[k];
  __syncthreads();
  // Rank inside the bucket; the zero keys at buf[nvalid..] are not touched.
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (v[k]) {
      const int st = cnt[bk[k]], en = bk[k] < 2047 ? static_cast<int>(cnt[bk[k] + 1]) : nvalid;
      int r = 0;
      for (int j = st; j < en; ++j) r += tmp[j] > x[k] ? 1 : 0;
      buf[st + r] = x[k];
    }
  }
  __syncthreads();
  return buf;
}

template <int T>
__global__ void __launch_bounds__(T, 1024 / T) topk_select_kernel(const SelectParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint64_t* sel = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* stage = sel + kTopK;
  uint32_t* hist = reinterpret_cast<uint32_t*>(stage + (T / 32) * kStageCap);
  uint32_t* hist2 = hist + kBins;                         // second-level histogram
  int* warp_tot = reinterpret_cast<int*>(hist2 + kBins);  // 32 ints
  int* res = warp_tot + 32;                               // bin, above, count, overflow, nsel
  int* wcnt = res + 8;                                    // staged keys per warp

  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int max_len = p.max_pages * kPage;
  // Launched programmatically after the score kernel.  Without ready counts
  // nothing in global memory is touched before that grid has completed; with
  // them, a row's scores and histogram are read once its own request's
  // tiles are scored (the counts are released after the stores they cover).
  if (p.ready == nullptr) griddep_wait();
  griddep_launch_dependents();
  int L = __ldg(p.seq_lens + b);
  L = L < 0 ? 0 : (L > max_len ? max_len : L);  // the score kernel flags bad lengths
  const int bt_row = p.row_req ? __ldg(p.row_req + b) : b;
  if (bt_row < 0) L = 0;  // a row outside every request: all -1
  if (p.ready != nullptr) {
    if (tid == 0) {
      // Each of the request's tiles is scored by four epilogue warps.
      const unsigned int need = 4u * static_cast<unsigned int>((L + kTileTok - 1) / kTileTok);
      const unsigned int base = p.ready[2 * b + 1];
      const bool ok = wait_count_since(p.ready + 2 * b, base, need, p.status, p.wait_limit_ns);
      // The consumed count moves past this call's tiles; after a timeout it
      // resynchronises with whatever was scored.
      p.ready[2 * b + 1] = ok ? base + need : ld_acquire_gpu_u32(p.ready + 2 * b);
      res[7] = ok ? 1 : 0;
    }
    __syncthreads();
    if (!res[7]) L = 0;  // the wait gave up (reported): the row is written as all -1
  }
  // Score rows are read through L2 only (ld.global.cg): with ready counts the
  // score grid may still be writing other rows, and each score is read once.
  const float* row = p.scores + static_cast<int64_t>(b) * p.score_stride;
  const unsigned int* ghist = p.hist + static_cast<int64_t>(b) * kBins;
  const int K = L < kTopK ? L : kTopK;
  const float4* row4 = reinterpret_cast<const float4*>(row);
  const int L4 = (L + 3) >> 2;  // float4s covering [0, L)
  // The histogram the score kernel accumulated for this request, copied
  // into shared memory ahead of the scores (no registers held meanwhile).
  if (L > kTopK && tid < kBins / 4) cp_async16(smem_u32(hist + 4 * tid), ghist + 4 * tid);
  // The main pass's first scores need no threshold: their loads are in
  // flight while the boundary bin is found.
  float4 nv[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int q = u * T + tid;
    nv[u] = (L > kTopK && q < L4) ? __ldcg(row4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int i = tid; i < kBins; i += T) hist2[i] = 0u;
  if (tid == 0) { res[3] = 0; res[4] = 0; res[5] = 0; }
  cp_async_wait_all();
  __syncthreads();

  if (L <= kTopK) {
    for (int i = tid; i < kTopK; i += T) sel[i] = i < L ? composite(__ldcg(row + i), i) : 0ull;
    __syncthreads();
  } else {
    find_bin<T>(hist, K, warp_tot, res);
    const uint32_t bin1 = static_cast<uint32_t>(res[0]);
    int need = K - res[1];
    int count = res[2];
    // One pass over the scores: every key whose top 11 bits are >= bin1 goes
    // to this warp's private staging area.  key >= bin1 << 21 is one
    // unordered float compare against the float with that key (NaN ranks
    // highest).  Each thread loads 4 float4 (16 scores) per round and packs
    // its verdicts into a 16-bit mask; a warp scan of the mask popcounts
    // places the (rare) winners, whose token indices are staged; their
    // scores are fetched after the pass with independent loads (a re-read
    // inside the loop would serialise one L2 round trip per winner).
    const uint32_t tkey = bin1 << 21;
    float thr = __uint_as_float((tkey & 0x80000000u) ? (tkey & 0x7FFFFFFFu) : ~tkey);
    // Bins above +inf hold only NaN (every NaN has the top key): stage NaN
    // and +inf then; the refinement below drops the +inf keys again.
    if (thr != thr) thr = INFINITY;
    uint64_t* mine = stage + warp * kStageCap;
    int wcount = 0;
    // Loads run one round ahead of the compares, so the L2 latency of round
    // r + 1 overlaps the work on round r (round 0's were issued on entry).
    for (int q0 = 0; q0 < L4; q0 += 4 * T) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        v[u] = nv[u];
        const int q = q0 + (4 + u) * T + tid;
        nv[u] = q < L4 ? __ldcg(row4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      uint32_t msk = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        msk |= (!(v[u].x < thr) ? 1u : 0u) << (4 * u);
        msk |= (!(v[u].y < thr) ? 2u : 0u) << (4 * u);
        msk |= (!(v[u].z < thr) ? 4u : 0u) << (4 * u);
        msk |= (!(v[u].w < thr) ? 8u : 0u) << (4 * u);
      }
      if (q0 + 4 * T > L4 - 1) {  // last round: drop positions >= L
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i0 = 4 * (q0 + u * T + tid);
          const int nv = L - i0;
          const uint32_t keep = nv >= 4 ? 0xFu : (nv > 0 ? (1u << nv) - 1u : 0u);
          msk &= ~(0xFu << (4 * u)) | (keep << (4 * u));
        }
      }
      const int cnt = __popc(msk);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int wtot = __shfl_sync(0xffffffffu, incl, 31);
      if (wtot) {
        int pos = wcount + incl - cnt;
        while (msk) {
          const int bit = __ffs(msk) - 1;
          msk &= msk - 1;
          const int i = 4 * (q0 + (bit >> 2) * T + tid) + (bit & 3);
          if (pos < kStageCap) mine[pos] = static_cast<uint64_t>(i);
          ++pos;
        }
        wcount += wtot;
      }
    }
    if (lane == 0) {
      wcnt[warp] = wcount;
      if (wcount > kStageCap) atomicOr(&res[3], 1);
    }
    __syncthreads();
    const bool staged = res[3] == 0;
    if (staged) {
      // Scores of this warp's staged tokens, four independent loads in
      // flight per lane; keys of the boundary bin count into the histogram
      // of the first refinement pass (hist2: next 11 key bits).  Selecting
      // the winners' scores from the main pass's registers instead measured
      // slower: the longer-lived registers spill, and any load the loop
      // waits on then waits behind the next round's score loads.
      const int avail = wcount;
      for (int j0 = lane; j0 < avail; j0 += 128) {
        int ti[4];
        float sv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) ti[u] = j0 + 32 * u < avail ? static_cast<int>(mine[j0 + 32 * u]) : 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) sv[u] = j0 + 32 * u < avail ? __ldcg(row + ti[u]) : 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (j0 + 32 * u < avail) {
            const uint64_t c = composite(sv[u], ti[u]);
            mine[j0 + 32 * u] = c;
            if (static_cast<uint32_t>(c >> 53) == bin1) atomicAdd(&hist2[(c >> 42) & 0x7FF], 1u);
          }
        }
      }
      __syncthreads();
    }
    uint64_t prefix = static_cast<uint64_t>(bin1) << 53;
    uint64_t mask = static_cast<uint64_t>(0x7FF) << 53;
    // Refine the boundary: 11-bit digits of the remaining 53 key bits.  With
    // the keys staged, the first pass's histogram (hist2) was built above.
    const int shifts[5] = {42, 31, 20, 9, 0};
    const int widths[5] = {11, 11, 11, 11, 9};
    for (int pass = 0; pass < 5 && count != need; ++pass) {
      const int sh = shifts[pass];
      const uint64_t dm = (static_cast<uint64_t>(1) << widths[pass]) - 1;
      if (pass > 0 || !staged) {
        for (int i = tid; i < kBins; i += T) hist[i] = 0;
        __syncthreads();
        if (staged) {
          const uint64_t* area = stage + warp * kStageCap;
          const int avail = wcnt[warp];
          for (int j = lane; j < avail; j += 32) {
            const uint64_t c = area[j];
            if ((c & mask) == prefix) atomicAdd(&hist[(c >> sh) & dm], 1u);
          }
        } else {
          for (int i = tid; i < L; i += T) {
            const uint64_t c = composite(__ldcg(row + i), i);
            if ((c & mask) == prefix) atomicAdd(&hist[(c >> sh) & dm], 1u);
          }
        }
        __syncthreads();
      }
      find_bin<T>(pass == 0 && staged ? hist2 : hist, need, warp_tot, res);
      prefix |= static_cast<uint64_t>(res[0]) << sh;
      mask |= dm << sh;
      need -= res[1];
      count = res[2];
    }
    // The K winners are the keys with (c & mask) >= prefix.
    if (staged) {
      // Lane l of warp w owns slots l + 32k of the warp's area (no bank
      // conflicts): count, block scan, write.
      const uint64_t* area = stage + warp * kStageCap;
      const int avail = wcnt[warp];
      int cnt = 0;
      for (int j = lane; j < avail; j += 32) cnt += (area[j] & mask) >= prefix ? 1 : 0;
      int total;
      const int incl = block_scan_incl<T>(cnt, warp_tot, total);
      int pos = incl - cnt;
      for (int j = lane; j < avail; j += 32) {
        const uint64_t c = area[j];
        if ((c & mask) >= prefix) {
          if (pos < kTopK) sel[pos] = c;
          ++pos;
        }
      }
    } else {
      const int Lr = (L + 31) & ~31;
      for (int i = tid; i < Lr; i += T) {
        const bool in = i < L;
        const uint64_t c = in ? composite(__ldcg(row + i), i) : 0ull;
        warp_append(in && (c & mask) >= prefix, c, sel, &res[4], kTopK);
      }
    }
    __syncthreads();
  }

  const uint64_t* sorted =
      sort_desc_2048<T>(sel, stage, hist, warp_tot, reinterpret_cast<uint32_t*>(stage + kTopK), &res[5]);

  int32_t* out = p.out + static_cast<int64_t>(b) * kTopK;
  const int32_t* bt = p.block_table + static_cast<int64_t>(bt_row < 0 ? 0 : bt_row) * p.max_pages;
  for (int i = tid; i < kTopK; i += T) {
    int32_t v = -1;
    if (i < K) {
      const int tok = static_cast<int>(~static_cast<uint32_t>(sorted[i]));
      if (tok >= 0 && tok < L) {
        v = __ldg(bt + (tok >> 6)) * kPage + (tok & 63);
      } else {  // only if the histogram did not match the scores
        atomicOr(p.status, DSA_DEV_STALE_WORKSPACE);
      }
    }
    out[i] = v;
  }
}

std::once_flag g_attr_once[64];
int g_attr_status[64];
std::once_flag g_sel_attr_once[64];
int g_sel_attr_status[64];

// One armed test fault (dsa_b200_test_inject, kind DSA_TEST_SKIP_READY),
// consumed by the next dsa_indexer_run: kind << 56 | the select's wait limit
// in ns; 0 = none.
std::atomic<unsigned long long> g_inject{0};

}  // namespace ix

void arm_indexer_test_fault(unsigned long long armed) { ix::g_inject.store(armed); }

int launch_topk_select(const float* scores, const unsigned int* hist, const int32_t* seq_lens,
                       const int32_t* block_table, const int32_t* row_req, int32_t* out, int rows,
                       int score_stride, int max_pages, unsigned int* status, unsigned int* ready,
                       unsigned long long wait_limit_ns, const DeviceInfo& info, cudaStream_t s) {
  if (ix::sel_smem<1024>() > info.max_smem_optin) return DSA_ERR_UNSUPPORTED_DEVICE;
  std::call_once(ix::g_sel_attr_once[info.device], [&]() {
    ix::g_sel_attr_status[info.device] =
        cudaFuncSetAttribute(ix::topk_select_kernel<1024>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(ix::sel_smem<1024>())) == cudaSuccess &&
                cudaFuncSetAttribute(ix::topk_select_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(ix::sel_smem<512>())) == cudaSuccess
            ? DSA_OK
            : DSA_ERR_CUDA;
  });
  if (ix::g_sel_attr_status[info.device] != DSA_OK) return ix::g_sel_attr_status[info.device];
  ix::SelectParams selp;
  selp.scores = scores;
  selp.row_req = row_req;
  selp.status = status;
  selp.hist = hist;
  selp.seq_lens = seq_lens;
  selp.block_table = block_table;
  selp.out = out;
  selp.ready = ready;
  selp.wait_limit_ns = wait_limit_ns;
  selp.score_stride = score_stride;
  selp.max_pages = max_pages;
  // One 1024-thread CTA per row while the rows fit the SMs in one wave (the
  // select is then a latency chain per row); more rows than SMs run two
  // 512-thread CTAs per SM, where the select is throughput-bound.
  const cudaError_t e =
      rows > info.num_sms
          ? launch_programmatic(ix::topk_select_kernel<512>, dim3(rows), dim3(512), ix::sel_smem<512>(), s, selp)
          : launch_programmatic(ix::topk_select_kernel<1024>, dim3(rows), dim3(1024), ix::sel_smem<1024>(), s,
                                selp);
  if (e != cudaSuccess) return DSA_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}

}  // namespace dsa

using namespace dsa;

extern "C" size_t dsa_indexer_workspace_bytes(int32_t batch, int32_t max_pages) {
  if (batch < 0 || max_pages < 0) return 0;
  return kWorkspaceHeader + ix::kReadyBytes + sizeof(uint32_t) * static_cast<size_t>(batch) * ix::kBins +
         sizeof(float) * static_cast<size_t>(batch) * static_cast<size_t>(max_pages) * ix::kPage;
}

extern "C" int dsa_indexer_run(const void* q_index_fp8, const void* k_index_cache_fp8,
                               int64_t num_pages, const float* weights, const int32_t* seq_lens,
                               const int32_t* block_table, int32_t batch, int32_t max_pages,
                               int32_t* topk_indices, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (batch < 0 || batch > ix::kMaxBatch) return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0) return DSA_OK;
  if (!q_index_fp8 || !k_index_cache_fp8 || !weights || !seq_lens || !block_table ||
      !topk_indices || !workspace)
    return DSA_ERR_INVALID_ARGUMENT;
  if (max_pages < 1 || max_pages > ix::kMaxPagesPerSeq) return DSA_ERR_INVALID_ARGUMENT;
  if (num_pages < 1 || num_pages > ix::kMaxPool) return DSA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_index_fp8) || !aligned16(k_index_cache_fp8) || !aligned16(workspace))
    return DSA_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(weights) | reinterpret_cast<uintptr_t>(seq_lens) |
       reinterpret_cast<uintptr_t>(block_table) | reinterpret_cast<uintptr_t>(topk_indices)) & 3u)
    return DSA_ERR_MISALIGNED;
  if (workspace_bytes < dsa_indexer_workspace_bytes(batch, max_pages))
    return DSA_ERR_WORKSPACE_TOO_SMALL;

  DeviceInfo info;
  int st = current_device_info(&info);
  if (st != DSA_OK) return st;
  const size_t smem1 = ix::score_smem_bytes(batch);
  if (smem1 > info.max_smem_optin || ix::sel_smem<1024>() > info.max_smem_optin)
    return DSA_ERR_UNSUPPORTED_DEVICE;
  std::call_once(ix::g_attr_once[info.device], [&]() {
    bool ok = cudaFuncSetAttribute(ix::indexer_score_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(info.max_smem_optin)) == cudaSuccess;
    ix::g_attr_status[info.device] = ok ? DSA_OK : DSA_ERR_CUDA;
  });
  if (ix::g_attr_status[info.device] != DSA_OK) return ix::g_attr_status[info.device];

  CUtensorMap kmap, qmap;
  st = encode_tmap_2d(&kmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_index_cache_fp8, 128,
                      static_cast<uint64_t>(num_pages) * ix::kPageRows, 128, 128, 64);
  if (st != DSA_OK) return st;
  st = encode_tmap_2d(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, q_index_fp8, 128,
                      static_cast<uint64_t>(batch) * ix::kHeads, 128, 128, 64);
  if (st != DSA_OK) return st;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  {
    // Launched normally: it starts after every earlier write to the inputs,
    // so the score kernel (launched programmatically after it) may read them
    // at once; only its histogram flushes wait for the clearing.
    const int64_t n16 = static_cast<int64_t>(batch) * ix::kBins * 4 / 16;
    const int blocks = static_cast<int>(std::min<int64_t>((n16 + 255) / 256, info.num_sms));
    ix::hist_clear_kernel<<<blocks, 256, 0, s>>>(
        reinterpret_cast<uint4*>(static_cast<uint8_t*>(workspace) + kWorkspaceHeader + ix::kReadyBytes), n16);
  }
  ix::ScoreParams sp;
  sp.k_cache = static_cast<const uint8_t*>(k_index_cache_fp8);
  sp.weights = weights;
  sp.seq_lens = seq_lens;
  sp.block_table = block_table;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  sp.ready = reinterpret_cast<unsigned int*>(ws + kWorkspaceHeader);
  sp.hist = reinterpret_cast<unsigned int*>(ws + kWorkspaceHeader + ix::kReadyBytes);
  sp.scores = reinterpret_cast<float*>(ws + kWorkspaceHeader + ix::kReadyBytes +
                                       sizeof(uint32_t) * static_cast<size_t>(batch) * ix::kBins);
  sp.status = static_cast<unsigned int*>(workspace);
  sp.num_pages = num_pages;
  sp.batch = batch;
  sp.max_pages = max_pages;
  sp.score_stride = max_pages * ix::kPage;
  sp.skip_ready_req = -1;
  unsigned long long wait_limit_ns = kWaitLimitNs;
  if (ix::g_inject.load(std::memory_order_relaxed) != 0) {
    const unsigned long long armed = ix::g_inject.exchange(0);
    if ((armed >> 56) == DSA_TEST_SKIP_READY) {
      sp.skip_ready_req = 0;
      wait_limit_ns = armed & ((1ull << 56) - 1);
    }
  }
  if (launch_programmatic(ix::indexer_score_kernel, dim3(info.num_sms), dim3(ix::kThreads), smem1, s,
                          kmap, qmap, sp) != cudaSuccess)
    return DSA_ERR_CUDA;

  return launch_topk_select(sp.scores, sp.hist, seq_lens, block_table, nullptr, topk_indices, batch,
                            sp.score_stride, max_pages, sp.status, sp.ready, wait_limit_ns, info, s);
}
