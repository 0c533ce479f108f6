// prefill.cu -- DSA lightning indexer for many query rows per request
// (prefill / chunked prefill) on sm_100a.
//
// Every query row t of request r is one decode-indexer problem: the top-2048
// tokens of  score(s) = sum_h w[t,h] * relu(scale_s * (q[t,h] . k_s))  over
// the first seq_lens[t] tokens of r's pages block_table[r, :] (causal rows
// see growing prefixes).  The decode kernel streams a request's K pages once
// per query row; with thousands of rows per request that is one K pass per
// row (34 GB of L2 traffic for 4096 rows over 65536 tokens).  Here the rows
// of a request are taken four at a time as the N dimension of a real FP8
// GEMM, so every 128-token K tile is read once per four rows and the
// tensor core, not the memory system, sets the pace:
//
//   prefill_plan_kernel (one CTA)  groups of <= 4 consecutive rows of one
//       request, the number of 128-token tiles each group needs (its longest
//       row), their prefix sums, and the request of every row.
//   prefill_score_kernel (persistent, one CTA per SM)  the (group, tile)
//       units are cut into equal contiguous slices.  Roles:
//         warps 16,17 TMA producers (alternate tiles): two 64-token FP8 pages
//                     (128-byte swizzle) into a 6-stage ring, their fp32
//                     scales into an 8-slot ring.
//         warps 18,19 MMA issuers (alternate tiles): tcgen05.mma
//                     kind::f8f6f4, M = 128 tokens, N = 256 (4 rows x 64
//                     heads), K = 128 (4 x K32), fp32 accumulators in TMEM
//                     (2 stages x 256 columns = all 512).  Warp 18 also loads
//                     a group's q rows (one 32 KB TMA box) and weights.
//         warps 0-15  epilogue: warp w reads TMEM sub-partition w & 3 (token
//                     rows) for query row w >> 2: sum_h w_h * relu(scale *
//                     acc_h) per token in registers, then the fp32 score and
//                     its radix-histogram count.  Four warps per scheduler
//                     keep enough independent FMA chains in flight.
//   topk_select_kernel (indexer.cu), one CTA per row, with the row's request
//       resolving its block-table row.
#include <mutex>

#include "host.h"
#include "ptx.cuh"

namespace dsa {
namespace pf {

constexpr int kPage = DSA_PAGE_SIZE;
constexpr int kHeads = DSA_INDEX_HEADS;                   // 64
constexpr int kDim = DSA_INDEX_DIM;                       // 128
constexpr int kPageBytes = DSA_INDEX_PAGE_BYTES;          // 8448
constexpr int kPageRows = kPageBytes / 128;               // 66
constexpr int kPageDataBytes = kPage * kDim;              // 8192
constexpr int kScaleBytes = kPage * 4;                    // 256
constexpr int kTileTok = 2 * kPage;                       // 128
constexpr int kGroupRows = 4;                             // query rows per unit
constexpr int kN = kGroupRows * kHeads;                   // 256
constexpr int kStageBytes = 2 * kPageDataBytes;           // 16384
constexpr int kStages = 6;
constexpr int kAccStages = 2;
constexpr int kTmemCols = kAccStages * kN;                // 512
constexpr int kScaleSlots = kStages + kAccStages;         // 8 (see the decode kernel)
constexpr int kQBytes = kN * kDim;                        // 32768
constexpr int kWBytes = kGroupRows * kHeads * 4;          // 1024
constexpr int kBins = 2048;
constexpr int kEpiWarps = 16;                             // four per TMEM sub-partition
constexpr int kProdWarp0 = 16;
constexpr int kProdWarps = 2;
constexpr int kMmaWarp0 = 18;
constexpr int kMmaWarps = 2;
constexpr int kThreads = 32 * (kMmaWarp0 + kMmaWarps);    // 640
constexpr int kPlanThreads = 1024;
constexpr int kMaxRows = 1 << 20;

constexpr uint32_t kIdesc = idesc_make(0, 0, false, false, 128, kN);

constexpr int kOffStage = 0;
constexpr int kOffQ = kOffStage + kStages * kStageBytes;              // 98304
constexpr int kOffW = kOffQ + 2 * kQBytes;                            // 163840
constexpr int kOffScale = kOffW + 2 * kWBytes;                        // 165888
constexpr int kOffHist = kOffScale + kScaleSlots * 2 * kScaleBytes;   // 169984
constexpr int kOffBar = kOffHist + kGroupRows * kBins * 4;            // 202752
constexpr int kOffMisc = kOffBar + 256;
constexpr int kOffInfo = kOffMisc + 64;                               // producer warps x 32 tiles
constexpr int kSmemBytes = 1024 + kOffInfo + kProdWarps * 32 * 12;
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kStages % kProdWarps == 0 && kScaleSlots % kProdWarps == 0, "producer stride");

// One group: rows [row0, row0 + nrows) of request req, `tiles` 128-token
// tiles (enough for its longest row).
struct Group {
  int row0, nrows, req, tiles;
};

struct PlanParams {
  const int32_t* cu_rows;   // [num_req + 1]
  const int32_t* seq_lens;  // [num_rows]
  Group* groups;            // [group_cap]
  int* tile_off;            // [group_cap + 1]: prefix sums of tiles; [group_cap] = number of groups
  int* req_gbase;           // [num_req + 1] scratch: first group of each request
  int32_t* row_req;         // [num_rows] request of each row (-1: in no request)
  unsigned int* status;
  int num_req, num_rows, group_cap, max_len;
};

struct ScoreParams {
  const uint8_t* k_cache;
  const float* weights;     // [num_rows][64]
  const int32_t* seq_lens;  // [num_rows]
  const int32_t* block_table;  // [num_req][max_pages]
  const Group* groups;
  const int* tile_off;      // [num_groups + 1], num_groups at tile_off[group_cap]
  float* scores;            // [num_rows][score_stride]
  unsigned int* hist;       // [num_rows][kBins], cleared by an async memset at every call
  unsigned int* status;
  int64_t num_pages;
  int num_rows, group_cap, max_pages, score_stride;
};

__device__ __forceinline__ int clamp_len(int L, int max_len, unsigned int* status) {
  if (L < 0 || L > max_len) {
    atomicOr(status, DSA_DEV_BAD_SEQ_LEN);
    L = L < 0 ? 0 : max_len;
  }
  return L;
}

// Inclusive prefix sum over the block (blockDim.x == kPlanThreads).
__device__ __forceinline__ int block_scan_incl(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    warp_tot[lane] = t;
  }
  __syncthreads();
  const int add = warp > 0 ? warp_tot[warp - 1] : 0;
  const int total = warp_tot[31];
  __syncthreads();
  warp_tot[32] = total;  // read by the caller after its next barrier
  return v + add;
}

// Request rows [lo_r, hi_r): cu_rows clamped into [0, num_rows] and made
// non-decreasing, so bad offsets never index outside the arrays.
__device__ __forceinline__ void req_rows(const PlanParams& p, int r, int& lo, int& hi) {
  int a = __ldg(p.cu_rows + r), b = __ldg(p.cu_rows + r + 1);
  a = min(max(a, 0), p.num_rows);
  b = min(max(b, a), p.num_rows);
  lo = a;
  hi = b;
}

__global__ void __launch_bounds__(kPlanThreads, 1) prefill_plan_kernel(const PlanParams p) {
  __shared__ int warp_tot[33];
  const int tid = threadIdx.x;
  griddep_launch_dependents();  // the score kernel waits for this grid before reading the plan
  if (tid == 0) {
    const int c0 = __ldg(p.cu_rows), cn = __ldg(p.cu_rows + p.num_req);
    if (c0 != 0 || cn != p.num_rows) atomicOr(p.status, DSA_DEV_BAD_SEQ_LEN);
  }
  for (int t = tid; t < p.num_rows; t += kPlanThreads) p.row_req[t] = -1;
  // Groups per request -> first group of each request.
  int carry = 0;
  for (int base = 0; base < p.num_req; base += kPlanThreads) {
    const int r = base + tid;
    int ng = 0;
    if (r < p.num_req) {
      int lo, hi;
      req_rows(p, r, lo, hi);
      if (__ldg(p.cu_rows + r + 1) < __ldg(p.cu_rows + r)) atomicOr(p.status, DSA_DEV_BAD_SEQ_LEN);
      ng = (hi - lo + kGroupRows - 1) / kGroupRows;
    }
    const int incl = block_scan_incl(ng, warp_tot);
    if (r < p.num_req) p.req_gbase[r] = carry + incl - ng;
    __syncthreads();
    carry += warp_tot[32];
    __syncthreads();
  }
  if (tid == 0) p.req_gbase[p.num_req] = carry;
  const int ngroups = min(carry, p.group_cap);
  __syncthreads();
  // Each group: rows, request, tiles; then prefix sums of the tiles.
  carry = 0;
  for (int base = 0; base < ngroups; base += kPlanThreads) {
    const int g = base + tid;
    int tiles = 0;
    if (g < ngroups) {
      int lo = 0, hi = p.num_req - 1;  // last request with req_gbase <= g
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.req_gbase[mid] <= g) lo = mid; else hi = mid - 1;
      }
      const int r = lo;
      int rlo, rhi;
      req_rows(p, r, rlo, rhi);
      const int row0 = rlo + kGroupRows * (g - p.req_gbase[r]);
      const int n = min(kGroupRows, rhi - row0);
      int maxL = 0;
      for (int i = 0; i < n; ++i) {
        maxL = max(maxL, clamp_len(__ldg(p.seq_lens + row0 + i), p.max_len, p.status));
        p.row_req[row0 + i] = r;
      }
      tiles = (maxL + kTileTok - 1) / kTileTok;
      p.groups[g] = Group{row0, n, r, tiles};
    }
    const int incl = block_scan_incl(tiles, warp_tot);
    if (g < ngroups) p.tile_off[g] = carry + incl - tiles;
    __syncthreads();
    carry += warp_tot[32];
    __syncthreads();
  }
  if (tid == 0) {
    p.tile_off[ngroups] = carry;
    p.tile_off[p.group_cap] = ngroups;
  }
}

// Group g with tile_off[g] <= u < tile_off[g + 1].
__device__ __forceinline__ int locate_group(const int* tile_off, int ngroups, int64_t u) {
  int lo = 0, hi = ngroups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(tile_off + mid) <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Walks a CTA's units in order: group, tile j inside it.  Groups with no
// tiles (all rows of length 0) are skipped.
struct Cursor {
  int g, j, ntiles;
  __device__ __forceinline__ void start(const int* tile_off, int ngroups, int64_t u) {
    g = locate_group(tile_off, ngroups, u);
    j = static_cast<int>(u - __ldg(tile_off + g));
    ntiles = __ldg(tile_off + g + 1) - __ldg(tile_off + g);
  }
  // Advances by one unit; returns true when a new group starts.
  __device__ __forceinline__ bool next(const int* tile_off, int ngroups) {
    if (++j < ntiles) return false;
    j = 0;
    do {
      ++g;
      ntiles = g < ngroups ? __ldg(tile_off + g + 1) - __ldg(tile_off + g) : 1;
    } while (ntiles == 0);
    return true;
  }
};

__device__ __forceinline__ int page_id(const ScoreParams& p, int req, int page_idx) {
  int pid = __ldg(p.block_table + static_cast<int64_t>(req) * p.max_pages + page_idx);
  if (pid < 0 || pid >= p.num_pages) {
    atomicOr(p.status, DSA_DEV_BAD_PAGE);
    pid = 0;
  }
  return pid;
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_score_kernel(const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap qmap, const ScoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_mem = smem + kOffStage;
  uint8_t* q_mem = smem + kOffQ;
  const float* w_mem = reinterpret_cast<const float*>(smem + kOffW);
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + kOffHist);  // [set][row of pair][bin]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* accfull = qempty + 2;
  uint64_t* accempty = accfull + kAccStages;
  uint64_t* drain = accempty + kAccStages;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + kOffMisc + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int max_len = p.max_pages * kPage;
  griddep_launch_dependents();

  if (tid == 0) {
    // qempty: both MMA issuers' commits and all eight epilogue warps (the
    // weights live in the same slot).  accfull: MMA commit + issuer arrive
    // (publishes the scale-ring entry).  accempty: the eight epilogue warps.
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(&qfull[s], 1); mbar_init(&qempty[s], kMmaWarps + kEpiWarps); }
    for (int s = 0; s < kAccStages; ++s) { mbar_init(&accfull[s], 2); mbar_init(&accempty[s], kEpiWarps); }
    for (int w = 0; w < kMmaWarps; ++w) mbar_init(&drain[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProdWarp0 && lane == 0) { prefetch_tensor_map(&kmap); prefetch_tensor_map(&qmap); }
  if (warp == kMmaWarp0) tmem_alloc(tmem_base_smem, kTmemCols);
  if (warp < kEpiWarps)
    for (int i = tid; i < kGroupRows * kBins; i += 32 * kEpiWarps) hist_all[i] = 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();  // the plan kernel's groups and offsets

  const uint32_t tmem_base = *tmem_base_smem;
  const int ngroups = __ldg(p.tile_off + p.group_cap);
  const int64_t total = ngroups > 0 ? __ldg(p.tile_off + ngroups) : 0;
  const int u0 = static_cast<int>(total * blockIdx.x / gridDim.x);
  const int u1 = static_cast<int>(total * (blockIdx.x + 1) / gridDim.x);
  const int nt = u1 - u0;
  const WaitCtx wctx{abort_flag, p.status, kWaitLimitNs};

  if (warp >= kProdWarp0 && warp < kProdWarp0 + kProdWarps) {
    // ------------------------------------------------------ producers
    // Warp 8+k owns tiles n = k, k+2, ... of this CTA's slice.  Lane l
    // resolves the l-th of the warp's next 32 tiles (group, its longest row,
    // the two page ids), one batch ahead, into shared memory; lane 0 then
    // issues the copies with no load latency between them.
    const int k = warp - kProdWarp0;
    int* info = reinterpret_cast<int*>(smem + kOffInfo) + k * 32 * 3;  // {p0, p1, npg}
    const int mine = nt > k ? (nt - k + kProdWarps - 1) / kProdWarps : 0;
    if (mine > 0) {
      const uint64_t policy = make_policy_evict_last();  // K tiles are re-read by every group
      // (g, j) of the warp's next unresolved tile, warp-uniform.
      Cursor cur;
      cur.start(p.tile_off, ngroups, u0 + k);
      int rp0 = 0, rp1 = 0, rnpg = 0;  // this lane's resolved tile
      auto resolve = [&](int base) {  // tiles i = base + lane of this warp
        rnpg = 0;
        int g = cur.g, j = cur.j + kProdWarps * lane;
        if (base + lane < mine) {
          int ntl = cur.ntiles;
          while (j >= ntl) { j -= ntl; ++g; ntl = __ldg(p.tile_off + g + 1) - __ldg(p.tile_off + g); }
          const Group gr = p.groups[g];
          int maxL = 0;
          for (int i = 0; i < gr.nrows; ++i)
            maxL = max(maxL, clamp_len(__ldg(p.seq_lens + gr.row0 + i), max_len, p.status));
          const int req_pages = (maxL + kPage - 1) / kPage;
          rnpg = (2 * j + 1 < req_pages) ? 2 : 1;
          rp0 = page_id(p, gr.req, 2 * j);
          rp1 = rnpg == 2 ? page_id(p, gr.req, 2 * j + 1) : 0;
        }
        // Advance the cursor past this batch (64 CTA tiles).
        const int adv = min(32, mine - base) * kProdWarps;
        int g2 = cur.g, j2 = cur.j + adv, ntl2 = cur.ntiles;
        while (j2 >= ntl2 && g2 + 1 < ngroups) {
          j2 -= ntl2; ++g2; ntl2 = __ldg(p.tile_off + g2 + 1) - __ldg(p.tile_off + g2);
        }
        cur.g = g2; cur.j = j2; cur.ntiles = ntl2;
      };
      resolve(0);
      int s = k, sslot = k, m = 0, ok = 1;
      uint32_t ph = 0;
      for (int b0 = 0; b0 < mine && ok; b0 += 32) {
        info[3 * lane] = rp0; info[3 * lane + 1] = rp1; info[3 * lane + 2] = rnpg;
        resolve(b0 + 32);
        __syncwarp();
        const int cnt = min(32, mine - b0);
        if (lane == 0) {
          for (int t = 0; t < cnt; ++t, ++m) {
            const int p0 = info[3 * t], p1 = info[3 * t + 1], npg = info[3 * t + 2];
            if (!mbar_wait(&empty[s], ph ^ 1, wctx)) { ok = 0; break; }
            uint8_t* st = stage_mem + s * kStageBytes;
            uint8_t* sc = smem + kOffScale + sslot * 2 * kScaleBytes;
            mbar_arrive_expect_tx(&full[s], npg * (kPageDataBytes + kScaleBytes));
            tma_load_2d_hint(st, &kmap, &full[s], 0, p0 * kPageRows, policy);
            bulk_load(sc, p.k_cache + static_cast<int64_t>(p0) * kPageBytes + kPageDataBytes,
                      kScaleBytes, &full[s]);
            if (npg == 2) {
              tma_load_2d_hint(st + kPageDataBytes, &kmap, &full[s], 0, p1 * kPageRows, policy);
              bulk_load(sc + kScaleBytes,
                        p.k_cache + static_cast<int64_t>(p1) * kPageBytes + kPageDataBytes,
                        kScaleBytes, &full[s]);
            }
            if ((s += kProdWarps) >= kStages) { s -= kStages; ph ^= 1; }
            if ((sslot += kProdWarps) >= kScaleSlots) sslot -= kScaleSlots;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        m = __shfl_sync(0xffffffffu, m, 0);
        s = __shfl_sync(0xffffffffu, s, 0);
        sslot = __shfl_sync(0xffffffffu, sslot, 0);
        ph = __shfl_sync(0xffffffffu, ph, 0);
        __syncwarp();
      }
      if (lane == 0) {  // let the last copies this thread issued land before the CTA can exit
        for (int i = (m > 2 ? m - 2 : 0); i < m; ++i) {
          const int n = k + kProdWarps * i;
          mbar_drain(&full[n % kStages], static_cast<uint32_t>((n / kStages) & 1), p.status);
        }
      }
    }
    __syncwarp();
  } else if (warp >= kMmaWarp0) {
    // ------------------------------------------------------ MMA issuers
    // Warp 18+r issues the tiles n with n % 2 == r (accumulator r); warp 18
    // also loads each group's q rows and weights once both issuers and all
    // epilogue warps released the slot.
    const int r = warp - kMmaWarp0;
    if (lane == 0 && nt > 0) {
      Cursor cur;
      cur.start(p.tile_off, ngroups, u0);
      int nq = 0, slot = 0, s = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true, new_group = true;
      for (int n = 0; n < nt && ok; ++n) {
        if (n > 0 && cur.next(p.tile_off, ngroups)) new_group = true;
        if (new_group) {
          new_group = false;
          if (nq > 0) umma_commit(&qempty[(nq - 1) & 1]);
          if (r == 0) {
            ok = mbar_wait(&qempty[nq & 1], ((nq >> 1) & 1) ^ 1, wctx);
            if (ok) {
              const Group gr = p.groups[cur.g];
              mbar_arrive_expect_tx(&qfull[nq & 1], kQBytes + gr.nrows * kHeads * 4);
              tma_load_2d(q_mem + (nq & 1) * kQBytes, &qmap, &qfull[nq & 1], 0, gr.row0 * kHeads);
              bulk_load(smem + kOffW + (nq & 1) * kWBytes, p.weights + static_cast<int64_t>(gr.row0) * kHeads,
                        gr.nrows * kHeads * 4, &qfull[nq & 1]);
            }
          }
          ok = ok && mbar_wait(&qfull[nq & 1], (nq >> 1) & 1, wctx);
          slot = nq & 1;
          ++nq;
          if (!ok) break;
        }
        if ((n & 1) == r) {
          ok = mbar_wait(&full[s], ph, wctx) && mbar_wait(&accempty[r], aph ^ 1, wctx);
          if (!ok) break;
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(stage_mem + s * kStageBytes), 16, 1024);
          const uint64_t bd = sdesc_sw128(smem_u32(q_mem + slot * kQBytes), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kDim / 32; ++kk)
            umma_f8(tmem_base + r * kN, ad + 2 * kk, bd + 2 * kk, kIdesc, kk > 0 ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&accfull[r]);
          mbar_arrive(&accfull[r]);
          aph ^= 1;
        }
        if (++s == kStages) { s = 0; ph ^= 1; }
      }
      umma_commit(&drain[r]);
      mbar_drain(&drain[r], 0, p.status);
      if (r == 0)
        for (int j = (nq > 2 ? nq - 2 : 0); j < nq; ++j) mbar_drain(&qfull[j & 1], (j >> 1) & 1, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ epilogue warps
    const int sp = warp & 3;           // TMEM sub-partition: token rows 32*sp .. +31
    const int q = warp >> 2;           // query row of the group
    const int row = sp * 32 + lane;    // token row of the tile
    uint32_t* hist = hist_all + q * kBins;
    const uint32_t bar_id = 1 + q;     // named barrier of row q's four warps
    if (nt > 0) {
      Cursor cur;
      cur.start(p.tile_off, ngroups, u0);
      Group gr{};
      int L = 0;
      int nq = 0;
      // Adds row q's counts into its global histogram and clears them (all
      // four warps of the row, after their last tile of the group).
      auto flush = [&]() {
        named_barrier_sync(bar_id, 128);
        if (q < gr.nrows) {
          unsigned int* g = p.hist + static_cast<int64_t>(gr.row0 + q) * kBins;
          for (int i = sp * 32 + lane; i < kBins; i += 128) {
            const uint32_t c = hist[i];
            if (c) { atomicAdd(g + i, c); hist[i] = 0; }
          }
        }
        named_barrier_sync(bar_id, 128);
      };
      auto enter = [&]() {
        gr = p.groups[cur.g];
        L = q < gr.nrows ? clamp_len(__ldg(p.seq_lens + gr.row0 + q), max_len, p.status) : 0;
      };
      enter();
      int slot = 0, sslot = 0;
      uint32_t aph = 0;
      bool ok = true;
      // After a wait gave up the loop keeps walking the tiles without
      // waiting or working, so the four warps of a row still meet at the
      // same flush barriers.
      for (int n = 0; n < nt; ++n) {
        bool new_group = n == 0;
        if (n > 0 && cur.next(p.tile_off, ngroups)) {
          flush();
          if (lane == 0) mbar_arrive(&qempty[(nq - 1) & 1]);
          enter();
          new_group = true;
        }
        if (new_group) {  // the group's weights (with its q rows) must have landed
          slot = nq & 1;
          ++nq;
          ok = ok && __all_sync(0xffffffffu, mbar_wait(&qfull[slot], ((nq - 1) >> 1) & 1, wctx));
        }
        const int a = n & 1;
        const uint32_t par = aph;
        if (a == 1) aph ^= 1;
        const int ss = sslot;  // this tile's scale slot
        if (++sslot == kScaleSlots) sslot = 0;
        ok = ok && __all_sync(0xffffffffu, mbar_wait(&accfull[a], par, wctx));
        if (!ok) continue;
        tc_fence_after();
        const float scale =
            *reinterpret_cast<const float*>(smem + kOffScale + ss * 2 * kScaleBytes + row * 4);
        // Row q's 64 accumulator columns in one load; the accumulator is
        // handed back before the math.
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + a * kN + q * kHeads;
        float v[64];
        tmem_ld32x2_wait(tbase, tbase + 32, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[a]);
        if (q >= gr.nrows) continue;  // uniform: the group has fewer rows
        const float4* w4 = reinterpret_cast<const float4*>(w_mem + slot * (kWBytes / 4) + q * kHeads);
        float sc;
        if (scale > 0.f) {
          // relu(scale * v) = scale * relu(v) for scale > 0.  The relu is
          // taken doubled, v + |v| = 2 relu(v) (one add, NaN-propagating,
          // -0 -> +0), and the doubled sum halved at the end: scaling by 2
          // commutes with every fp32 rounding, so the score is bit-identical
          // to sum_h w_h relu(v_h) with even and odd heads accumulated
          // separately in head order, as in the decode kernel.
          float f0 = 0.f, f1 = 0.f;
#pragma unroll
          for (int h4 = 0; h4 < 16; ++h4) {
            const float4 ww = w4[h4];
            fma2(f0, f1, relu2(v[4 * h4 + 0]), relu2(v[4 * h4 + 1]), ww.x, ww.y);
            fma2(f0, f1, relu2(v[4 * h4 + 2]), relu2(v[4 * h4 + 3]), ww.z, ww.w);
          }
          sc = scale * (0.5f * (f0 + f1));
        } else {
          // zero, negative or NaN scale: relu(scale * v) term by term
          float g0 = 0.f;
#pragma unroll
          for (int h4 = 0; h4 < 16; ++h4) {
            const float4 ww = w4[h4];
            const float wv[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float x = v[4 * h4 + i] * scale;
              g0 += (x <= 0.f ? 0.f : x) * wv[i];
            }
          }
          sc = g0;
        }
        const int tok = cur.j * kTileTok + row;
        if (tok < L) {
          p.scores[static_cast<int64_t>(gr.row0 + q) * p.score_stride + tok] = sc;
          atomicAdd(&hist[score_key(sc) >> 21], 1u);
        }
      }
      flush();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

std::once_flag g_attr_once[64];
int g_attr_status[64];

inline int group_cap(int num_rows, int num_req) {
  return (num_rows + (kGroupRows - 1) * num_req) / kGroupRows + 1;
}

}  // namespace pf
}  // namespace dsa

using namespace dsa;

namespace {

struct PrefillLayout {
  size_t hist, scores, groups, tile_off, req_gbase, row_req, total;
};

PrefillLayout prefill_layout(int32_t num_rows, int32_t num_requests, int32_t max_pages) {
  const size_t cap = static_cast<size_t>(pf::group_cap(num_rows, num_requests));
  PrefillLayout l;
  l.hist = kWorkspaceHeader;
  l.scores = l.hist + sizeof(uint32_t) * static_cast<size_t>(num_rows) * pf::kBins;
  l.groups = l.scores + sizeof(float) * static_cast<size_t>(num_rows) * static_cast<size_t>(max_pages) *
                            pf::kPage;
  l.tile_off = l.groups + sizeof(pf::Group) * cap;
  l.req_gbase = l.tile_off + sizeof(int) * (cap + 1);
  l.row_req = l.req_gbase + sizeof(int) * (static_cast<size_t>(num_requests) + 1);
  l.total = l.row_req + sizeof(int32_t) * static_cast<size_t>(num_rows);
  return l;
}

}  // namespace

extern "C" size_t dsa_indexer_prefill_workspace_bytes(int32_t num_rows, int32_t num_requests,
                                                      int32_t max_pages) {
  if (num_rows < 0 || num_requests < 0 || max_pages < 0) return 0;
  return prefill_layout(num_rows, num_requests, max_pages).total;
}

extern "C" int dsa_indexer_prefill_run(const void* q_index_fp8, const void* k_index_cache_fp8,
                                       int64_t num_pages, const float* weights,
                                       const int32_t* seq_lens, const int32_t* block_table,
                                       const int32_t* cu_seqlens_q, int32_t num_rows,
                                       int32_t num_requests, int32_t max_pages,
                                       int32_t* topk_indices, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (num_rows < 0 || num_rows > pf::kMaxRows) return DSA_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return DSA_OK;
  if (num_requests < 1 || num_requests > num_rows) return DSA_ERR_INVALID_ARGUMENT;
  if (!q_index_fp8 || !k_index_cache_fp8 || !weights || !seq_lens || !block_table ||
      !cu_seqlens_q || !topk_indices || !workspace)
    return DSA_ERR_INVALID_ARGUMENT;
  if (max_pages < 1 || max_pages > (1 << 20)) return DSA_ERR_INVALID_ARGUMENT;
  if (num_pages < 1 || num_pages > (int64_t(1) << 31) / pf::kPageRows - 1) return DSA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_index_fp8) || !aligned16(k_index_cache_fp8) || !aligned16(workspace) ||
      !aligned16(weights))
    return DSA_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(seq_lens) | reinterpret_cast<uintptr_t>(block_table) |
       reinterpret_cast<uintptr_t>(cu_seqlens_q) | reinterpret_cast<uintptr_t>(topk_indices)) & 3u)
    return DSA_ERR_MISALIGNED;
  const PrefillLayout lay = prefill_layout(num_rows, num_requests, max_pages);
  if (workspace_bytes < lay.total) return DSA_ERR_WORKSPACE_TOO_SMALL;

  DeviceInfo info;
  int st = current_device_info(&info);
  if (st != DSA_OK) return st;
  if (static_cast<size_t>(pf::kSmemBytes) > info.max_smem_optin) return DSA_ERR_UNSUPPORTED_DEVICE;
  std::call_once(pf::g_attr_once[info.device], [&]() {
    pf::g_attr_status[info.device] =
        cudaFuncSetAttribute(pf::prefill_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             pf::kSmemBytes) == cudaSuccess
            ? DSA_OK
            : DSA_ERR_CUDA;
  });
  if (pf::g_attr_status[info.device] != DSA_OK) return pf::g_attr_status[info.device];

  CUtensorMap kmap, qmap;
  st = encode_tmap_2d(&kmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_index_cache_fp8, 128,
                      static_cast<uint64_t>(num_pages) * pf::kPageRows, 128, 128, 64);
  if (st != DSA_OK) return st;
  // q rows of a group: 4 query rows x 64 heads = 256 rows of 128 bytes.
  st = encode_tmap_2d(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, q_index_fp8, 128,
                      static_cast<uint64_t>(num_rows) * pf::kHeads, 128, 128, pf::kN);
  if (st != DSA_OK) return st;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + lay.hist, 0, lay.scores - lay.hist, s) != cudaSuccess) return DSA_ERR_CUDA;

  const int cap = pf::group_cap(num_rows, num_requests);
  pf::PlanParams pp;
  pp.cu_rows = cu_seqlens_q;
  pp.seq_lens = seq_lens;
  pp.groups = reinterpret_cast<pf::Group*>(ws + lay.groups);
  pp.tile_off = reinterpret_cast<int*>(ws + lay.tile_off);
  pp.req_gbase = reinterpret_cast<int*>(ws + lay.req_gbase);
  pp.row_req = reinterpret_cast<int32_t*>(ws + lay.row_req);
  pp.status = reinterpret_cast<unsigned int*>(ws);
  pp.num_req = num_requests;
  pp.num_rows = num_rows;
  pp.group_cap = cap;
  pp.max_len = max_pages * pf::kPage;
  pf::prefill_plan_kernel<<<1, pf::kPlanThreads, 0, s>>>(pp);

  pf::ScoreParams sp;
  sp.k_cache = static_cast<const uint8_t*>(k_index_cache_fp8);
  sp.weights = weights;
  sp.seq_lens = seq_lens;
  sp.block_table = block_table;
  sp.groups = pp.groups;
  sp.tile_off = pp.tile_off;
  sp.scores = reinterpret_cast<float*>(ws + lay.scores);
  sp.hist = reinterpret_cast<unsigned int*>(ws + lay.hist);
  sp.status = pp.status;
  sp.num_pages = num_pages;
  sp.num_rows = num_rows;
  sp.group_cap = cap;
  sp.max_pages = max_pages;
  sp.score_stride = max_pages * pf::kPage;
  if (launch_programmatic(pf::prefill_score_kernel, dim3(info.num_sms), dim3(pf::kThreads),
                          pf::kSmemBytes, s, kmap, qmap, sp) != cudaSuccess)
    return DSA_ERR_CUDA;
  return launch_topk_select(sp.scores, sp.hist, seq_lens, block_table, pp.row_req, topk_indices,
                            num_rows, sp.score_stride, max_pages, sp.status, nullptr, kWaitLimitNs, info, s);
}
