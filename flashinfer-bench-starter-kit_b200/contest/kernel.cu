// kernel.cu -- torch binding of the B200 DSA kernels for the contest harness.
//
// The harness builds a CUDA solution from its packed sources and calls the
// entry point named in config.toml destination-passing style, with the
// definition's inputs then outputs (README.md:227-231, 259-279 of the
// starter kit).  These two functions keep the reference operators'
// signatures (dsa_indexer/solution/triton/kernel.py:364 and
// dsa_attention/solution/triton/kernel.py:241), launch on the current torch
// stream and keep one workspace per device and stream across calls.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <tuple>

#include "dsa_b200.h"

namespace {

// Streams whose workspace is kept per (device, operator); a harness that
// makes a fresh stream per run would otherwise keep every old buffer.
constexpr int kMaxStreamsPerOp = 8;

struct Entry {
  torch::Tensor buf;
  uint64_t last_use = 0;
};

std::mutex g_mu;
std::map<std::tuple<int, int, cudaStream_t>, Entry> g_ws;  // (device, op, stream)
uint64_t g_calls = 0;

// Calls on different streams may run concurrently, so each stream has its
// own buffer.  Beyond kMaxStreamsPerOp streams of a (device, operator) the
// least recently used buffer is dropped: the caching allocator hands its
// memory out again only to later work on the stream it was allocated on
// (the one it served), which is ordered after every kernel that used it.
torch::Tensor workspace(const torch::Device& dev, int op, size_t bytes, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_mu);
  const int device = static_cast<int>(dev.index());
  auto key = std::make_tuple(device, op, stream);
  auto it = g_ws.find(key);
  if (it == g_ws.end()) {
    int n = 0;
    auto lru = g_ws.end();
    for (auto e = g_ws.begin(); e != g_ws.end(); ++e) {
      if (std::get<0>(e->first) != device || std::get<1>(e->first) != op) continue;
      ++n;
      if (lru == g_ws.end() || e->second.last_use < lru->second.last_use) lru = e;
    }
    if (n >= kMaxStreamsPerOp && lru != g_ws.end()) g_ws.erase(lru);
    it = g_ws.emplace(key, Entry{}).first;
  }
  Entry& e = it->second;
  e.last_use = ++g_calls;
  if (!e.buf.defined() || static_cast<size_t>(e.buf.numel()) < bytes) {
    // Zero-filled once; the kernels clear what must start at zero themselves.
    e.buf = torch::zeros({static_cast<int64_t>(bytes)},
                         torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  }
  return e.buf;
}

void check(int st, const char* what) {
  TORCH_CHECK(st == DSA_OK, what, ": ", dsa_b200_status_string(st));
}

}  // namespace

void dsa_indexer(torch::Tensor q_index_fp8, torch::Tensor k_index_cache_fp8, torch::Tensor weights,
                 torch::Tensor seq_lens, torch::Tensor block_table, torch::Tensor topk_indices) {
  TORCH_CHECK(q_index_fp8.is_cuda() && q_index_fp8.dim() == 3, "q_index_fp8 must be [B, 64, 128] on CUDA");
  TORCH_CHECK(topk_indices.is_contiguous() && topk_indices.scalar_type() == torch::kInt32,
              "topk_indices must be contiguous int32");
  const c10::cuda::CUDAGuard guard(q_index_fp8.device());
  const int32_t batch = static_cast<int32_t>(q_index_fp8.size(0));
  if (batch == 0) return;
  auto q = q_index_fp8.contiguous();
  auto k = k_index_cache_fp8.contiguous();
  auto w = weights.to(torch::kFloat32).contiguous();
  auto sl = seq_lens.to(torch::kInt32).contiguous();
  auto bt = block_table.to(torch::kInt32).contiguous();
  const int32_t max_pages = static_cast<int32_t>(bt.size(1));
  const int64_t num_pages = k.numel() * k.element_size() / DSA_INDEX_PAGE_BYTES;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  const size_t bytes = dsa_indexer_workspace_bytes(batch, max_pages);
  auto ws = workspace(q.device(), 0, bytes, stream);
  check(dsa_indexer_run(q.data_ptr(), k.data_ptr(), num_pages, w.data_ptr<float>(),
                        sl.data_ptr<int32_t>(), bt.data_ptr<int32_t>(), batch, max_pages,
                        topk_indices.data_ptr<int32_t>(), ws.data_ptr(), static_cast<size_t>(ws.numel()),
                        stream),
        "dsa_indexer_run");
}

void dsa_attention(torch::Tensor q_nope, torch::Tensor q_pe, torch::Tensor ckv_cache, torch::Tensor kpe_cache,
                   torch::Tensor sparse_indices, double sm_scale, torch::Tensor output, torch::Tensor lse) {
  TORCH_CHECK(q_nope.is_cuda() && q_nope.dim() == 3, "q_nope must be [T, 16, 512] on CUDA");
  TORCH_CHECK(output.is_contiguous() && lse.is_contiguous(), "output and lse must be contiguous");
  const c10::cuda::CUDAGuard guard(q_nope.device());
  const int32_t tokens = static_cast<int32_t>(q_nope.size(0));
  if (tokens == 0) return;
  auto qn = q_nope.contiguous();
  auto qp = q_pe.contiguous();
  auto ckv = ckv_cache.contiguous();
  auto kpe = kpe_cache.contiguous();
  auto idx = sparse_indices.to(torch::kInt32).contiguous();
  const int64_t num_slots = ckv.numel() / DSA_CKV_DIM;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  const size_t bytes = dsa_attention_workspace_bytes(tokens);
  auto ws = workspace(qn.device(), 1, bytes, stream);
  check(dsa_attention_run(qn.data_ptr(), qp.data_ptr(), ckv.data_ptr(), kpe.data_ptr(), num_slots,
                          idx.data_ptr<int32_t>(), tokens, static_cast<float>(sm_scale),
                          output.data_ptr(), lse.data_ptr<float>(), ws.data_ptr(),
                          static_cast<size_t>(ws.numel()), stream),
        "dsa_attention_run");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("dsa_indexer", &dsa_indexer, "DSA top-k indexer (destination-passing)");
  m.def("dsa_attention", &dsa_attention, "DSA sparse MLA attention (destination-passing)");
}
