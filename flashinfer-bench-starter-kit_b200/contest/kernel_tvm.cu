// kernel_tvm.cu -- TVM-FFI binding of the B200 DSA kernels for the contest harness.
//
// TVM-FFI is the harness's default binding for CUDA solutions (README.md:259-279
// of the starter kit; its template, solution/cuda/binding.py, is an empty
// stub).  The two exported functions take the definitions' inputs then outputs
// in destination-passing style, with the reference operators' argument lists
// (dsa_indexer/solution/triton/kernel.py:364 and
// dsa_attention/solution/triton/kernel.py:241).  They launch on the stream the
// caller's framework has current for the tensors' device (TVM-FFI records
// torch's current stream for the call and TVMFFIEnvGetStream returns it), and
// keep one zero-filled workspace per (device, operator, stream), grown with
// cudaMalloc when a larger problem arrives: make the first call of the
// largest size before capturing a CUDA graph.
//
// Errors raise ValueError (bad shapes, dtypes, devices) or RuntimeError (a
// non-zero status from the C ABI, with its text).
#include <cuda_runtime.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <map>
#include <mutex>
#include <tuple>

#include "dsa_b200.h"

namespace {

using tvm::ffi::TensorView;

struct Buffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  uint64_t last_use = 0;  // call counter of the entry's latest use
};

// Streams whose workspace is kept per (device, operator); a harness that
// makes a fresh stream per run would otherwise keep every old buffer.
constexpr int kMaxStreamsPerOp = 8;

std::mutex g_mu;
std::map<std::tuple<int, int, cudaStream_t>, Buffer> g_ws;  // (device, op, stream)
uint64_t g_calls = 0;

// The buffer is passed with its full size on every call: the attention
// kernels place their merge counters at its end.  Calls on different
// streams may run concurrently, so each stream has its own buffer; beyond
// kMaxStreamsPerOp streams of a (device, operator) the least recently used
// buffer is freed (cudaFree waits for the device, so no kernel still reads
// it; skipped while the stream is being captured, where freeing is illegal).
Buffer workspace(int device, int op, size_t bytes, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_mu);
  const auto key = std::make_tuple(device, op, stream);
  auto it = g_ws.find(key);
  if (it == g_ws.end()) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(stream, &cap);
    int n = 0;
    auto lru = g_ws.end();
    for (auto e = g_ws.begin(); e != g_ws.end(); ++e) {
      if (std::get<0>(e->first) != device || std::get<1>(e->first) != op) continue;
      ++n;
      if (lru == g_ws.end() || e->second.last_use < lru->second.last_use) lru = e;
    }
    if (n >= kMaxStreamsPerOp && cap == cudaStreamCaptureStatusNone && lru != g_ws.end()) {
      cudaFree(lru->second.ptr);
      g_ws.erase(lru);
    }
    it = g_ws.emplace(key, Buffer{}).first;
  }
  Buffer& b = it->second;
  b.last_use = ++g_calls;
  if (b.bytes >= bytes) return b;
  // cudaFree waits for the device, so kernels still reading the old buffer
  // finish first; the new one is zero-filled once (the kernels clear what
  // must start at zero on every call themselves).
  if (b.ptr != nullptr) cudaFree(b.ptr);
  b.ptr = nullptr;
  b.bytes = 0;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess || cudaMemset(p, 0, bytes) != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    cudaGetLastError();
    TVM_FFI_THROW(RuntimeError) << "DSA workspace allocation of " << bytes
                                << " bytes failed (first call of a size inside a graph capture?)";
  }
  b.ptr = p;
  b.bytes = bytes;
  return b;
}

// Makes `dev` current for the call and restores the previous device after it.
class DeviceScope {
 public:
  explicit DeviceScope(const DLDevice& dev) {
    TVM_FFI_CHECK(dev.device_type == kDLCUDA, ValueError) << "DSA tensors must be on a CUDA device";
    cudaGetDevice(&prev_);
    if (prev_ != dev.device_id) cudaSetDevice(dev.device_id);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != prev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
};

cudaStream_t current_stream(const DLDevice& dev) {
  return static_cast<cudaStream_t>(TVMFFIEnvGetStream(dev.device_type, dev.device_id));
}

bool has_type(const TensorView& t, uint8_t code, uint8_t bits) {
  const DLDataType d = t.dtype();
  return d.code == code && d.bits == bits && d.lanes == 1;
}

void same_device(const TensorView& a, const TensorView& b, const char* name) {
  TVM_FFI_CHECK(b.device().device_type == a.device().device_type && b.device().device_id == a.device().device_id,
                ValueError)
      << name << " is on another device";
}

void check_status(int st, const char* what) {
  TVM_FFI_CHECK(st == DSA_OK, RuntimeError) << what << ": " << dsa_b200_status_string(st);
}

}  // namespace

void dsa_indexer(TensorView q_index_fp8, TensorView k_index_cache_fp8, TensorView weights, TensorView seq_lens,
                 TensorView block_table, TensorView topk_indices) {
  TVM_FFI_CHECK(q_index_fp8.ndim() == 3 && q_index_fp8.size(1) == DSA_INDEX_HEADS &&
                    q_index_fp8.size(2) == DSA_INDEX_DIM && q_index_fp8.dtype().bits == 8,
                ValueError)
      << "q_index_fp8 must be [B, 64, 128] float8_e4m3fn";
  const int64_t batch = q_index_fp8.size(0);
  TVM_FFI_CHECK(k_index_cache_fp8.dtype().bits == 8 &&
                    k_index_cache_fp8.numel() % DSA_INDEX_PAGE_BYTES == 0,
                ValueError)
      << "k_index_cache_fp8 must be 8448-byte pages of 8-bit elements";
  TVM_FFI_CHECK(has_type(weights, kDLFloat, 32) && weights.numel() == batch * DSA_INDEX_HEADS, ValueError)
      << "weights must be [B, 64] float32";
  TVM_FFI_CHECK(has_type(seq_lens, kDLInt, 32) && seq_lens.numel() == batch, ValueError)
      << "seq_lens must be [B] int32";
  TVM_FFI_CHECK(has_type(block_table, kDLInt, 32) && block_table.ndim() == 2 && block_table.size(0) == batch,
                ValueError)
      << "block_table must be [B, max_pages] int32";
  TVM_FFI_CHECK(has_type(topk_indices, kDLInt, 32) && topk_indices.ndim() == 2 &&
                    topk_indices.size(0) == batch && topk_indices.size(1) == DSA_TOPK,
                ValueError)
      << "topk_indices must be [B, 2048] int32";
  for (const TensorView* t : {&q_index_fp8, &k_index_cache_fp8, &weights, &seq_lens, &block_table, &topk_indices})
    TVM_FFI_CHECK(t->IsContiguous(), ValueError) << "DSA indexer tensors must be contiguous";
  same_device(q_index_fp8, k_index_cache_fp8, "k_index_cache_fp8");
  same_device(q_index_fp8, weights, "weights");
  same_device(q_index_fp8, seq_lens, "seq_lens");
  same_device(q_index_fp8, block_table, "block_table");
  same_device(q_index_fp8, topk_indices, "topk_indices");
  if (batch == 0) return;
  const DLDevice dev = q_index_fp8.device();
  DeviceScope scope(dev);
  const int32_t max_pages = static_cast<int32_t>(block_table.size(1));
  const int64_t num_pages = k_index_cache_fp8.numel() / DSA_INDEX_PAGE_BYTES;
  cudaStream_t stream = current_stream(dev);
  const size_t bytes = dsa_indexer_workspace_bytes(static_cast<int32_t>(batch), max_pages);
  const Buffer ws = workspace(dev.device_id, 0, bytes, stream);
  check_status(dsa_indexer_run(q_index_fp8.data_ptr(), k_index_cache_fp8.data_ptr(), num_pages,
                               static_cast<const float*>(weights.data_ptr()),
                               static_cast<const int32_t*>(seq_lens.data_ptr()),
                               static_cast<const int32_t*>(block_table.data_ptr()), static_cast<int32_t>(batch),
                               max_pages, static_cast<int32_t*>(topk_indices.data_ptr()), ws.ptr, ws.bytes, stream),
               "dsa_indexer_run");
}

void dsa_attention(TensorView q_nope, TensorView q_pe, TensorView ckv_cache, TensorView kpe_cache,
                   TensorView sparse_indices, double sm_scale, TensorView output, TensorView lse) {
  TVM_FFI_CHECK(has_type(q_nope, kDLBfloat, 16) && q_nope.ndim() == 3 && q_nope.size(1) == DSA_ATTN_HEADS &&
                    q_nope.size(2) == DSA_CKV_DIM,
                ValueError)
      << "q_nope must be [T, 16, 512] bfloat16";
  const int64_t tokens = q_nope.size(0);
  TVM_FFI_CHECK(has_type(q_pe, kDLBfloat, 16) && q_pe.numel() == tokens * DSA_ATTN_HEADS * DSA_KPE_DIM, ValueError)
      << "q_pe must be [T, 16, 64] bfloat16";
  TVM_FFI_CHECK(has_type(ckv_cache, kDLBfloat, 16) && ckv_cache.numel() % DSA_CKV_DIM == 0, ValueError)
      << "ckv_cache must be [pages, 64, 512] bfloat16";
  const int64_t num_slots = ckv_cache.numel() / DSA_CKV_DIM;
  TVM_FFI_CHECK(has_type(kpe_cache, kDLBfloat, 16) && kpe_cache.numel() == num_slots * DSA_KPE_DIM, ValueError)
      << "kpe_cache must be [pages, 64, 64] bfloat16 with as many slots as ckv_cache";
  TVM_FFI_CHECK(has_type(sparse_indices, kDLInt, 32) && sparse_indices.numel() == tokens * DSA_TOPK, ValueError)
      << "sparse_indices must be [T, 2048] int32";
  TVM_FFI_CHECK(has_type(output, kDLBfloat, 16) && output.numel() == tokens * DSA_ATTN_HEADS * DSA_CKV_DIM,
                ValueError)
      << "output must be [T, 16, 512] bfloat16";
  TVM_FFI_CHECK(has_type(lse, kDLFloat, 32) && lse.numel() == tokens * DSA_ATTN_HEADS, ValueError)
      << "lse must be [T, 16] float32";
  for (const TensorView* t : {&q_nope, &q_pe, &ckv_cache, &kpe_cache, &sparse_indices, &output, &lse})
    TVM_FFI_CHECK(t->IsContiguous(), ValueError) << "DSA attention tensors must be contiguous";
  same_device(q_nope, q_pe, "q_pe");
  same_device(q_nope, ckv_cache, "ckv_cache");
  same_device(q_nope, kpe_cache, "kpe_cache");
  same_device(q_nope, sparse_indices, "sparse_indices");
  same_device(q_nope, output, "output");
  same_device(q_nope, lse, "lse");
  if (tokens == 0) return;
  const DLDevice dev = q_nope.device();
  DeviceScope scope(dev);
  cudaStream_t stream = current_stream(dev);
  const size_t bytes = dsa_attention_workspace_bytes(static_cast<int32_t>(tokens));
  const Buffer ws = workspace(dev.device_id, 1, bytes, stream);
  check_status(dsa_attention_run(q_nope.data_ptr(), q_pe.data_ptr(), ckv_cache.data_ptr(), kpe_cache.data_ptr(),
                                 num_slots, static_cast<const int32_t*>(sparse_indices.data_ptr()),
                                 static_cast<int32_t>(tokens), static_cast<float>(sm_scale), output.data_ptr(),
                                 static_cast<float*>(lse.data_ptr()), ws.ptr, ws.bytes, stream),
               "dsa_attention_run");
}

TVM_FFI_DLL_EXPORT_TYPED_FUNC(dsa_indexer, dsa_indexer);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dsa_attention, dsa_attention);
