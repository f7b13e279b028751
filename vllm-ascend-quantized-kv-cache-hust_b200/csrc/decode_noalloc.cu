// qkv_kivi_paged_decode_noalloc: the fused KIVI decode for callers that cannot
// allocate device memory.
//
// Some callers cannot hand this library a workspace: an engine that has given
// all free device memory to its own KV-cache pool up front (vLLM sizes its
// cache to fill the GPU), a host in another language calling through the C ABI
// with no tensor allocator of its own, or a serving loop that must not call
// cudaMalloc because that call can synchronise the whole device. For them this
// entry point keeps the split-KV partial results in a file-scope device array
// instead of a caller workspace, and itself calls no cudaMalloc, cudaFree or
// other allocating routine.
//
// The array is sized kNoAllocScratchBytes (8 MiB) and exists on every GPU that
// loads the library until the process exits. Its device address is resolved
// once per device, on the first call made with that device current
// (cudaGetSymbolAddress); that first call should therefore come before any
// stream capture. All calls on a device share the one array: calls that
// overlap on the GPU (different streams, or several host threads) race on it
// and must be serialised by the caller. Nothing in it has to start at zero —
// every call writes each partial result before the combine step reads it.
#include <mutex>

#include "decode_common.cuh"

namespace qkv {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;

// split-KV partials of qkv_kivi_paged_decode_noalloc (see above)
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (resolved once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(QKV_ERR_UNSUPPORTED, "qkv_kivi_paged_decode_noalloc: device index beyond 63");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return QKV_OK;
}

}  // namespace
}  // namespace qkv

extern "C" {

int qkv_kivi_paged_decode_noalloc(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* out, int64_t out_stride,
    qkv_stream_t stream) {
  using namespace qkv;
  if (batch <= 0)
    return qkv_kivi_paged_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn,
                                 res_key, res_value, res_rows, res_capacity, block_table, bt_stride,
                                 seq_lens, res_state, batch, num_heads, num_kv_heads, head_size,
                                 group_size, block_size, num_blocks, max_seq_len, scale, nullptr, 0,
                                 out, out_stride, stream);
  const size_t need = qkv_kivi_paged_decode_workspace(batch, num_heads, num_kv_heads, head_size,
                                                      group_size, block_size, max_seq_len);
  if (need > kNoAllocScratchBytes)
    return set_error(QKV_ERR_WORKSPACE,
                     "qkv_kivi_paged_decode_noalloc: this batch needs " + std::to_string(need) +
                         " bytes of split-KV scratch, more than the library's static " +
                         std::to_string(kNoAllocScratchBytes) +
                         " bytes; call qkv_kivi_paged_decode with a caller workspace");
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = scratch_address(&scratch);
    if (rc != QKV_OK) return rc;
  }
  return qkv_kivi_paged_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn,
                               res_key, res_value, res_rows, res_capacity, block_table, bt_stride,
                               seq_lens, res_state, batch, num_heads, num_kv_heads, head_size,
                               group_size, block_size, num_blocks, max_seq_len, scale, scratch,
                               need > 0 ? kNoAllocScratchBytes : 0, out, out_stride, stream);
}

}  // extern "C"
