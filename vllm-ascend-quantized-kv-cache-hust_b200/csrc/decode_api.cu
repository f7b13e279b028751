// C ABI of the paged decode kernels: argument validation, split planning and
// dispatch between the tensor-core kernels (production geometries) and the
// geometry-general CUDA-core kernels.
#include <cmath>

#include "decode_common.cuh"

namespace qkv {

int launch_decode_generic(const DecodeParams& p, int mode, cudaStream_t stream);
SplitPlan plan_for(const DecodeParams& p, bool kivi, int max_seq_len);
SplitPlan plan_generic(const DecodeParams& p, bool kivi, int max_seq_len);
bool kivi_tma_geometry(const DecodeParams& p);
bool kivi_tma_supported(const DecodeParams& p);
SplitPlan plan_kivi_tma(int batch, int kvh, int group, int max_seq_len, int sms);
int launch_kivi_tma(const DecodeParams& p, cudaStream_t stream, bool combine = true, int* splits_used = nullptr);
bool int8_tma_geometry(const DecodeParams& p);
bool int8_tma_supported(const DecodeParams& p);
SplitPlan plan_int8_tma(int batch, int kvh, int max_seq_len, int sms);
int launch_int8_tma(const DecodeParams& p, cudaStream_t stream);
bool prefill_tc_supported(int head_size, int gqa, const void* q, const void* k, const void* v,
                          const void* out);
int launch_prefill_tc(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                      const int32_t* cu_q, const int32_t* cu_k, int num_reqs, int total_q, int total_k,
                      int num_heads, int kvh, int causal, float scale, __nv_bfloat16* out,
                      cudaStream_t stream);
int launch_kivi_gather(const DecodeParams& p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                       __nv_bfloat16* dense_v, cudaStream_t stream);
int launch_int8_gather(const DecodeParams& p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                       __nv_bfloat16* dense_v, cudaStream_t stream);
bool fp8_tma_geometry(const DecodeParams& p);
bool fp8_tma_supported(const DecodeParams& p);
SplitPlan plan_fp8_tma(int batch, int kvh, int max_seq_len, int sms);
int launch_fp8_tma(const DecodeParams& p, cudaStream_t stream);

namespace {

int check_decode_args(const char* fn, int batch, int num_heads, int kvh,
                      int head_size, int block_size, int64_t num_blocks,
                      int max_seq_len) {
  const std::string f(fn);
  QKV_CHECK_ARG(batch >= 0 && kvh > 0 && num_heads > 0 && num_blocks > 0,
                f + ": bad sizes");
  QKV_CHECK_ARG(num_heads % kvh == 0,
                f + ": num_heads must be a multiple of num_kv_heads");
  QKV_CHECK_ARG(head_size > 0 && head_size % 8 == 0 && head_size <= 256,
                f + ": head_size must be a multiple of 8 and <= 256");
  QKV_CHECK_ARG(block_size > 0 && block_size % 8 == 0,
                f + ": block_size must be a multiple of 8");
  QKV_CHECK_ARG(max_seq_len >= 0, f + ": max_seq_len must be >= 0");
  return QKV_OK;
}

}  // namespace

// Split plan of the generic CUDA-core kernels (one window split for KIVI).
SplitPlan plan_generic(const DecodeParams& p, bool kivi, int max_seq_len) {
  return plan_splits(p.batch, p.kvh, p.blk, max_seq_len, kivi, sm_count(), 4, 256);
}

// Split plan of the kernel a call with these arguments runs.
SplitPlan plan_for(const DecodeParams& p, bool kivi, int max_seq_len) {
  if (kivi) {
    if (kivi_tma_supported(p)) return plan_kivi_tma(p.batch, p.kvh, p.group, max_seq_len, sm_count());
    return plan_generic(p, true, max_seq_len);
  }
  if (int8_tma_supported(p)) return plan_int8_tma(p.batch, p.kvh, max_seq_len, sm_count());
  return plan_generic(p, false, max_seq_len);
}

}  // namespace qkv

extern "C" {

size_t qkv_int8_paged_decode_workspace(int batch, int num_heads,
                                       int num_kv_heads, int head_size,
                                       int block_size, int max_seq_len) {
  using namespace qkv;
  if (batch <= 0 || num_kv_heads <= 0 || block_size <= 0) return 0;
  DecodeParams p{};
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.blk = block_size;
  p.group = head_size;
  // the larger of the two kernels' plans: the call may take either path
  size_t a = 0;
  if (int8_tma_geometry(p))
    a = workspace_bytes(batch, num_heads, head_size,
                        plan_int8_tma(batch, num_kv_heads, max_seq_len, sm_count()).total);
  const size_t b = workspace_bytes(batch, num_heads, head_size,
                                   plan_generic(p, false, max_seq_len).total);
  return a > b ? a : b;
}

size_t qkv_kivi_paged_decode_workspace(int batch, int num_heads,
                                       int num_kv_heads, int head_size,
                                       int group_size, int block_size,
                                       int max_seq_len) {
  using namespace qkv;
  if (batch <= 0 || num_kv_heads <= 0 || block_size <= 0) return 0;
  DecodeParams p{};
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.blk = block_size;
  p.group = group_size;
  // the larger of the two kernels' plans: the call may take either path
  size_t a = 0;
  if (kivi_tma_geometry(p))
    a = workspace_bytes(batch, num_heads, head_size,
                        plan_kivi_tma(batch, num_kv_heads, group_size, max_seq_len, sm_count()).total);
  const size_t b = workspace_bytes(batch, num_heads, head_size,
                                   plan_generic(p, true, max_seq_len).total);
  return a > b ? a : b;
}

int qkv_int8_paged_decode(const void* query, int64_t q_stride,
                          const int8_t* key_cache, const int8_t* value_cache,
                          const void* k_aq_scale, const void* v_aq_scale,
                          const int32_t* block_table, int64_t bt_stride,
                          const int32_t* seq_lens, int batch, int num_heads,
                          int num_kv_heads, int head_size, int block_size,
                          int64_t num_blocks, int max_seq_len, float scale,
                          void* workspace, size_t workspace_bytes_, void* out,
                          int64_t out_stride, qkv_stream_t stream) {
  using namespace qkv;
  int rc = check_decode_args("qkv_int8_paged_decode", batch, num_heads,
                             num_kv_heads, head_size, block_size, num_blocks,
                             max_seq_len);
  if (rc != QKV_OK) return rc;
  if (batch == 0) return QKV_OK;
  QKV_CHECK_ARG(query && key_cache && value_cache && k_aq_scale && v_aq_scale &&
                    block_table && seq_lens && out,
                "qkv_int8_paged_decode: null pointer");
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.q_stride = q_stride;
  p.kc = key_cache;
  p.vc = value_cache;
  p.k_aq = static_cast<const __nv_bfloat16*>(k_aq_scale);
  p.v_aq = static_cast<const __nv_bfloat16*>(v_aq_scale);
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.group = head_size;
  p.blk = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.err = device_error_ptr();
  const SplitPlan plan = plan_for(p, false, max_seq_len);
  p.num_hist_splits = plan.hist_splits;
  p.split_tokens = plan.split_tokens;
  p.splits_total = plan.total;
  const size_t need = workspace_bytes(batch, num_heads, head_size, plan.total);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes_ < need)
      return set_error(QKV_ERR_WORKSPACE,
                       "qkv_int8_paged_decode: workspace needs " +
                           std::to_string(need) + " bytes");
    p.ws_acc = static_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + static_cast<size_t>(batch) * num_heads * plan.total *
                             head_size;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (int8_tma_supported(p)) return launch_int8_tma(p, s);
  return launch_decode_generic(p, kInt8Pages, s);  // planned for it by plan_for
}

namespace qkv {
namespace {

// The KIVI decode; with combine == false and several splits on the
// page-pipelined kernel, the split partials stay in the workspace and
// *splits_used reports their count (1: `out` was written).
int kivi_decode(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* workspace, size_t workspace_bytes_,
    void* out, int64_t out_stride, qkv_stream_t stream, bool combine, int* splits_used,
    bool after_ring_write = false) {
  if (splits_used != nullptr) *splits_used = 1;
  int rc = check_decode_args("qkv_kivi_paged_decode", batch, num_heads,
                             num_kv_heads, head_size, block_size, num_blocks,
                             max_seq_len);
  if (rc != QKV_OK) return rc;
  QKV_CHECK_ARG(group_size > 0 && group_size % 8 == 0 &&
                    head_size % group_size == 0 && block_size % group_size == 0,
                "qkv_kivi_paged_decode: group_size must be a multiple of 8 "
                "dividing head_size and block_size");
  QKV_CHECK_ARG(res_state == nullptr || (res_rows > 0 && res_capacity > 0),
                "qkv_kivi_paged_decode: residual window needs rows and capacity");
  if (batch == 0) return QKV_OK;
  QKV_CHECK_ARG(query && k_quant && k_scale && k_mn && v_quant && v_scale &&
                    v_mn && block_table && seq_lens && out,
                "qkv_kivi_paged_decode: null pointer");
  QKV_CHECK_ARG(res_state == nullptr || (res_key && res_value),
                "qkv_kivi_paged_decode: residual buffers are NULL");
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.q_stride = q_stride;
  p.kq = k_quant;
  p.ks = k_scale;
  p.km = k_mn;
  p.vq = v_quant;
  p.vs = v_scale;
  p.vm = v_mn;
  p.rk = static_cast<const __nv_bfloat16*>(res_key);
  p.rv = static_cast<const __nv_bfloat16*>(res_value);
  p.res_rows = res_rows;
  p.res_cap = res_capacity;
  p.res_state = res_state;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.group = group_size;
  p.blk = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.err = device_error_ptr();
  p.after_ring_write = after_ring_write ? 1 : 0;
  const SplitPlan plan = plan_for(p, true, max_seq_len);
  p.num_hist_splits = plan.hist_splits;
  p.split_tokens = plan.split_tokens;
  p.splits_total = plan.total;
  const bool tma = kivi_tma_supported(p);
  // the page-pipelined kernel has window CTAs only when there is a window:
  // the partials (and their layout in the workspace) shrink to match
  if (tma && res_state == nullptr) p.splits_total = p.num_hist_splits;
  const size_t need = workspace_bytes(batch, num_heads, head_size, p.splits_total);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes_ < need)
      return set_error(QKV_ERR_WORKSPACE,
                       "qkv_kivi_paged_decode: workspace needs " +
                           std::to_string(need) + " bytes");
    p.ws_acc = static_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + static_cast<size_t>(batch) * num_heads * p.splits_total *
                             head_size;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tma) return launch_kivi_tma(p, s, combine, splits_used);
  return launch_decode_generic(p, kKiviPages, s);  // planned for it by plan_for
}

}  // namespace

// (C++ linkage, declared in qkv_common.cuh: not part of the C ABI)
extern "C++" int kivi_paged_decode_after_ring_write(
    const void* query, int64_t q_stride, const int32_t* k_quant, const float* k_scale, const float* k_mn,
    const int32_t* v_quant, const float* v_scale, const float* v_mn, const void* res_key, const void* res_value,
    int res_rows, int res_capacity, const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads, int head_size, int group_size,
    int block_size, int64_t num_blocks, int max_seq_len, float scale, void* workspace, size_t workspace_bytes_,
    void* out, int64_t out_stride, qkv_stream_t stream) {
  return kivi_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key, res_value, res_rows,
                     res_capacity, block_table, bt_stride, seq_lens, res_state, batch, num_heads, num_kv_heads,
                     head_size, group_size, block_size, num_blocks, max_seq_len, scale, workspace, workspace_bytes_,
                     out, out_stride, stream, true, nullptr, true);
}

}  // namespace qkv

int qkv_kivi_paged_decode(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* workspace, size_t workspace_bytes_,
    void* out, int64_t out_stride, qkv_stream_t stream) {
  return qkv::kivi_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key, res_value,
                          res_rows, res_capacity, block_table, bt_stride, seq_lens, res_state, batch, num_heads,
                          num_kv_heads, head_size, group_size, block_size, num_blocks, max_seq_len, scale,
                          workspace, workspace_bytes_, out, out_stride, stream, true, nullptr);
}

int qkv_kivi_paged_decode_partials(
    const void* query, int64_t q_stride, const int32_t* k_quant,
    const float* k_scale, const float* k_mn, const int32_t* v_quant,
    const float* v_scale, const float* v_mn, const void* res_key,
    const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads,
    int head_size, int group_size, int block_size, int64_t num_blocks,
    int max_seq_len, float scale, void* workspace, size_t workspace_bytes_,
    void* out, int64_t out_stride, int* splits_used, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(splits_used != nullptr, "qkv_kivi_paged_decode_partials: null splits_used");
  return kivi_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key, res_value, res_rows,
                     res_capacity, block_table, bt_stride, seq_lens, res_state, batch, num_heads, num_kv_heads,
                     head_size, group_size, block_size, num_blocks, max_seq_len, scale, workspace, workspace_bytes_,
                     out, out_stride, stream, false, splits_used);
}

size_t qkv_dense_prefill_workspace(int total_q, int num_heads,
                                   int num_kv_heads, int head_size,
                                   int max_kv_len) {
  using namespace qkv;
  if (total_q <= 0 || num_kv_heads <= 0) return 0;
  const SplitPlan plan = plan_splits(total_q, num_kv_heads, 128, max_kv_len,
                                     false, sm_count(), 4, 512);
  return workspace_bytes(total_q, num_heads, head_size, plan.total);
}

int qkv_dense_prefill(const void* query, const void* key, const void* value,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                      int num_reqs, int total_q, int total_k, int num_heads,
                      int num_kv_heads, int head_size, int causal,
                      int max_kv_len, float scale, void* workspace,
                      size_t workspace_bytes_, void* out, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(num_reqs >= 0 && total_q >= 0 && total_k >= 0 && num_kv_heads > 0 &&
                    num_heads > 0 && num_heads % num_kv_heads == 0,
                "qkv_dense_prefill: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && head_size % 8 == 0 && head_size <= 256,
                "qkv_dense_prefill: head_size must be a multiple of 8 and <= 256");
  if (total_q == 0 || num_reqs == 0) return QKV_OK;
  QKV_CHECK_ARG(query && key && value && cu_seqlens_q && cu_seqlens_k && out,
                "qkv_dense_prefill: null pointer");
  if (total_k > 0 && prefill_tc_supported(head_size, num_heads / num_kv_heads, query, key, value, out))
    return launch_prefill_tc(static_cast<const __nv_bfloat16*>(query), static_cast<const __nv_bfloat16*>(key),
                             static_cast<const __nv_bfloat16*>(value), cu_seqlens_q, cu_seqlens_k, num_reqs,
                             total_q, total_k, num_heads, num_kv_heads, causal, scale,
                             static_cast<__nv_bfloat16*>(out), reinterpret_cast<cudaStream_t>(stream));
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.q_stride = static_cast<int64_t>(num_heads) * head_size;
  p.dk = static_cast<const __nv_bfloat16*>(key);
  p.dv = static_cast<const __nv_bfloat16*>(value);
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.num_reqs = num_reqs;
  p.causal = causal;
  p.batch = total_q;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.group = head_size;
  p.blk = 128;
  p.num_blocks = 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = static_cast<int64_t>(num_heads) * head_size;
  p.err = device_error_ptr();
  const SplitPlan plan = plan_splits(total_q, num_kv_heads, 128, max_kv_len,
                                     false, sm_count(), 4, 512);
  p.num_hist_splits = plan.hist_splits;
  p.split_tokens = plan.split_tokens;
  p.splits_total = plan.total;
  const size_t need = workspace_bytes(total_q, num_heads, head_size, plan.total);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes_ < need)
      return set_error(QKV_ERR_WORKSPACE, "qkv_dense_prefill: workspace needs " +
                                              std::to_string(need) + " bytes");
    p.ws_acc = static_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + static_cast<size_t>(total_q) * num_heads * plan.total *
                             head_size;
  }
  return launch_decode_generic(p, kDense, reinterpret_cast<cudaStream_t>(stream));
}

int qkv_kivi_dequant_gather(
    const int32_t* k_quant, const float* k_scale, const float* k_mn,
    const int32_t* v_quant, const float* v_scale, const float* v_mn,
    const void* res_key, const void* res_value, int res_rows, int res_capacity,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* cu_seqlens_k, const int32_t* res_state, int batch,
    int num_kv_heads, int head_size, int group_size, int block_size,
    int64_t num_blocks, int total_k, void* out_key, void* out_value,
    qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(batch >= 0 && total_k >= 0 && num_kv_heads > 0 && num_blocks > 0,
                "qkv_kivi_dequant_gather: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && head_size % 8 == 0 && group_size > 0 && group_size % 8 == 0 &&
                    head_size % group_size == 0 && block_size > 0 && block_size % group_size == 0,
                "qkv_kivi_dequant_gather: bad geometry");
  QKV_CHECK_ARG(res_state == nullptr || (res_key && res_value && res_rows > 0 && res_capacity > 0),
                "qkv_kivi_dequant_gather: residual window needs buffers, rows and capacity");
  if (batch == 0 || total_k == 0) return QKV_OK;
  QKV_CHECK_ARG(k_quant && k_scale && k_mn && v_quant && v_scale && v_mn && block_table && seq_lens &&
                    cu_seqlens_k && out_key && out_value,
                "qkv_kivi_dequant_gather: null pointer");
  const auto al16 = [](const void* x) { return x == nullptr || (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  QKV_CHECK_ARG(al16(out_key) && al16(out_value) && al16(res_key) && al16(res_value),
                "qkv_kivi_dequant_gather: outputs and windows must be 16-byte aligned");
  DecodeParams p{};
  p.kq = k_quant;
  p.ks = k_scale;
  p.km = k_mn;
  p.vq = v_quant;
  p.vs = v_scale;
  p.vm = v_mn;
  p.rk = static_cast<const __nv_bfloat16*>(res_key);
  p.rv = static_cast<const __nv_bfloat16*>(res_value);
  p.res_rows = res_rows;
  p.res_cap = res_capacity;
  p.res_state = res_state;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.num_reqs = batch;
  p.batch = batch;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.group = group_size;
  p.blk = block_size;
  p.num_blocks = num_blocks;
  p.err = device_error_ptr();
  return launch_kivi_gather(p, cu_seqlens_k, total_k, static_cast<__nv_bfloat16*>(out_key),
                            static_cast<__nv_bfloat16*>(out_value), reinterpret_cast<cudaStream_t>(stream));
}

int qkv_int8_dequant_gather(
    const int8_t* key_cache, const int8_t* value_cache, const void* k_aq_scale, const void* v_aq_scale,
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* cu_seqlens_k,
    int batch, int num_kv_heads, int head_size, int block_size, int64_t num_blocks, int total_k,
    void* out_key, void* out_value, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(batch >= 0 && total_k >= 0 && num_kv_heads > 0 && num_blocks > 0 && block_size > 0,
                "qkv_int8_dequant_gather: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && head_size % 16 == 0, "qkv_int8_dequant_gather: head_size must be a multiple of 16");
  if (batch == 0 || total_k == 0) return QKV_OK;
  QKV_CHECK_ARG(key_cache && value_cache && k_aq_scale && v_aq_scale && block_table && seq_lens && cu_seqlens_k &&
                    out_key && out_value,
                "qkv_int8_dequant_gather: null pointer");
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  QKV_CHECK_ARG(al16(key_cache) && al16(value_cache) && al16(k_aq_scale) && al16(v_aq_scale) && al16(out_key) &&
                    al16(out_value),
                "qkv_int8_dequant_gather: caches, scales and outputs must be 16-byte aligned");
  DecodeParams p{};
  p.kc = key_cache;
  p.vc = value_cache;
  p.k_aq = static_cast<const __nv_bfloat16*>(k_aq_scale);
  p.v_aq = static_cast<const __nv_bfloat16*>(v_aq_scale);
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.num_reqs = batch;
  p.batch = batch;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.blk = block_size;
  p.num_blocks = num_blocks;
  p.err = device_error_ptr();
  return launch_int8_gather(p, cu_seqlens_k, total_k, static_cast<__nv_bfloat16*>(out_key),
                            static_cast<__nv_bfloat16*>(out_value), reinterpret_cast<cudaStream_t>(stream));
}

size_t qkv_fp8_paged_decode_workspace(int batch, int num_heads, int num_kv_heads, int head_size, int block_size,
                                      int max_seq_len) {
  using namespace qkv;
  if (batch <= 0 || num_kv_heads <= 0 || block_size <= 0) return 0;
  DecodeParams p{};
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.blk = block_size;
  p.group = head_size;
  size_t a = 0;
  if (fp8_tma_geometry(p))
    a = workspace_bytes(batch, num_heads, head_size, plan_fp8_tma(batch, num_kv_heads, max_seq_len, sm_count()).total);
  const size_t b = workspace_bytes(batch, num_heads, head_size, plan_generic(p, false, max_seq_len).total);
  return a > b ? a : b;
}

int qkv_fp8_paged_decode(const void* query, int64_t q_stride, const uint8_t* k_data, const float* k_scale,
                         const uint8_t* v_data, const float* v_scale, const int32_t* block_table, int64_t bt_stride,
                         const int32_t* seq_lens, int batch, int num_heads, int num_kv_heads, int head_size,
                         int block_size, int64_t num_blocks, int max_seq_len, float scale, void* workspace,
                         size_t workspace_bytes_, void* out, int64_t out_stride, qkv_stream_t stream) {
  using namespace qkv;
  int rc = check_decode_args("qkv_fp8_paged_decode", batch, num_heads, num_kv_heads, head_size, block_size,
                             num_blocks, max_seq_len);
  if (rc != QKV_OK) return rc;
  if (batch == 0) return QKV_OK;
  QKV_CHECK_ARG(query && k_data && k_scale && v_data && v_scale && block_table && seq_lens && out,
                "qkv_fp8_paged_decode: null pointer");
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(query);
  p.q_stride = q_stride;
  p.kc = reinterpret_cast<const int8_t*>(k_data);
  p.vc = reinterpret_cast<const int8_t*>(v_data);
  p.ks = k_scale;
  p.vs = v_scale;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.batch = batch;
  p.num_heads = num_heads;
  p.kvh = num_kv_heads;
  p.head_size = head_size;
  p.gqa = num_heads / num_kv_heads;
  p.group = head_size;
  p.blk = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.err = device_error_ptr();
  const bool tma = fp8_tma_supported(p);
  const SplitPlan plan =
      tma ? plan_fp8_tma(batch, num_kv_heads, max_seq_len, sm_count()) : plan_generic(p, false, max_seq_len);
  p.num_hist_splits = plan.hist_splits;
  p.split_tokens = plan.split_tokens;
  p.splits_total = plan.total;
  const size_t need = workspace_bytes(batch, num_heads, head_size, plan.total);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes_ < need)
      return set_error(QKV_ERR_WORKSPACE, "qkv_fp8_paged_decode: workspace needs " + std::to_string(need) +
                                              " bytes");
    p.ws_acc = static_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + static_cast<size_t>(batch) * num_heads * plan.total * head_size;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tma) return launch_fp8_tma(p, s);
  return launch_decode_generic(p, kFp8Pages, s);
}

}  // extern "C"
