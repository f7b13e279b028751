// Device side of a residual-window plan (the planner is window_plan.cpp):
// gather the tokens a plan names (ring lanes or new tokens) into dense
// buffers, and scatter dense tokens into ring lanes. Replaces the per-step
// index_select / index_copy_ sequence of the reference's window writes
// (methods/kivi_int4/attention_backend.py:411-462) with one launch each, both
// sides together. A token row is row_bytes (a multiple of 16) whatever the
// residual dtype; one thread moves 16 bytes of one row.
#include "decode_common.cuh"

namespace qkv {

namespace {

__global__ void window_gather_kernel(const uint4* ring_k, const uint4* ring_v, int64_t ring_lanes,
                                     const uint4* new_k, const uint4* new_v, int64_t n_new,
                                     const int64_t* k_src, int64_t nk, const int64_t* v_src, int64_t nv,
                                     int64_t row_words, uint4* out_k, uint4* out_v, int* err) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = (nk + nv) * row_words;
  if (idx >= total) return;
  const int64_t item = idx / row_words, w = idx - item * row_words;
  const bool key = item < nk;
  const int64_t i = key ? item : item - nk;
  const int64_t src = key ? k_src[i] : v_src[i];
  const uint4* ring = key ? ring_k : ring_v;
  const uint4* fresh = key ? new_k : new_v;
  uint4 val = make_uint4(0, 0, 0, 0);
  if (src >= 0 && src < ring_lanes) {
    val = ring[src * row_words + w];
  } else if (src < 0 && -1 - src < n_new) {
    val = fresh[(-1 - src) * row_words + w];
  } else if (w == 0) {
    record_error(err, kErrWindowSource);
  }
  (key ? out_k : out_v)[i * row_words + w] = val;
}

// Rows written into the ring lanes: item i of the dense k_data / v_data, or,
// with k_src / v_src, the new token -1 - src[i] of new_k / new_v.
__global__ void window_scatter_kernel(uint4* ring_k, uint4* ring_v, int64_t ring_lanes, const int64_t* k_lanes,
                                      int64_t nk, const uint4* k_data, const int64_t* v_lanes, int64_t nv,
                                      const uint4* v_data, int64_t row_words, int* err, const int64_t* k_src,
                                      const int64_t* v_src, int64_t n_new) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = (nk + nv) * row_words;
  if (idx >= total) return;
  const int64_t item = idx / row_words, w = idx - item * row_words;
  const bool key = item < nk;
  const int64_t i = key ? item : item - nk;
  const int64_t lane = key ? k_lanes[i] : v_lanes[i];
  if (lane < 0 || lane >= ring_lanes) {
    if (w == 0) record_error(err, kErrWindowSource);
    return;
  }
  const int64_t* src = key ? k_src : v_src;
  int64_t row = i;
  if (src != nullptr) {
    row = -1 - src[i];
    if (row < 0 || row >= n_new) {
      if (w == 0) record_error(err, kErrWindowSource);
      return;
    }
  }
  (key ? ring_k : ring_v)[lane * row_words + w] = (key ? k_data : v_data)[row * row_words + w];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned grid_for(int64_t threads, int block) { return static_cast<unsigned>((threads + block - 1) / block); }

}  // namespace

// Ring writes whose rows are all new tokens, read in place (k_src / v_src:
// -1 - token), one launch for both sides.
int scatter_new_tokens(void* ring_key, void* ring_value, int64_t ring_lanes, const int64_t* k_lanes,
                       const int64_t* k_src, int64_t nk, const int64_t* v_lanes, const int64_t* v_src, int64_t nv,
                       const void* new_key, const void* new_value, int64_t n_new, int64_t row_bytes,
                       cudaStream_t stream) {
  if (nk + nv == 0) return QKV_OK;
  QKV_CHECK_ARG(row_bytes > 0 && row_bytes % 16 == 0 && new_key && new_value && aligned16(new_key) &&
                    aligned16(new_value) && aligned16(ring_key) && aligned16(ring_value),
                "scatter_new_tokens: bad rows");
  const int64_t row_words = row_bytes / 16;
  const int64_t threads = (nk + nv) * row_words;
  window_scatter_kernel<<<grid_for(threads, 256), 256, 0, stream>>>(
      static_cast<uint4*>(ring_key), static_cast<uint4*>(ring_value), ring_lanes, k_lanes, nk,
      static_cast<const uint4*>(new_key), v_lanes, nv, static_cast<const uint4*>(new_value), row_words,
      device_error_ptr(), k_src, v_src, n_new);
  QKV_CHECK_LAUNCH("window_scatter_kernel");
  return QKV_OK;
}

}  // namespace qkv

extern "C" {

int qkv_kivi_window_gather(const void* ring_key, const void* ring_value, int64_t ring_lanes, const void* new_key,
                           const void* new_value, int64_t n_new, const int64_t* k_src, int64_t nk,
                           const int64_t* v_src, int64_t nv, int64_t row_bytes, void* out_k, void* out_v,
                           qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(nk >= 0 && nv >= 0 && ring_lanes >= 0 && n_new >= 0 && row_bytes > 0 && row_bytes % 16 == 0,
                "qkv_kivi_window_gather: bad sizes (row_bytes must be a positive multiple of 16)");
  if (nk + nv == 0) return QKV_OK;
  QKV_CHECK_ARG((nk == 0 || (k_src && out_k)) && (nv == 0 || (v_src && out_v)) && ring_key && ring_value,
                "qkv_kivi_window_gather: null pointer");
  QKV_CHECK_ARG(aligned16(ring_key) && aligned16(ring_value) && aligned16(out_k) && aligned16(out_v) &&
                    (new_key == nullptr || aligned16(new_key)) && (new_value == nullptr || aligned16(new_value)),
                "qkv_kivi_window_gather: buffers must be 16-byte aligned");
  const int64_t row_words = row_bytes / 16;
  const int64_t threads = (nk + nv) * row_words;
  QKV_CHECK_ARG(threads / 256 < 0x7FFFFFFFll, "qkv_kivi_window_gather: too many tokens");
  window_gather_kernel<<<grid_for(threads, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(ring_key), static_cast<const uint4*>(ring_value), ring_lanes,
      static_cast<const uint4*>(new_key), static_cast<const uint4*>(new_value), new_key ? n_new : 0, k_src, nk,
      v_src, nv, row_words, static_cast<uint4*>(out_k), static_cast<uint4*>(out_v), device_error_ptr());
  QKV_CHECK_LAUNCH("window_gather_kernel");
  return QKV_OK;
}

int qkv_kivi_window_scatter(void* ring_key, void* ring_value, int64_t ring_lanes, const int64_t* k_lanes, int64_t nk,
                            const void* k_data, const int64_t* v_lanes, int64_t nv, const void* v_data,
                            int64_t row_bytes, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(nk >= 0 && nv >= 0 && ring_lanes >= 0 && row_bytes > 0 && row_bytes % 16 == 0,
                "qkv_kivi_window_scatter: bad sizes (row_bytes must be a positive multiple of 16)");
  if (nk + nv == 0) return QKV_OK;
  QKV_CHECK_ARG((nk == 0 || (k_lanes && k_data)) && (nv == 0 || (v_lanes && v_data)) && ring_key && ring_value,
                "qkv_kivi_window_scatter: null pointer");
  QKV_CHECK_ARG(aligned16(ring_key) && aligned16(ring_value) && aligned16(k_data) && aligned16(v_data),
                "qkv_kivi_window_scatter: buffers must be 16-byte aligned");
  const int64_t row_words = row_bytes / 16;
  const int64_t threads = (nk + nv) * row_words;
  QKV_CHECK_ARG(threads / 256 < 0x7FFFFFFFll, "qkv_kivi_window_scatter: too many tokens");
  window_scatter_kernel<<<grid_for(threads, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(ring_key), static_cast<uint4*>(ring_value), ring_lanes, k_lanes, nk,
      static_cast<const uint4*>(k_data), v_lanes, nv, static_cast<const uint4*>(v_data), row_words,
      device_error_ptr(), nullptr, nullptr, 0);
  QKV_CHECK_LAUNCH("window_scatter_kernel");
  return QKV_OK;
}

}  // extern "C"
