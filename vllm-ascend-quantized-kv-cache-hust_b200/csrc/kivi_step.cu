// One KIVI decode step in one call (host runtime + launches).
//
// The DecodeOnly branch of the reference's forward
// (methods/kivi_int4/attention_backend.py:1006-1040 -> _write_kivi_cache
// :562-606, _sync_kivi_residual_windows :813-836,
// _forward_kivi_paged_decode_attention :1193-1230) walks tokens in Python,
// reads slot ids back from the device and launches a pack per flush. Here a
// step is: plan both windows for one new token per request (the native
// planner of window_plan.cpp), check that every window still holds its
// request's last positions and prune the ones that do not, then stage every
// index the device needs (plan lists, window state per request, lengths) in
// one pinned buffer, copy it with ONE host-to-device copy, and launch the
// gather of flushed / written rows, the key and value packs, the ring scatter
// and the decode attention — all on the caller's stream, with no host sync.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <unordered_set>
#include <vector>

#include "qkv_common.cuh"
#include "qkv_sm100.h"
#include "window_plan.h"

namespace qkv {

// internal launchers (kivi_pack.cu, window_apply.cu)
int pack_value_from_sources(const __nv_bfloat16* ring, int64_t ring_lanes, const __nv_bfloat16* fresh,
                            int64_t n_new, const int64_t* src, const int64_t* slots, int64_t num_tokens, int kvh,
                            int head_size, int group_size, int block_size, int64_t num_blocks, int32_t* vq,
                            float* vs, float* vm, cudaStream_t stream);
int scatter_new_tokens(void* ring_key, void* ring_value, int64_t ring_lanes, const int64_t* k_lanes,
                       const int64_t* k_src, int64_t nk, const int64_t* v_lanes, const int64_t* v_src, int64_t nv,
                       const void* new_key, const void* new_value, int64_t n_new, int64_t row_bytes,
                       cudaStream_t stream);

namespace {

// Pinned staging ring: a buffer is rewritten only after the copy that last
// read it has completed (its event), so steps never wait on each other.
struct Pinned {
  void* host = nullptr;
  size_t cap = 0;
  cudaEvent_t done = nullptr;
};

struct StepRuntime {
  int device = 0;
  Pinned pinned[2];
  int turn = 0;
  void* dev = nullptr;  // device staging: index lists, then gathered rows
  size_t dev_cap = 0;
  std::vector<int64_t> scratch64;
  std::vector<int64_t> live;
};

size_t align16(size_t x) { return (x + 15) & ~size_t{15}; }

int ensure_pinned(Pinned& p, size_t bytes) {
  if (p.done == nullptr) {
    const cudaError_t e = cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_error(e, "cudaEventCreate(step staging)");
  } else {
    const cudaError_t e = cudaEventSynchronize(p.done);  // the copy that last read this buffer
    if (e != cudaSuccess) return cuda_error(e, "cudaEventSynchronize(step staging)");
  }
  if (p.cap >= bytes) return QKV_OK;
  if (p.host != nullptr) cudaFreeHost(p.host);
  p.host = nullptr;
  const size_t cap = std::max(bytes, std::max(p.cap * 2, size_t{1} << 16));
  const cudaError_t e = cudaHostAlloc(&p.host, cap, cudaHostAllocDefault);
  if (e != cudaSuccess) return cuda_error(e, "cudaHostAlloc(step staging)");
  p.cap = cap;
  return QKV_OK;
}

int ensure_device(StepRuntime& rt, size_t bytes, cudaStream_t stream) {
  if (rt.dev_cap >= bytes) return QKV_OK;
  if (rt.dev != nullptr) {
    // kernels of earlier steps may still read the old buffer
    const cudaError_t s = cudaStreamSynchronize(stream);
    if (s != cudaSuccess) return cuda_error(s, "cudaStreamSynchronize(step staging)");
    cudaFree(rt.dev);
    rt.dev = nullptr;
  }
  const size_t cap = std::max(bytes, std::max(rt.dev_cap * 2, size_t{1} << 20));
  const cudaError_t e = cudaMalloc(&rt.dev, cap);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(step staging)");
  rt.dev_cap = cap;
  return QKV_OK;
}

// True when ring[k] == base + k for k in [0, n): the slots of consecutive
// positions inside one page.
bool is_run(const int64_t* ring, int64_t n, int64_t base) {
  int64_t bad = 0;
  for (int64_t k = 0; k < n; ++k) bad |= ring[k] ^ (base + k);
  return bad == 0;
}

// Whether both windows of `row` hold exactly the slots of positions
// [L - n, L) in FIFO order. Walks page runs (one table lookup and one division
// per page touched) and compares each contiguous piece of the ring against an
// arithmetic progression.
bool window_holds_last_positions(const win::Window& w, int64_t row, int64_t L, const int32_t* table, int cols,
                                 int blk) {
  for (const win::Side& sd : w.side) {
    const int64_t n = sd.length[row];
    if (n > L) return false;
    if (n == 0) continue;
    const int64_t* ring = sd.slots + row * w.cap;
    int64_t lane = sd.start[row] % w.cap;
    int64_t pos = L - n, col = pos / blk, off = pos % blk;
    for (int64_t j = 0; j < n;) {
      if (col >= cols || table[col] < 0) return false;
      // positions of this page, cut where the ring wraps
      const int64_t run = std::min(std::min(n - j, static_cast<int64_t>(blk) - off), w.cap - lane);
      if (!is_run(ring + lane, run, static_cast<int64_t>(table[col]) * blk + off)) return false;
      j += run;
      off += run;
      lane += run;
      if (lane == w.cap) lane = 0;
      if (off == blk) {
        off = 0;
        ++col;
      }
    }
  }
  return true;
}

}  // namespace
}  // namespace qkv

extern "C" {

QKV_API void* qkv_kivi_step_create(void) { return new (std::nothrow) qkv::StepRuntime(); }

QKV_API void qkv_kivi_step_destroy(void* h) {
  auto* rt = static_cast<qkv::StepRuntime*>(h);
  if (rt == nullptr) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(rt->device);
  for (auto& p : rt->pinned) {
    if (p.done != nullptr) {
      cudaEventSynchronize(p.done);
      cudaEventDestroy(p.done);
    }
    if (p.host != nullptr) cudaFreeHost(p.host);
  }
  if (rt->dev != nullptr) {
    cudaDeviceSynchronize();
    cudaFree(rt->dev);
  }
  cudaSetDevice(prev);
  delete rt;
}

QKV_API int qkv_kivi_decode_step(
    void* step, void* window, int batch, const int64_t* rows, const int64_t* slots, const int32_t* seq_lens,
    const int32_t* block_table_host, int table_cols, const int32_t* block_table, int64_t bt_stride,
    const void* query, int64_t q_stride, const void* new_key, const void* new_value, int32_t* k_quant,
    float* k_scale, float* k_mn, int32_t* v_quant, float* v_scale, float* v_mn, void* res_key, void* res_value,
    int num_heads, int num_kv_heads, int head_size, int group_size, int block_size, int64_t num_blocks,
    float scale, void* workspace, size_t workspace_bytes, void* out, int64_t out_stride, qkv_stream_t stream) {
  using namespace qkv;
  auto* rt = static_cast<StepRuntime*>(step);
  auto* w = static_cast<win::Window*>(window);
  QKV_CHECK_ARG(rt != nullptr && w != nullptr, "qkv_kivi_decode_step: null runtime or window");
  QKV_CHECK_ARG(batch > 0 && batch <= w->rows && table_cols > 0 && block_size > 0 && num_kv_heads > 0 &&
                    head_size > 0 && head_size % 8 == 0,
                "qkv_kivi_decode_step: bad sizes");
  QKV_CHECK_ARG(rows && slots && seq_lens && block_table_host && query && new_key && new_value &&
                    res_key && res_value && out,
                "qkv_kivi_decode_step: null pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaGetDevice(&rt->device);
  const int cap = w->cap;
  const int64_t ring_lanes = static_cast<int64_t>(w->rows) * cap;
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_size * 2;  // bf16 rings

  // ---- 1. plan one token per request on both windows
  qkv_window_begin(w);
  std::vector<int64_t>& tok = rt->scratch64;
  tok.resize(batch);
  for (int b = 0; b < batch; ++b) tok[b] = b;
  for (int b = 0; b < batch; ++b)
    QKV_CHECK_ARG(rows[b] >= 0 && rows[b] < w->rows && slots[b] >= 0, "qkv_kivi_decode_step: bad row or slot");
  if (qkv_window_store_one_each(w, batch, rows, slots, tok.data(), 1, block_size) != QKV_OK)
    return set_error(QKV_ERR_INVALID, "KIVI key flush requires contiguous aligned token groups.");
  if (qkv_window_store_one_each(w, batch, rows, slots, tok.data(), 0, 0) != QKV_OK)
    return set_error(QKV_ERR_INVALID, "qkv_kivi_decode_step: value window store failed");

  // ---- 2. sync: a window that no longer holds its request's last positions
  // keeps only the slots the request owns (compacted, FIFO order)
  int32_t max_len = 0;
  for (int b = 0; b < batch; ++b) {
    const int64_t L = std::max<int32_t>(seq_lens[b], 0);
    max_len = std::max<int32_t>(max_len, static_cast<int32_t>(L));
    const int32_t* trow = block_table_host + static_cast<int64_t>(b) * table_cols;
    if (window_holds_last_positions(*w, rows[b], L, trow, table_cols, block_size)) continue;
    rt->live.clear();
    for (int64_t p = 0; p < L; ++p) {
      const int64_t col = p / block_size;
      if (col < table_cols && trow[col] >= 0)
        rt->live.push_back(static_cast<int64_t>(trow[col]) * block_size + p % block_size);
    }
    for (int k = 1; k >= 0; --k)
      qkv_window_prune(w, static_cast<int>(rows[b]), static_cast<int>(rt->live.size()), rt->live.data(), k);
  }

  // ---- 3. the plan's lists (deduplicated flushes, ring writes)
  int64_t nf[2], nw[2];
  for (int k = 0; k < 2; ++k) qkv_window_plan_counts(w, 1 - k, &nf[k], &nw[k]);
  // staging layout (int64): [k_src: nf0+nw0][v_src: nf1+nw1][k_fslots][v_fslots][k_lanes][v_lanes]
  // then int32: res_state [B, 6], seq_lens [B], and (without a device block
  // table) the host table [B, table_cols]; then (device only) gathered rows
  const int64_t n64 = nf[0] + nw[0] + nf[1] + nw[1] + nf[0] + nf[1] + nw[0] + nw[1];
  const size_t bytes64 = align16(static_cast<size_t>(n64) * 8);
  const bool stage_table = block_table == nullptr;
  const size_t table_words = stage_table ? static_cast<size_t>(batch) * table_cols : 0;
  const size_t bytes32 = align16((static_cast<size_t>(batch) * 7 + table_words) * 4);
  const size_t rows_k = static_cast<size_t>(nf[0] + nw[0]), rows_v = static_cast<size_t>(nf[1] + nw[1]);
  const size_t staged = bytes64 + bytes32;
  const size_t total = staged + (rows_k + rows_v) * static_cast<size_t>(row_bytes);
  Pinned& pin = rt->pinned[rt->turn];
  rt->turn ^= 1;
  int rc = ensure_pinned(pin, staged);
  if (rc != QKV_OK) return rc;
  if ((rc = ensure_device(*rt, total, st)) != QKV_OK) return rc;
  auto* h64 = static_cast<int64_t*>(pin.host);
  int64_t* k_src = h64;
  int64_t* v_src = k_src + nf[0] + nw[0];
  int64_t* k_fsl = v_src + nf[1] + nw[1];
  int64_t* v_fsl = k_fsl + nf[0];
  int64_t* k_lan = v_fsl + nf[1];
  int64_t* v_lan = k_lan + nw[0];
  // export writes flush sources then write sources of each side contiguously
  for (int k = 0; k < 2; ++k) {
    int64_t* src = k == 0 ? k_src : v_src;
    qkv_window_plan_export(w, 1 - k, src, k == 0 ? k_fsl : v_fsl, k == 0 ? k_lan : v_lan, src + nf[k]);
  }
  auto* h32 = reinterpret_cast<int32_t*>(static_cast<char*>(pin.host) + bytes64);
  for (int b = 0; b < batch; ++b) {
    const int64_t r = rows[b];
    int32_t* s6 = h32 + 6 * b;
    s6[0] = static_cast<int32_t>(r);
    s6[1] = static_cast<int32_t>(w->side[0].start[r]);
    s6[2] = static_cast<int32_t>(w->side[0].length[r]);
    s6[3] = static_cast<int32_t>(w->side[1].start[r]);
    s6[4] = static_cast<int32_t>(w->side[1].length[r]);
    s6[5] = seq_lens[b];
    h32[6 * batch + b] = seq_lens[b];
  }
  if (stage_table) std::memcpy(h32 + 7 * batch, block_table_host, table_words * 4);
  cudaError_t e = cudaMemcpyAsync(rt->dev, pin.host, staged, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync(step staging)");
  e = cudaEventRecord(pin.done, st);
  if (e != cudaSuccess) return cuda_error(e, "cudaEventRecord(step staging)");

  // device views of the staged lists
  auto* d64 = static_cast<int64_t*>(rt->dev);
  const int64_t* dk_src = d64;
  const int64_t* dv_src = dk_src + nf[0] + nw[0];
  const int64_t* dk_fsl = dv_src + nf[1] + nw[1];
  const int64_t* dv_fsl = dk_fsl + nf[0];
  const int64_t* dk_lan = dv_fsl + nf[1];
  const int64_t* dv_lan = dk_lan + nw[0];
  auto* d32 = reinterpret_cast<const int32_t*>(static_cast<char*>(rt->dev) + bytes64);
  char* gk = static_cast<char*>(rt->dev) + staged;
  char* gv = gk + rows_k * row_bytes;

  // ---- 4. gather, packs, scatter, decode
  // A steady decode step (no key window flushes, every ring write a new
  // token) needs no snapshot: the value pack reads its flushed lanes in place
  // before the scatter overwrites them (stream order), and the scatter reads
  // the new tokens directly. Otherwise the plan's rows are gathered first.
  bool direct = nf[0] == 0 && (head_size / 8 & (head_size / 8 - 1)) == 0 && head_size / 8 <= 32;
  for (int64_t i = 0; direct && i < nw[0]; ++i) direct = k_src[nf[0] + i] < 0;
  for (int64_t i = 0; direct && i < nw[1]; ++i) direct = v_src[nf[1] + i] < 0;
  if (direct) {
    if (nf[1] > 0) {
      rc = pack_value_from_sources(static_cast<const __nv_bfloat16*>(res_value), ring_lanes,
                                   static_cast<const __nv_bfloat16*>(new_value), batch, dv_src, dv_fsl, nf[1],
                                   num_kv_heads, head_size, group_size, block_size, num_blocks, v_quant, v_scale,
                                   v_mn, st);
      if (rc != QKV_OK) return rc;
    }
    rc = scatter_new_tokens(res_key, res_value, ring_lanes, dk_lan, dk_src + nf[0], nw[0], dv_lan, dv_src + nf[1],
                            nw[1], new_key, new_value, batch, row_bytes, st);
    if (rc != QKV_OK) return rc;
    // when the scatter launched (ring writes exist), it is the last launch
    // and wrote only the rings (the pack and the staged metadata are
    // complete): the decode may overlap it
    if (nw[0] + nw[1] > 0)
      return kivi_paged_decode_after_ring_write(
          query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key, res_value, w->rows, cap,
          stage_table ? d32 + 7 * batch : block_table, stage_table ? table_cols : bt_stride, d32 + 6 * batch, d32,
          batch, num_heads, num_kv_heads, head_size, group_size, block_size, num_blocks, std::max(max_len, 1), scale,
          workspace, workspace_bytes, out, out_stride, stream);
    return qkv_kivi_paged_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key,
                                 res_value, w->rows, cap, stage_table ? d32 + 7 * batch : block_table,
                                 stage_table ? table_cols : bt_stride, d32 + 6 * batch, d32, batch, num_heads,
                                 num_kv_heads, head_size, group_size, block_size, num_blocks, std::max(max_len, 1),
                                 scale, workspace, workspace_bytes, out, out_stride, stream);
  }
  if (rows_k + rows_v > 0) {
    rc = qkv_kivi_window_gather(res_key, res_value, ring_lanes, new_key, new_value, batch, dk_src,
                                static_cast<int64_t>(rows_k), dv_src, static_cast<int64_t>(rows_v), row_bytes, gk, gv,
                                stream);
    if (rc != QKV_OK) return rc;
  }
  if (nf[0] > 0) {
    rc = qkv_kivi_pack_key(gk, QKV_BF16, dk_fsl, QKV_I64, nf[0], num_kv_heads, head_size, group_size, block_size,
                           num_blocks, k_quant, k_scale, k_mn, stream);
    if (rc != QKV_OK) return rc;
  }
  if (nf[1] > 0) {
    rc = qkv_kivi_pack_value(gv, QKV_BF16, dv_fsl, QKV_I64, nf[1], num_kv_heads, head_size, group_size, block_size,
                             num_blocks, v_quant, v_scale, v_mn, stream);
    if (rc != QKV_OK) return rc;
  }
  if (nw[0] + nw[1] > 0) {
    rc = qkv_kivi_window_scatter(res_key, res_value, ring_lanes, dk_lan, nw[0], gk + nf[0] * row_bytes, dv_lan,
                                 nw[1], gv + nf[1] * row_bytes, row_bytes, stream);
    if (rc != QKV_OK) return rc;
  }
  return qkv_kivi_paged_decode(query, q_stride, k_quant, k_scale, k_mn, v_quant, v_scale, v_mn, res_key, res_value,
                               w->rows, cap, stage_table ? d32 + 7 * batch : block_table,
                               stage_table ? table_cols : bt_stride, d32 + 6 * batch, d32, batch, num_heads,
                               num_kv_heads, head_size, group_size, block_size, num_blocks, std::max(max_len, 1),
                               scale, workspace, workspace_bytes, out, out_stride, stream);
}

}  // extern "C"
