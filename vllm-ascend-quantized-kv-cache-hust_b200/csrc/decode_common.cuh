// Shared pieces of the paged decode kernels: the parameter block, the
// split-KV plan and the combine kernel that merges per-split partial softmax
// states into the bf16 output.
#pragma once

#include "qkv_common.cuh"

namespace qkv {

// Decode attention over the quantised pages of one layer. One CTA owns one
// (request, kv head, split); the split index num_hist_splits (KIVI only) is the
// "tail" split that covers the positions whose key or value still lives in the
// bf16 residual window.
struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_stride;
  // INT8 pages [NB, blk, KVH, D] and bf16 antiquant scales [KVH, D]
  const int8_t* kc;
  const int8_t* vc;
  const __nv_bfloat16* k_aq;
  const __nv_bfloat16* v_aq;
  // KIVI views
  const int32_t* kq;
  const float* ks;
  const float* km;
  const int32_t* vq;
  const float* vs;
  const float* vm;
  const __nv_bfloat16* rk;  // [res_rows, res_cap, KVH, D]
  const __nv_bfloat16* rv;
  int res_rows;
  int res_cap;
  const int32_t* res_state;  // [B, 6]
  // dense bf16 K/V [total_k, KVH, D] of a TND prefill (mode kDense); query row
  // r belongs to the request b with cu_q[b] <= r < cu_q[b+1]
  const __nv_bfloat16* dk;
  const __nv_bfloat16* dv;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_reqs;
  int causal;
  // common
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int batch, num_heads, kvh, head_size, gqa, group, blk;
  int64_t num_blocks;
  float scale_log2;  // softmax scale * log2(e)
  int num_hist_splits;
  int split_tokens;  // tokens per history split (multiple of blk)
  int splits_total;  // history splits (+1 tail split for KIVI)
  int split_base;    // blockIdx.x + split_base = split index of a CTA
  int split_mid;     // KIVI page-pipelined grid: 0 (kv head, request, split), 1 (kv head, split, request)
  // the launch before the decode wrote only the bf16 residual rings: the
  // decode may start before it ends (programmatic dependent launch), its
  // window CTAs waiting for it
  int after_ring_write;
  float* ws_acc;     // [B, Hq, splits_total, D]   (unnormalised)
  float* ws_ml;      // [B, Hq, splits_total, 2]   (running max, sum)
  __nv_bfloat16* out;
  int64_t out_stride;
  int* err;
};

// Where a decode/prefill kernel reads K and V from.
enum SourceMode : int { kInt8Pages = 0, kKiviPages = 1, kDense = 2, kFp8Pages = 3 };

struct SplitPlan {
  int hist_splits;
  int split_tokens;
  int total;
};

// Splits every request's quantised history into `hist_splits` page-aligned
// ranges so that batch * kvh * splits CTAs cover about `waves` x the SM count.
inline SplitPlan plan_splits(int batch, int kvh, int blk, int max_seq_len,
                             bool tail_split, int sms, int waves,
                             int min_split_tokens) {
  SplitPlan p;
  const int pages = max_seq_len > 0 ? (max_seq_len + blk - 1) / blk : 1;
  const int units = batch * kvh > 0 ? batch * kvh : 1;
  int splits = (sms * waves + units - 1) / units;
  const int min_pages = (min_split_tokens + blk - 1) / blk;
  int max_splits = pages / (min_pages > 0 ? min_pages : 1);
  if (max_splits < 1) max_splits = 1;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  const int pages_per_split = (pages + splits - 1) / splits;
  p.split_tokens = pages_per_split * blk;
  p.hist_splits = (pages + pages_per_split - 1) / pages_per_split;
  p.total = p.hist_splits + (tail_split ? 1 : 0);
  return p;
}

inline size_t workspace_bytes(int batch, int num_heads, int head_size,
                              int splits_total) {
  if (splits_total <= 1) return 0;
  const size_t rows = static_cast<size_t>(batch) * num_heads * splits_total;
  return rows * head_size * sizeof(float) + rows * 2 * sizeof(float);
}

// Residual-window bookkeeping of one query row: keys at positions
// [k_begin, end) and values at [v_begin, end) live in the bf16 window of
// residual row `row`, starting at ring lanes k_start / v_start.
struct TailState {
  int row, k_start, k_begin, v_start, v_begin, end;
};

constexpr int kResStateFields = 6;

__device__ __forceinline__ TailState load_tail_state(const DecodeParams& p,
                                                     int b, int seq_len) {
  TailState s{-1, 0, seq_len, 0, seq_len, seq_len};
  if (p.res_state == nullptr) return s;
  const int32_t* r = p.res_state + static_cast<int64_t>(b) * kResStateFields;
  if (r[0] < 0) return s;
  if (r[0] >= p.res_rows) {
    record_error(p.err, kErrResidualRow);
    return s;
  }
  const int cap = p.res_cap;
  const int end = max(r[5], 0);
  const int k_len = min(max(r[2], 0), min(cap, end));
  const int v_len = min(max(r[4], 0), min(cap, end));
  s.row = r[0];
  s.k_start = ((r[1] % cap) + cap) % cap;
  s.v_start = ((r[3] % cap) + cap) % cap;
  s.end = end;
  // a row never reads past its own causal length
  s.k_begin = min(end - k_len, seq_len);
  s.v_begin = min(end - v_len, seq_len);
  return s;
}

// Physical page of position `pos` of request b, or -1 (recorded) when the
// block table entry is out of range.
__device__ __forceinline__ int64_t page_of(const DecodeParams& p, int b,
                                           int pos) {
  const int col = pos / p.blk;
  if (col >= p.bt_stride) {  // the table row does not cover this position
    record_error(p.err, kErrBlock);
    return -1;
  }
  const int64_t page = p.bt[static_cast<int64_t>(b) * p.bt_stride + col];
  if (page < 0 || page >= p.num_blocks) {
    record_error(p.err, page < 0 ? kErrNegativeBlock : kErrBlock);
    return -1;
  }
  return page;
}

// Writes one split's state: directly normalised into `out` when the request
// has a single split, otherwise into the workspace for combine_kernel.
__device__ __forceinline__ void store_partial(const DecodeParams& p, int b,
                                              int hq, int split, int d,
                                              float acc, float m, float l) {
  if (p.splits_total == 1) {
    const float o = l > 0.0f ? acc / l : 0.0f;
    p.out[static_cast<int64_t>(b) * p.out_stride +
          static_cast<int64_t>(hq) * p.head_size + d] = __float2bfloat16_rn(o);
  } else {
    const int64_t row =
        (static_cast<int64_t>(b) * p.num_heads + hq) * p.splits_total + split;
    p.ws_acc[row * p.head_size + d] = acc;
    if (d == 0) {
      p.ws_ml[row * 2] = m;
      p.ws_ml[row * 2 + 1] = l;
    }
  }
}

// A split with nothing to attend writes only the (max, sum) = (-inf, 0) of
// its rows (kv head h's G query heads): the combine skips such a split
// without reading its sums. Only for plans of several splits (with one, the
// output itself is written by the full path).
__device__ __forceinline__ void empty_split(const DecodeParams& p, int b, int h, int split) {
  const int G = p.gqa;
  if (static_cast<int>(threadIdx.x) < G) {
    const int64_t row =
        (static_cast<int64_t>(b) * p.num_heads + static_cast<int64_t>(h) * G + threadIdx.x) * p.splits_total + split;
    p.ws_ml[row * 2] = -__int_as_float(0x7f800000);
    p.ws_ml[row * 2 + 1] = 0.0f;
  }
}

// Waits until the grid this one was launched behind with programmatic
// stream serialisation has completed and its writes are visible; returns at
// once for a grid launched without it.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Launch attributes of a programmatic dependent launch (the grid may start
// before the previous one on the stream ends; it calls grid_dependency_wait
// before reading what that grid wrote).
struct PdlConfig {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  PdlConfig(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
};

void launch_combine(const DecodeParams& p, cudaStream_t stream);

}  // namespace qkv
