// FP8 per-token-head KV: the store (each (token, head) quantised to E4M3 with
// its own fp32 scale, scattered into the paged views) and the dense gather
// (E4M3 pages -> bf16 rows of whole requests) of the fp8_per_token_head
// method (methods/fp8_per_token_head/semantics.py:52-76, byte_cache.py; the
// reference's store kernel is ops/triton/per_token_head_store.py:262-294).
//
// Store, per (token, head), in the semantics' operation order:
//     amax  = max |x|                          (fp32)
//     scale = max(amax / 448, 1e-6)            (fp32 division, then floor)
//     code  = e4m3(clamp(x / scale, -448, 448)) (fp32 division; RNE to E4M3)
// One warp per (token, head): each lane holds D / 32 channels, the amax is a
// warp reduction, the codes go out as 4-byte words.
#include <cuda_fp8.h>

#include "decode_common.cuh"

namespace qkv {

namespace {

constexpr float kE4m3Max = 448.0f;
constexpr float kScaleFloor = 1e-6f;

template <typename T>
__global__ void fp8_store_kernel(const T* key, const T* value, const void* slots, int slot_dtype,
                                 int64_t num_tokens, int kvh, int D, int blk, int64_t num_blocks,
                                 uint8_t* k_data, float* k_scale, uint8_t* v_data, float* v_scale, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= num_tokens * kvh) return;
  const int64_t tok = item / kvh;
  const int h = static_cast<int>(item % kvh);
  const int64_t slot = load_index(slots, slot_dtype, tok);
  if (slot < 0) return;
  if (slot >= num_blocks * blk) {
    if (lane == 0) record_error(err, kErrSlot);
    return;
  }
  const int64_t row = slot * kvh + h;  // [NB * blk, KVH] (page-major, then slot in page)
  for (int side = 0; side < 2; ++side) {
    const T* x = (side == 0 ? key : value) + (tok * kvh + h) * D;
    uint8_t* dst = (side == 0 ? k_data : v_data) + row * D;
    float* sdst = (side == 0 ? k_scale : v_scale) + row;
    float amax = 0.0f;
    for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(to_f32(x[d])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fmaxf(__fdiv_rn(amax, kE4m3Max), kScaleFloor);
    if (lane == 0) *sdst = scale;
    for (int d0 = 4 * lane; d0 < D; d0 += 128) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float q = fminf(fmaxf(__fdiv_rn(to_f32(x[d0 + i]), scale), -kE4m3Max), kE4m3Max);
        const uint32_t c = __nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
        word |= (c & 0xFFu) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(dst + d0) = word;
    }
  }
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t c) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(c), __NV_E4M3);
  return __half2float(__half(h));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Dense gather: one thread per (token, head, 16 channels); bf16(code * scale)
// with the product rounded to fp32 first (the semantics' dequantise, then the
// cast of the attention inputs).
__global__ void fp8_gather_kernel(const DecodeParams p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                                  __nv_bfloat16* dense_v) {
  const int chunks = p.head_size / 16;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t per_token = static_cast<int64_t>(p.kvh) * chunks;
  if (idx >= static_cast<int64_t>(total_k) * per_token) return;
  const int tok = static_cast<int>(idx / per_token);
  const int hc = static_cast<int>(idx % per_token);
  const int h = hc / chunks, c = hc % chunks;
  int lo = 0, hi = p.num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_k[mid] <= tok) lo = mid; else hi = mid - 1;
  }
  const int t = tok - cu_k[lo];
  const int64_t page = page_of(p, lo, t);
  uint4 ko[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, vo[2] = {ko[0], ko[1]};
  if (page >= 0) {
    const int64_t row = (page * p.blk + t % p.blk) * p.kvh + h;
    for (int side = 0; side < 2; ++side) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(side == 0 ? p.kc : p.vc) + row * p.head_size + 16 * c;
      const float sc = (side == 0 ? p.ks : p.vs)[row];
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
      const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = pack_bf16x2(__fmul_rn(e4m3_to_f32(b[2 * i]), sc), __fmul_rn(e4m3_to_f32(b[2 * i + 1]), sc));
      uint4* o = side == 0 ? ko : vo;
      o[0] = make_uint4(w[0], w[1], w[2], w[3]);
      o[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
  const int64_t off = (static_cast<int64_t>(tok) * p.kvh + h) * p.head_size + 16 * c;
  reinterpret_cast<uint4*>(dense_k + off)[0] = ko[0];
  reinterpret_cast<uint4*>(dense_k + off)[1] = ko[1];
  reinterpret_cast<uint4*>(dense_v + off)[0] = vo[0];
  reinterpret_cast<uint4*>(dense_v + off)[1] = vo[1];
}

bool aligned(const void* x, unsigned a) { return (reinterpret_cast<uintptr_t>(x) & (a - 1)) == 0; }

}  // namespace

}  // namespace qkv

extern "C" {

int qkv_fp8_store(const void* key, const void* value, int kv_dtype, const void* slot_mapping, int slot_dtype,
                  int64_t num_tokens, int num_kv_heads, int head_size, int block_size, int64_t num_blocks,
                  uint8_t* k_data, float* k_scale, uint8_t* v_data, float* v_scale, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(num_tokens >= 0 && num_kv_heads > 0 && block_size > 0 && num_blocks > 0,
                "qkv_fp8_store: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && head_size % 4 == 0,
                "fp8_per_token_head requires head_size divisible by 4 (fp32 scale alignment), got " +
                    std::to_string(head_size) + ".");
  QKV_CHECK_ARG(kv_dtype == QKV_F32 || kv_dtype == QKV_BF16 || kv_dtype == QKV_F16, "qkv_fp8_store: bad dtype");
  QKV_CHECK_ARG(slot_dtype == QKV_I32 || slot_dtype == QKV_I64,
                "fp8_per_token_head slot_mapping must be int32/int64.");
  if (num_tokens == 0) return QKV_OK;
  QKV_CHECK_ARG(key && value && slot_mapping && k_data && k_scale && v_data && v_scale,
                "qkv_fp8_store: null pointer");
  QKV_CHECK_ARG(aligned(k_data, 4) && aligned(v_data, 4), "qkv_fp8_store: data caches must be 4-byte aligned");
  const int64_t items = num_tokens * num_kv_heads;
  const int warps = 8;
  const int64_t grid = (items + warps - 1) / warps;
  QKV_CHECK_ARG(grid <= 0x7FFFFFFFll, "qkv_fp8_store: too many tokens");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = device_error_ptr();
  if (kv_dtype == QKV_BF16)
    fp8_store_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), 32 * warps, 0, s>>>(
        static_cast<const __nv_bfloat16*>(key), static_cast<const __nv_bfloat16*>(value), slot_mapping,
        slot_dtype, num_tokens, num_kv_heads, head_size, block_size, num_blocks, k_data, k_scale, v_data, v_scale,
        err);
  else if (kv_dtype == QKV_F16)
    fp8_store_kernel<__half><<<static_cast<unsigned>(grid), 32 * warps, 0, s>>>(
        static_cast<const __half*>(key), static_cast<const __half*>(value), slot_mapping, slot_dtype, num_tokens,
        num_kv_heads, head_size, block_size, num_blocks, k_data, k_scale, v_data, v_scale, err);
  else
    fp8_store_kernel<float><<<static_cast<unsigned>(grid), 32 * warps, 0, s>>>(
        static_cast<const float*>(key), static_cast<const float*>(value), slot_mapping, slot_dtype, num_tokens,
        num_kv_heads, head_size, block_size, num_blocks, k_data, k_scale, v_data, v_scale, err);
  QKV_CHECK_LAUNCH("fp8_store_kernel");
  return QKV_OK;
}

int qkv_fp8_dequant_gather(const uint8_t* k_data, const float* k_scale, const uint8_t* v_data,
                           const float* v_scale, const int32_t* block_table, int64_t bt_stride,
                           const int32_t* seq_lens, const int32_t* cu_seqlens_k, int batch, int num_kv_heads,
                           int head_size, int block_size, int64_t num_blocks, int total_k, void* out_key,
                           void* out_value, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(batch >= 0 && total_k >= 0 && num_kv_heads > 0 && num_blocks > 0 && block_size > 0,
                "qkv_fp8_dequant_gather: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && head_size % 16 == 0, "qkv_fp8_dequant_gather: head_size must be a multiple of 16");
  if (batch == 0 || total_k == 0) return QKV_OK;
  QKV_CHECK_ARG(k_data && k_scale && v_data && v_scale && block_table && seq_lens && cu_seqlens_k && out_key &&
                    out_value,
                "qkv_fp8_dequant_gather: null pointer");
  QKV_CHECK_ARG(aligned(k_data, 16) && aligned(v_data, 16) && aligned(out_key, 16) && aligned(out_value, 16),
                "qkv_fp8_dequant_gather: data caches and outputs must be 16-byte aligned");
  DecodeParams p{};
  p.kc = reinterpret_cast<const int8_t*>(k_data);
  p.vc = reinterpret_cast<const int8_t*>(v_data);
  p.ks = k_scale;
  p.vs = v_scale;
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
  const int64_t threads = static_cast<int64_t>(total_k) * num_kv_heads * (head_size / 16);
  const int64_t grid = (threads + 255) / 256;
  QKV_CHECK_ARG(grid <= 0x7FFFFFFFll, "qkv_fp8_dequant_gather: too many elements");
  fp8_gather_kernel<<<static_cast<unsigned>(grid), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      p, cu_seqlens_k, total_k, static_cast<__nv_bfloat16*>(out_key), static_cast<__nv_bfloat16*>(out_value));
  QKV_CHECK_LAUNCH("fp8_gather_kernel");
  return QKV_OK;
}

}  // extern "C"
