// INT8 dynamic per-channel KV: scale calibration and quantised paged write.
//
// Bit-exact restatement of methods/int8_dynamic/attention_backend.py:130-171
// as torch evaluates it on bf16 tensors:
//   amax = max_t |x[t, h, d]|, clamped below at bf16(1e-12)       (exact)
//   inv  = bf16(bf16(1 / amax) * 127)    (torch implements scalar / tensor
//                                         as reciprocal() * scalar)
//   aq   = bf16(1 / inv)                 (the BNSD antiquant scale)
//   code = clamp(rint(bf16(x * inv) + 0), -128, 127)   (round half to even)
#include "qkv_common.cuh"

namespace qkv {
namespace {

constexpr int kScaleCols = 32;   // channels per CTA (one per lane)
constexpr int kScaleWarps = 8;   // token stripes per CTA

// grid.x = column tiles over kvh*D, grid.y = 0 (key) / 1 (value).
__global__ void __launch_bounds__(kScaleCols * kScaleWarps)
int8_scales_kernel(const __nv_bfloat16* __restrict__ key,
                   const __nv_bfloat16* __restrict__ value, int64_t num_tokens,
                   int cols, __nv_bfloat16* __restrict__ k_inv,
                   __nv_bfloat16* __restrict__ v_inv,
                   __nv_bfloat16* __restrict__ k_aq,
                   __nv_bfloat16* __restrict__ v_aq) {
  __shared__ float red[kScaleWarps][kScaleCols];
  const int lane = threadIdx.x % kScaleCols;
  const int warp = threadIdx.x / kScaleCols;
  const int col = blockIdx.x * kScaleCols + lane;
  const __nv_bfloat16* src = blockIdx.y == 0 ? key : value;
  float amax = 0.0f;
  if (col < cols) {
    for (int64_t t = warp; t < num_tokens; t += kScaleWarps)
      amax = fmaxf(amax, fabsf(__bfloat162float(src[t * cols + col])));
  }
  red[warp][lane] = amax;
  __syncthreads();
  if (warp != 0 || col >= cols) return;
#pragma unroll
  for (int w = 1; w < kScaleWarps; ++w) amax = fmaxf(amax, red[w][lane]);
  const float floor_bf16 = __bfloat162float(__float2bfloat16_rn(1e-12f));
  amax = fmaxf(amax, floor_bf16);
  const float recip = bf16_round(__fdiv_rn(1.0f, amax));
  const __nv_bfloat16 inv = __float2bfloat16_rn(__fmul_rn(recip, 127.0f));
  const __nv_bfloat16 aq = __float2bfloat16_rn(__fdiv_rn(1.0f, __bfloat162float(inv)));
  if (blockIdx.y == 0) {
    k_inv[col] = inv;
    k_aq[col] = aq;
  } else {
    v_inv[col] = inv;
    v_aq[col] = aq;
  }
}

__device__ __forceinline__ int8_t quant_int8(float x, float inv) {
  // x and inv are bf16 values: their fp32 product is exact, then rounded to
  // bf16 as torch's bf16 multiply does; adding the zero offset is exact.
  float q = rintf(bf16_round(__fmul_rn(x, inv)));
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(q));
}

// One thread per (token, side, head, 16-channel chunk): reads 32 B of bf16,
// writes 16 B of codes at the token's slot.
__global__ void __launch_bounds__(256)
int8_quant_store_kernel(const __nv_bfloat16* __restrict__ key,
                        const __nv_bfloat16* __restrict__ value,
                        const void* __restrict__ slots, int slot_dtype,
                        int64_t num_tokens, int cols, int64_t num_slots,
                        const __nv_bfloat16* __restrict__ k_inv,
                        const __nv_bfloat16* __restrict__ v_inv,
                        int8_t* __restrict__ kc, int8_t* __restrict__ vc,
                        int* err) {
  const int chunks = cols / 16;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid >= num_tokens * 2 * chunks) return;
  const int c = static_cast<int>(tid % chunks);
  const int side = static_cast<int>((tid / chunks) % 2);
  const int64_t token = tid / (2 * chunks);
  const int64_t slot = load_index(slots, slot_dtype, token);
  if (slot < 0) return;
  if (slot >= num_slots) {
    record_error(err, kErrSlot);
    return;
  }
  const __nv_bfloat16* src = (side == 0 ? key : value) + token * cols + c * 16;
  const __nv_bfloat16* inv = (side == 0 ? k_inv : v_inv) + c * 16;
  int8_t* dst = (side == 0 ? kc : vc) + slot * cols + c * 16;
  uint4 xr[2], ir[2];
  xr[0] = reinterpret_cast<const uint4*>(src)[0];
  xr[1] = reinterpret_cast<const uint4*>(src)[1];
  ir[0] = reinterpret_cast<const uint4*>(inv)[0];
  ir[1] = reinterpret_cast<const uint4*>(inv)[1];
  const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(xr);
  const __nv_bfloat16* iv = reinterpret_cast<const __nv_bfloat16*>(ir);
  uint32_t out[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t packed = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = w * 4 + b;
      const int8_t q = quant_int8(__bfloat162float(xv[i]), __bfloat162float(iv[i]));
      packed |= static_cast<uint32_t>(static_cast<uint8_t>(q)) << (8 * b);
    }
    out[w] = packed;
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1], out[2], out[3]);
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace
}  // namespace qkv

extern "C" {

int qkv_int8_scales(const void* key, const void* value, int64_t num_tokens,
                    int num_kv_heads, int head_size, void* k_inv_scale,
                    void* v_inv_scale, void* k_aq_scale, void* v_aq_scale,
                    qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(num_tokens >= 0 && num_kv_heads > 0 && head_size > 0,
                "qkv_int8_scales: bad sizes");
  QKV_CHECK_ARG(key && value && k_inv_scale && v_inv_scale && k_aq_scale &&
                    v_aq_scale,
                "qkv_int8_scales: null pointer");
  const int cols = num_kv_heads * head_size;
  dim3 grid((cols + kScaleCols - 1) / kScaleCols, 2);
  int8_scales_kernel<<<grid, kScaleCols * kScaleWarps, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(key),
      static_cast<const __nv_bfloat16*>(value), num_tokens, cols,
      static_cast<__nv_bfloat16*>(k_inv_scale),
      static_cast<__nv_bfloat16*>(v_inv_scale),
      static_cast<__nv_bfloat16*>(k_aq_scale),
      static_cast<__nv_bfloat16*>(v_aq_scale));
  QKV_CHECK_LAUNCH("int8_scales_kernel");
  return QKV_OK;
}

int qkv_int8_quant_store(const void* key, const void* value,
                         const void* slot_mapping, int slot_dtype,
                         int64_t num_tokens, int num_kv_heads, int head_size,
                         int block_size, int64_t num_blocks,
                         const void* k_inv_scale, const void* v_inv_scale,
                         int8_t* key_cache, int8_t* value_cache,
                         qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(slot_dtype == QKV_I32 || slot_dtype == QKV_I64,
                "qkv_int8_quant_store: slot_mapping must be int32/int64");
  QKV_CHECK_ARG(num_tokens >= 0 && num_kv_heads > 0 && block_size > 0 &&
                    num_blocks > 0,
                "qkv_int8_quant_store: bad sizes");
  QKV_CHECK_ARG(head_size > 0 && (num_kv_heads * head_size) % 16 == 0,
                "qkv_int8_quant_store: num_kv_heads*head_size must be a "
                "multiple of 16");
  if (num_tokens == 0) return QKV_OK;
  QKV_CHECK_ARG(key && value && slot_mapping && k_inv_scale && v_inv_scale &&
                    key_cache && value_cache,
                "qkv_int8_quant_store: null pointer");
  QKV_CHECK_ARG(aligned16(key) && aligned16(value) && aligned16(k_inv_scale) &&
                    aligned16(v_inv_scale) && aligned16(key_cache) &&
                    aligned16(value_cache),
                "qkv_int8_quant_store: tensors must be 16-byte aligned");
  const int cols = num_kv_heads * head_size;
  const int64_t threads = num_tokens * 2 * (cols / 16);
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  int8_quant_store_kernel<<<grid, block, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(key),
      static_cast<const __nv_bfloat16*>(value), slot_mapping, slot_dtype,
      num_tokens, cols, num_blocks * block_size,
      static_cast<const __nv_bfloat16*>(k_inv_scale),
      static_cast<const __nv_bfloat16*>(v_inv_scale), key_cache, value_cache,
      device_error_ptr());
  QKV_CHECK_LAUNCH("int8_quant_store_kernel");
  return QKV_OK;
}

}  // extern "C"
