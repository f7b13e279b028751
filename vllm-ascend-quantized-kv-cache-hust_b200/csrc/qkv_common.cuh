// Shared helpers of libqkv_sm100: host-side error plumbing, the device error
// word, element loads for the input dtypes, and the bf16 rounding helpers the
// bit-exact kernels rely on.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/qkv_sm100.h"

namespace qkv {

// ---------------------------------------------------------------- host side

// Records `msg` as the calling thread's last error and returns `status`.
int set_error(int status, const std::string& msg);

// Maps a failed CUDA runtime call to QKV_ERR_CUDA with its name.
int cuda_error(cudaError_t err, const char* what);

// SM count of the current device (cached per device).
int sm_count();

#define QKV_CHECK_ARG(cond, msg)                                   \
  do {                                                             \
    if (!(cond)) return ::qkv::set_error(QKV_ERR_INVALID, (msg));  \
  } while (0)

#define QKV_CHECK_LAUNCH(what)                                     \
  do {                                                             \
    cudaError_t _e = cudaGetLastError();                           \
    if (_e != cudaSuccess) return ::qkv::cuda_error(_e, (what));   \
  } while (0)

// -------------------------------------------------------------- device side

// Device error codes (mirrored in qkv_sm100.h, qkv_device_error()).
enum DeviceError : int {
  kErrSlot = 1,
  kErrBlock = 2,
  kErrResidualRow = 3,
  kErrNegativeBlock = 4,
  kErrPipelineTimeout = 5,  // a bounded wait on an in-kernel copy gave up
  kErrWindowSource = 6,     // a window plan source or lane out of range
  kErrPeerTimeout = 7,      // a bounded wait for the other ranks' flags gave up
};

// Device address of this device's error word (a __device__ int defined in
// qkv_abi.cu, resolved once per device with cudaGetSymbolAddress). Kernels get
// it as a parameter and record the first bad index they skip.
int* device_error_ptr();

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// Element loads for the floating-point input dtypes (qkv_dtype).
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) {
  return __half2float(x);
}

// Round an fp32 value to bf16 (round-to-nearest-even) and back: the rounding
// torch applies after every bf16 elementwise op on CPU.
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ int64_t load_index(const void* p, int dtype,
                                              int64_t i) {
  return dtype == QKV_I64 ? static_cast<const int64_t*>(p)[i]
                          : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// qkv_kivi_paged_decode for a caller whose last launch on `stream` wrote only
// the bf16 residual rings (the one-call decode step's ring scatter): the
// page-pipelined kernel starts before that launch ends, its history CTAs read
// pages and metadata written by earlier launches, and its window CTAs wait
// for the rings.
int kivi_paged_decode_after_ring_write(
    const void* query, int64_t q_stride, const int32_t* k_quant, const float* k_scale, const float* k_mn,
    const int32_t* v_quant, const float* v_scale, const float* v_mn, const void* res_key, const void* res_value,
    int res_rows, int res_capacity, const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* res_state, int batch, int num_heads, int num_kv_heads, int head_size, int group_size,
    int block_size, int64_t num_blocks, int max_seq_len, float scale, void* workspace, size_t workspace_bytes,
    void* out, int64_t out_stride, qkv_stream_t stream);

}  // namespace qkv
