// Library-wide entry points of libqkv_sm100: version, thread-local error
// messages, the per-device error word and the cached device properties.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "qkv_common.cuh"

namespace qkv {

namespace {
thread_local int t_status = QKV_OK;
thread_local std::string t_message;

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int* g_err_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
}  // namespace

// First kernel-recorded error on this device (0 = none).
__device__ int g_device_error = 0;

int set_error(int status, const std::string& msg) {
  t_status = status;
  t_message = msg;
  return status;
}

int cuda_error(cudaError_t err, const char* what) {
  return set_error(QKV_ERR_CUDA, std::string(what) + ": " +
                                     cudaGetErrorName(err) + " (" +
                                     cudaGetErrorString(err) + ")");
}

int* device_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return 148;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess ||
        n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

}  // namespace qkv

extern "C" {

const char* qkv_version(void) { return "qkv_sm100 0.1.0 (sm_100a)"; }

int qkv_last_error(char* buf, int len) {
  if (buf != nullptr && len > 0) {
    std::strncpy(buf, qkv::t_message.c_str(), static_cast<size_t>(len) - 1);
    buf[len - 1] = '\0';
  }
  return qkv::t_status;
}

int qkv_device_error(int* code, qkv_stream_t stream) {
  if (code == nullptr)
    return qkv::set_error(QKV_ERR_INVALID, "qkv_device_error: code is NULL");
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return qkv::cuda_error(e, "cudaStreamSynchronize");
  int* p = qkv::device_error_ptr();
  if (p == nullptr)
    return qkv::set_error(QKV_ERR_CUDA, "cannot resolve the device error word");
  int value = 0;
  e = cudaMemcpy(&value, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return qkv::cuda_error(e, "cudaMemcpy(error word)");
  if (value != 0) {
    const int zero = 0;
    e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return qkv::cuda_error(e, "cudaMemcpy(clear error)");
  }
  *code = value;
  return QKV_OK;
}

}  // extern "C"
