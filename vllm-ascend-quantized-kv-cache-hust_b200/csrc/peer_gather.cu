// All-gather of the per-rank attention outputs over NVLink peer memory: the
// one exchange of the KV-head-sharded path (rank i computes query heads
// [Hq i/N, Hq (i+1)/N) of every request). Replaces the NCCL all-gather plus
// the head permute that follows it with one kernel that writes the final
// [B, Hq, D] layout.
//
// Protocol (one round, no barrier, no fence): every 4-byte word of a rank's
// slice travels to each peer together with the call's epoch in ONE 8-byte
// store into the peer's receive buffer; a receiver polls each 8-byte word
// until its flag equals the epoch, then the data word is the current one
// (an aligned 8-byte store and load are single accesses). Receive buffers are
// double-buffered by epoch parity: a rank reaches call e + 2 only after every
// peer has sent its call e + 1 words, i.e. after every peer finished
// receiving call e, so call e + 2 never overwrites words still unread.
//
// Each rank owns one device allocation, opened by its peers through CUDA IPC:
//   [0, recv)        receive words: [2 parities][world][slice_words] x 8 B
//   [recv, +64)      control: epoch (calls made), done (CTA counter)
// The epoch lives on the device, so the kernel can be captured in a CUDA
// graph and replayed. Waits give up after about a second, record an error in
// the device error word and return.
#include <cstring>

#include "decode_common.cuh"

namespace qkv {

namespace {

constexpr int kMaxPeers = 8;
constexpr int kCtlBytes = 64;
constexpr long long kPeerWaitCycles = 2000000000LL;  // ~1 s at 2 GHz

struct PeerGatherArgs {
  const uint32_t* local;       // [B, row_words] this rank's slice
  uint2* recv[kMaxPeers];      // each rank's receive words (as mapped here)
  uint32_t* ctl;               // this rank's control words
  uint32_t* out;               // [B, world * row_words] on this rank
  int64_t batch, row_words;    // row_words = Hq/N * D * 2 / 4
  int64_t slice_words;         // receive words per (parity, source rank)
  int rank, world;
  int* err;
};

__device__ __forceinline__ void store_word(uint2* p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};\n" ::"l"(p), "r"(data), "r"(flag) : "memory");
}
__device__ __forceinline__ uint2 load_word(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) peer_gather_kernel(const PeerGatherArgs a) {
  __shared__ uint32_t epoch_sh;
  __shared__ int last;
  if (threadIdx.x == 0) epoch_sh = *reinterpret_cast<volatile uint32_t*>(a.ctl) + 1;
  __syncthreads();
  const uint32_t e = epoch_sh;
  const int par = static_cast<int>(e & 1u);
  const int64_t n = a.batch * a.row_words;
  const int64_t full_row = static_cast<int64_t>(a.world) * a.row_words;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // send: this rank's words to every peer (and straight into its own output)
  for (int64_t i = t0; i < n; i += stride) {
    const uint32_t d = a.local[i];
    const int64_t b = i / a.row_words, w = i - b * a.row_words;
    a.out[b * full_row + a.rank * a.row_words + w] = d;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < a.world && r != a.rank)
        store_word(a.recv[r] + (static_cast<int64_t>(par) * a.world + a.rank) * a.slice_words + i, d, e);
  }
  // receive: every peer's words, polled until they carry this call's epoch
  const uint2* mine = a.recv[a.rank] + static_cast<int64_t>(par) * a.world * a.slice_words;
  const long long start = clock64();
  bool ok = true;
  for (int64_t j = t0; j < (a.world - 1) * n && ok; j += stride) {
    const int64_t k = j / n, i = j - k * n;
    const int src = static_cast<int>(k) + (static_cast<int>(k) >= a.rank ? 1 : 0);
    const uint2* p = mine + static_cast<int64_t>(src) * a.slice_words + i;
    uint2 v = load_word(p);
    while (v.y != e) {
      if (clock64() - start > kPeerWaitCycles) {
        ok = false;
        break;
      }
      __nanosleep(32);
      v = load_word(p);
    }
    if (!ok) break;
    const int64_t b = i / a.row_words, w = i - b * a.row_words;
    a.out[b * full_row + src * a.row_words + w] = v.x;
  }
  if (!ok) record_error(a.err, kErrPeerTimeout);
  // the last CTA of this call advances the epoch for the next one
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(reinterpret_cast<int*>(a.ctl + 1), 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    a.ctl[1] = 0;
    a.ctl[0] = e;
  }
}

size_t recv_bytes(int64_t slice_bytes_max, int world) {
  // 4-byte data words carried in 8-byte receive words, two parities
  return static_cast<size_t>(2) * world * (slice_bytes_max / 4) * 8;
}

}  // namespace

}  // namespace qkv

extern "C" {

size_t qkv_peer_buffer_bytes(int64_t slice_bytes_max, int world) {
  if (slice_bytes_max <= 0 || world <= 0) return 0;
  return qkv::recv_bytes(slice_bytes_max, world) + qkv::kCtlBytes;
}

int qkv_peer_alloc(int64_t slice_bytes_max, int world, void** ptr) {
  using namespace qkv;
  QKV_CHECK_ARG(ptr != nullptr && slice_bytes_max > 0 && slice_bytes_max % 16 == 0 && world >= 1 &&
                    world <= kMaxPeers,
                "qkv_peer_alloc: bad arguments");
  const size_t bytes = qkv_peer_buffer_bytes(slice_bytes_max, world);
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaMemset(peer buffer)");
  return QKV_OK;
}

int qkv_peer_free(void* ptr) {
  using namespace qkv;
  if (ptr == nullptr) return QKV_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? QKV_OK : cuda_error(e, "cudaFree(peer buffer)");
}

int qkv_ipc_handle(const void* ptr, void* handle_out) {
  using namespace qkv;
  QKV_CHECK_ARG(ptr != nullptr && handle_out != nullptr, "qkv_ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == QKV_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_error(e, "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  return QKV_OK;
}

int qkv_ipc_open(const void* handle, void** ptr) {
  using namespace qkv;
  QKV_CHECK_ARG(handle != nullptr && ptr != nullptr, "qkv_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? QKV_OK : cuda_error(e, "cudaIpcOpenMemHandle");
}

int qkv_ipc_close(void* ptr) {
  using namespace qkv;
  if (ptr == nullptr) return QKV_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? QKV_OK : cuda_error(e, "cudaIpcCloseMemHandle");
}

int qkv_peer_allgather(const void* local, int64_t batch, int64_t row_bytes, void* const* buffers,
                       int64_t slice_bytes_max, void* out, int rank, int world, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
                "qkv_peer_allgather: world must be 1..8 and rank inside it");
  QKV_CHECK_ARG(batch >= 0 && row_bytes > 0 && row_bytes % 4 == 0,
                "qkv_peer_allgather: a row must be a positive multiple of 4 bytes");
  QKV_CHECK_ARG(batch * row_bytes <= slice_bytes_max,
                "qkv_peer_allgather: the slice does not fit the peer buffers");
  QKV_CHECK_ARG(local != nullptr && buffers != nullptr && out != nullptr, "qkv_peer_allgather: null pointer");
  QKV_CHECK_ARG((reinterpret_cast<uintptr_t>(local) & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0,
                "qkv_peer_allgather: local and out must be 4-byte aligned");
  PeerGatherArgs a{};
  a.local = static_cast<const uint32_t*>(local);
  const size_t recv = recv_bytes(slice_bytes_max, world);
  for (int r = 0; r < world; ++r) {
    QKV_CHECK_ARG(buffers[r] != nullptr, "qkv_peer_allgather: null peer buffer");
    a.recv[r] = static_cast<uint2*>(buffers[r]);
  }
  a.ctl = reinterpret_cast<uint32_t*>(static_cast<char*>(buffers[rank]) + recv);
  a.out = static_cast<uint32_t*>(out);
  a.batch = batch;
  a.row_words = row_bytes / 4;
  a.slice_words = slice_bytes_max / 4;
  a.rank = rank;
  a.world = world;
  a.err = device_error_ptr();
  const int64_t work = batch * a.row_words * (world > 1 ? world - 1 : 1);
  int blocks = static_cast<int>((work + 255) / 256);
  blocks = blocks < 1 ? 1 : (blocks > 128 ? 128 : blocks);
  peer_gather_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  QKV_CHECK_LAUNCH("peer_gather_kernel");
  return QKV_OK;
}

}  // extern "C"
