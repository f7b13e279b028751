// All-gather of the per-rank attention outputs over NVLink peer memory: the
// one exchange of the KV-head-sharded path (rank i computes query heads
// [Hq i/N, Hq (i+1)/N) of every request). Replaces the NCCL all-gather plus
// the head permute that follows it with one kernel that writes the final
// [B, Hq, D] layout.
//
// Protocol (one round, no barrier, no fence): every 4-byte word of a rank's
// slice travels to each peer together with the call's epoch as ONE 64-bit
// scalar (epoch << 32 | data), written with one st.relaxed.sys.u64 into the
// peer's receive buffer; a receiver polls the word with ld.relaxed.sys.u64
// until its high half equals the epoch, and its low half is then the data of
// the same store. An aligned 64-bit scalar access is a single access in the
// PTX memory model, so the epoch is never seen beside a stale data half (a
// vector access, v2.u32, would be two accesses of unspecified order). Receive buffers are
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

#include <math_constants.h>

#include "decode_common.cuh"

namespace qkv {

namespace {

constexpr int kMaxPeers = 8;
constexpr int kCtlBytes = 64;
constexpr long long kPeerWaitCycles = 2000000000LL;  // ~1 s at 2 GHz

struct PeerGatherArgs {
  const uint32_t* local;       // [B, row_words] this rank's slice
  unsigned long long* recv[kMaxPeers];  // each rank's receive words (as mapped here)
  const unsigned long long* own;        // recv[rank], passed on its own (no dynamic index)
  uint32_t* ctl;               // this rank's control words
  uint32_t* out;               // [B, world * row_words] on this rank
  int64_t batch, row_words;    // row_words = Hq/N * D * 2 / 4
  int64_t slice_words;         // receive words per (parity, source rank)
  int rank, world;
  int* err;
};

// One receive word: data in the low 32 bits, the call's epoch in the high 32.
__device__ __forceinline__ void store_word(unsigned long long* p, uint32_t data, uint32_t flag) {
  const unsigned long long w = (static_cast<unsigned long long>(flag) << 32) | data;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long load_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t word_flag(unsigned long long v) { return static_cast<uint32_t>(v >> 32); }
__device__ __forceinline__ uint32_t word_data(unsigned long long v) { return static_cast<uint32_t>(v); }

// The call's epoch (read by thread 0 of every CTA before any CTA of the call
// can advance it; a call starts after the previous one ended).
__device__ __forceinline__ uint32_t call_epoch(const PeerGatherArgs& a) {
  __shared__ uint32_t epoch_sh;
  if (threadIdx.x == 0) epoch_sh = *reinterpret_cast<volatile uint32_t*>(a.ctl) + 1;
  __syncthreads();
  return epoch_sh;
}

// Word i of this rank's slice: into its own output and to every peer.
__device__ __forceinline__ void send_word(const PeerGatherArgs& a, uint32_t e, int64_t i, uint32_t d) {
  const int par = static_cast<int>(e & 1u);
  const int64_t b = i / a.row_words, w = i - b * a.row_words;
  a.out[b * static_cast<int64_t>(a.world) * a.row_words + a.rank * a.row_words + w] = d;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r)
    if (r < a.world && r != a.rank)
      store_word(a.recv[r] + (static_cast<int64_t>(par) * a.world + a.rank) * a.slice_words + i, d, e);
}

// Receives every peer's words of call e (polled until they carry e) into the
// output, then the last CTA of the call advances the epoch.
__device__ void receive_and_finish(const PeerGatherArgs& a, uint32_t e) {
  __shared__ int last;
  const int par = static_cast<int>(e & 1u);
  const int64_t n = a.batch * a.row_words;
  const int64_t full_row = static_cast<int64_t>(a.world) * a.row_words;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const unsigned long long* mine = a.own + static_cast<int64_t>(par) * a.world * a.slice_words;
  const long long start = clock64();
  bool ok = true;
  for (int64_t j = t0; j < (a.world - 1) * n && ok; j += stride) {
    const int64_t k = j / n, i = j - k * n;
    const int src = static_cast<int>(k) + (static_cast<int>(k) >= a.rank ? 1 : 0);
    const unsigned long long* p = mine + static_cast<int64_t>(src) * a.slice_words + i;
    unsigned long long v = load_word(p);
    while (word_flag(v) != e) {
      if (clock64() - start > kPeerWaitCycles) {
        ok = false;
        break;
      }
      __nanosleep(32);
      v = load_word(p);
    }
    if (!ok) break;
    const int64_t b = i / a.row_words, w = i - b * a.row_words;
    a.out[b * full_row + src * a.row_words + w] = word_data(v);
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

__global__ void __launch_bounds__(256) peer_gather_kernel(const PeerGatherArgs a) {
  const uint32_t e = call_epoch(a);
  const int64_t n = a.batch * a.row_words;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    send_word(a, e, i, a.local[i]);
  receive_and_finish(a, e);
}

// Split partials of the decode kernel on this rank: [B, Hq/N, S, D] sums and
// [B, Hq/N, S, 2] (max, sum) pairs.
struct Partials {
  const float* acc;
  const float* ml;
  int splits, head_size;
};

constexpr int kCombineWeights = 128;  // splits whose weights one warp stages

// Combine + all-gather: warp per (request, head) row merges the row's splits
// with exactly combine_kernel's arithmetic (max over splits, then in split
// order num += w acc, den += w l with w = exp2(m - max), out = num / den),
// packs bf16 pairs and sends them; then receives as above.
__global__ void __launch_bounds__(256) peer_combine_gather_kernel(const PeerGatherArgs a, const Partials pt) {
  __shared__ float wts[8][kCombineWeights];
  const uint32_t e = call_epoch(a);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = pt.splits, D = pt.head_size;
  const int pairs = D / 2;  // 4-byte words per row (row_words)
  const int64_t rows = a.batch * (a.row_words / pairs);
  const int64_t wstride = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows; row += wstride) {
    const float* ml = pt.ml + row * S * 2;
    const float* acc = pt.acc + row * S * D;
    float M = -CUDART_INF_F;
    for (int s = lane; s < S; s += 32) M = fmaxf(M, ml[2 * s]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const bool staged = S <= kCombineWeights;
    if (staged)
      for (int s = lane; s < S; s += 32) {
        const float m = ml[2 * s];
        wts[warp][s] = (M == -CUDART_INF_F || m == -CUDART_INF_F) ? 0.0f : exp2f(m - M);
      }
    __syncwarp();
    for (int wi = lane; wi < pairs; wi += 32) {
      float n0 = 0.0f, n1 = 0.0f, den = 0.0f;
      if (M != -CUDART_INF_F) {
        int s = 0;
        if (staged) {
          // 4 splits' loads in flight, then the FMAs in split order
          for (; s + 4 <= S; s += 4) {
            float2 v[4];
            float l[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              v[k] = *reinterpret_cast<const float2*>(acc + static_cast<int64_t>(s + k) * D + 2 * wi);
              l[k] = ml[2 * (s + k) + 1];
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float w = wts[warp][s + k];
              if (w == 0.0f && ml[2 * (s + k)] == -CUDART_INF_F) continue;
              n0 = fmaf(w, v[k].x, n0);
              n1 = fmaf(w, v[k].y, n1);
              den = fmaf(w, l[k], den);
            }
          }
        }
        for (; s < S; ++s) {
          const float m = ml[2 * s];
          if (m == -CUDART_INF_F) continue;
          const float w = staged ? wts[warp][s] : exp2f(m - M);
          const float2 v = *reinterpret_cast<const float2*>(acc + static_cast<int64_t>(s) * D + 2 * wi);
          n0 = fmaf(w, v.x, n0);
          n1 = fmaf(w, v.y, n1);
          den = fmaf(w, ml[2 * s + 1], den);
        }
      }
      const __nv_bfloat162 h = __floats2bfloat162_rn(den > 0.0f ? n0 / den : 0.0f, den > 0.0f ? n1 / den : 0.0f);
      send_word(a, e, row * pairs + wi, *reinterpret_cast<const uint32_t*>(&h));
    }
    __syncwarp();
  }
  receive_and_finish(a, e);
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
    a.recv[r] = static_cast<unsigned long long*>(buffers[r]);
  }
  a.ctl = reinterpret_cast<uint32_t*>(static_cast<char*>(buffers[rank]) + recv);
  a.own = a.recv[rank];
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

int qkv_peer_combine_allgather(const float* partial_acc, const float* partial_ml, int splits, int64_t batch,
                               int local_heads, int head_size, const void* local, void* const* buffers,
                               int64_t slice_bytes_max, void* out, int rank, int world, qkv_stream_t stream) {
  using namespace qkv;
  QKV_CHECK_ARG(local_heads > 0 && head_size > 0 && head_size % 2 == 0, "qkv_peer_combine_allgather: bad head sizes");
  const int64_t row_bytes = static_cast<int64_t>(local_heads) * head_size * 2;
  if (splits <= 1)  // the decode wrote its output itself
    return qkv_peer_allgather(local, batch, row_bytes, buffers, slice_bytes_max, out, rank, world, stream);
  QKV_CHECK_ARG(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
                "qkv_peer_combine_allgather: world must be 1..8 and rank inside it");
  QKV_CHECK_ARG(batch >= 0 && batch * row_bytes <= slice_bytes_max,
                "qkv_peer_combine_allgather: the slice does not fit the peer buffers");
  QKV_CHECK_ARG(partial_acc != nullptr && partial_ml != nullptr && buffers != nullptr && out != nullptr,
                "qkv_peer_combine_allgather: null pointer");
  QKV_CHECK_ARG((reinterpret_cast<uintptr_t>(partial_acc) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0,
                "qkv_peer_combine_allgather: misaligned partials or output");
  PeerGatherArgs a{};
  const size_t recv = recv_bytes(slice_bytes_max, world);
  for (int r = 0; r < world; ++r) {
    QKV_CHECK_ARG(buffers[r] != nullptr, "qkv_peer_combine_allgather: null peer buffer");
    a.recv[r] = static_cast<unsigned long long*>(buffers[r]);
  }
  a.ctl = reinterpret_cast<uint32_t*>(static_cast<char*>(buffers[rank]) + recv);
  a.own = a.recv[rank];
  a.out = static_cast<uint32_t*>(out);
  a.batch = batch;
  a.row_words = row_bytes / 4;
  a.slice_words = slice_bytes_max / 4;
  a.rank = rank;
  a.world = world;
  a.err = device_error_ptr();
  const Partials pt{partial_acc, partial_ml, splits, head_size};
  const int64_t rows = batch * local_heads;
  const int64_t recv_work = batch * a.row_words * (world - 1);
  int64_t blocks = (rows + 7) / 8;
  const int64_t rb = (recv_work + 255) / 256;
  if (rb > blocks) blocks = rb;
  blocks = blocks < 1 ? 1 : (blocks > 128 ? 128 : blocks);
  peer_combine_gather_kernel<<<static_cast<int>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, pt);
  QKV_CHECK_LAUNCH("peer_combine_gather_kernel");
  return QKV_OK;
}

}  // extern "C"
