// Geometry-general paged decode kernels (CUDA cores, fp32 math) and the
// split-KV combine kernel.
//
// These kernels serve every geometry the reference accepts (head_size <= 256,
// gqa <= 16, any block/group size). They dequantise each element exactly the
// way the reference's dequantise-then-attend path does before its attention
// call, so their output is the reference result up to fp32 summation order:
//   INT8: k = bf16(code * aq)  (methods/int8_dynamic/attention_backend.py:398-403)
//   KIVI: k = bf16(code * scale + mn), mul and add rounded separately
//         (ops/kivi_gather.py:110-136, cast to the query dtype at :150-156);
//         residual positions read the bf16 window
//         (methods/kivi_int4/attention_backend.py:889-935).
// The production geometries run the tensor-core kernels in decode_mma.cu.
#include <math_constants.h>

#include "decode_common.cuh"

namespace qkv {
namespace {

constexpr int kGenThreads = 128;
constexpr int kGenChunk = 128;  // positions per softmax step (one per thread)
constexpr int kGenMaxG = 16;
#define kNegInf (-CUDART_INF_F)

__device__ __forceinline__ float int8_dequant(int8_t code, float aq) {
  return bf16_round(__fmul_rn(static_cast<float>(code), aq));
}

__device__ __forceinline__ float kivi_dequant(uint32_t code, float scale,
                                              float mn) {
  return bf16_round(__fadd_rn(__fmul_rn(static_cast<float>(code), scale), mn));
}

template <int MODE>
__global__ void __launch_bounds__(kGenThreads)
decode_generic_kernel(const DecodeParams p) {
  constexpr bool KIVI = MODE == kKiviPages;
  constexpr bool DENSE = MODE == kDense;
  extern __shared__ float smem[];
  const int G = p.gqa, D = p.head_size;
  float* qs = smem;                    // [G][D]   q * scale * log2(e)
  float* sc = qs + G * D;              // [G][kGenChunk] scores, then probs
  float* st_m = sc + G * kGenChunk;    // [G] running max (log2 units)
  float* st_l = st_m + G;              // [G] running sum
  float* st_a = st_l + G;              // [G] rescale factor of this step

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int L;
  int64_t kv_base = 0;  // first dense K/V row of this query's request
  if constexpr (DENSE) {
    // query row b -> request: the last r with cu_q[r] <= b
    int lo = 0, hi = p.num_reqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cu_q[mid] <= b) lo = mid; else hi = mid - 1;
    }
    const int q_len = p.cu_q[lo + 1] - p.cu_q[lo];
    const int kv_len = p.cu_k[lo + 1] - p.cu_k[lo];
    kv_base = p.cu_k[lo];
    L = p.causal ? kv_len - q_len + (b - p.cu_q[lo]) + 1 : kv_len;
    L = max(min(L, kv_len), 0);
  } else {
    L = max(p.seq_lens[b], 0);
  }
  const TailState ts = KIVI ? load_tail_state(p, b, L) : TailState{-1, 0, L, 0, L, L};
  const int lk = ts.k_begin;  // first position whose key is in the window
  const int lv = ts.v_begin;  // first position whose value is in the window
  const int body_end = min(lk, lv);
  int t0, t1;
  bool tail = false;
  if (split < p.num_hist_splits) {
    t0 = split * p.split_tokens;
    t1 = min(body_end, t0 + p.split_tokens);
  } else {
    t0 = body_end;
    t1 = L;
    tail = true;
  }

  const __nv_bfloat16* qrow = p.q + static_cast<int64_t>(b) * p.q_stride +
                              static_cast<int64_t>(h) * G * D;
  for (int i = tid; i < G * D; i += kGenThreads)
    qs[i] = __bfloat162float(qrow[i]) * p.scale_log2;
  if (tid < G) {
    st_m[tid] = kNegInf;
    st_l[tid] = 0.0f;
  }
  float acc[kGenMaxG][2];
#pragma unroll
  for (int j = 0; j < kGenMaxG; ++j) acc[j][0] = acc[j][1] = 0.0f;
  __syncthreads();

  const int64_t kvh = p.kvh;
  for (int c = t0; c < t1; c += kGenChunk) {
    // ---- scores: one position per thread
    const int t = c + tid;
    float dots[kGenMaxG];
#pragma unroll
    for (int j = 0; j < kGenMaxG; ++j) dots[j] = 0.0f;
    bool valid = t < t1;
    if (valid) {
      if constexpr (DENSE) {
        const __nv_bfloat16* kr = p.dk + ((kv_base + t) * kvh + h) * D;
        for (int d = 0; d < D; ++d) {
          const float kd = __bfloat162float(kr[d]);
#pragma unroll
          for (int j = 0; j < kGenMaxG; ++j)
            if (j < G) dots[j] += qs[j * D + d] * kd;
        }
      } else if (KIVI && tail && t >= lk) {
        const int laneR = (ts.k_start + (t - lk)) % p.res_cap;
        const __nv_bfloat16* kr =
            p.rk + ((static_cast<int64_t>(ts.row) * p.res_cap + laneR) * kvh + h) * D;
        for (int d = 0; d < D; ++d) {
          const float kd = __bfloat162float(kr[d]);
#pragma unroll
          for (int j = 0; j < kGenMaxG; ++j)
            if (j < G) dots[j] += qs[j * D + d] * kd;
        }
      } else {
        const int64_t page = page_of(p, b, t);
        if (page < 0) {
          valid = false;
        } else {
          const int off = t % p.blk;
          if constexpr (KIVI) {
            const int wpb = p.blk >> 3;      // words per channel per page
            const int gpb = p.blk / p.group;  // key groups per page
            const int64_t chan0 = (page * kvh + h) * D;
            for (int d = 0; d < D; ++d) {
              const int64_t chan = chan0 + d;
              const uint32_t w = static_cast<uint32_t>(p.kq[chan * wpb + (off >> 3)]);
              const uint32_t code = (w >> (4 * (off & 7))) & 0xFu;
              const int64_t si = chan * gpb + off / p.group;
              const float kd = kivi_dequant(code, p.ks[si], p.km[si]);
#pragma unroll
              for (int j = 0; j < kGenMaxG; ++j)
                if (j < G) dots[j] += qs[j * D + d] * kd;
            }
          } else {
            const int8_t* kr = p.kc + ((page * p.blk + off) * kvh + h) * D;
            const __nv_bfloat16* aq = p.k_aq + static_cast<int64_t>(h) * D;
            for (int d = 0; d < D; ++d) {
              const float kd = int8_dequant(kr[d], __bfloat162float(aq[d]));
#pragma unroll
              for (int j = 0; j < kGenMaxG; ++j)
                if (j < G) dots[j] += qs[j * D + d] * kd;
            }
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kGenMaxG; ++j)
      if (j < G) sc[j * kGenChunk + tid] = valid ? dots[j] : kNegInf;
    __syncthreads();

    // ---- online softmax update, one warp per head
    for (int j = warp; j < G; j += kGenThreads / 32) {
      float v[kGenChunk / 32];
      float mx = kNegInf;
#pragma unroll
      for (int i = 0; i < kGenChunk / 32; ++i) {
        v[i] = sc[j * kGenChunk + lane * (kGenChunk / 32) + i];
        mx = fmaxf(mx, v[i]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = st_m[j];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < kGenChunk / 32; ++i) {
        const float pr = (v[i] == kNegInf) ? 0.0f : exp2f(v[i] - m_new);
        sc[j * kGenChunk + lane * (kGenChunk / 32) + i] = pr;
        sum += pr;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float alpha =
            (m_new == kNegInf) ? 1.0f : (m_old == kNegInf ? 0.0f : exp2f(m_old - m_new));
        st_m[j] = m_new;
        st_l[j] = st_l[j] * alpha + sum;
        st_a[j] = alpha;
      }
    }
    __syncthreads();

    // ---- P @ V: thread owns channels tid and tid + 128
    const int n = min(kGenChunk, t1 - c);
#pragma unroll
    for (int dd = 0; dd < 2; ++dd) {
      const int d = tid + dd * kGenThreads;
      if (d >= D) break;
#pragma unroll
      for (int j = 0; j < kGenMaxG; ++j)
        if (j < G) acc[j][dd] *= st_a[j];
      for (int tt = 0; tt < n; ++tt) {
        const int pos = c + tt;
        float vd = 0.0f;
        if constexpr (DENSE) {
          vd = __bfloat162float(p.dv[((kv_base + pos) * kvh + h) * D + d]);
        } else if (KIVI && tail && pos >= lv) {
          const int laneR = (ts.v_start + (pos - lv)) % p.res_cap;
          vd = __bfloat162float(
              p.rv[((static_cast<int64_t>(ts.row) * p.res_cap + laneR) * kvh + h) * D + d]);
        } else {
          const int64_t page = page_of(p, b, pos);
          if (page >= 0) {
            const int off = pos % p.blk;
            const int64_t row = (page * p.blk + off) * kvh + h;
            if constexpr (KIVI) {
              const uint32_t w = static_cast<uint32_t>(p.vq[row * (D >> 3) + (d >> 3)]);
              const uint32_t code = (w >> (4 * (d & 7))) & 0xFu;
              const int64_t si = row * (D / p.group) + d / p.group;
              vd = kivi_dequant(code, p.vs[si], p.vm[si]);
            } else {
              vd = int8_dequant(p.vc[row * D + d],
                                __bfloat162float(p.v_aq[static_cast<int64_t>(h) * D + d]));
            }
          }
        }
#pragma unroll
        for (int j = 0; j < kGenMaxG; ++j)
          if (j < G) acc[j][dd] += sc[j * kGenChunk + tt] * vd;
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int dd = 0; dd < 2; ++dd) {
    const int d = tid + dd * kGenThreads;
    if (d >= D) break;
#pragma unroll
    for (int j = 0; j < kGenMaxG; ++j)
      if (j < G) store_partial(p, b, h * G + j, split, d, acc[j][dd], st_m[j], st_l[j]);
  }
}

// grid (num_heads, batch), one thread per channel.
__global__ void combine_kernel(const DecodeParams p) {
  const int hq = blockIdx.x, b = blockIdx.y;
  const int S = p.splits_total;
  const int64_t row0 = (static_cast<int64_t>(b) * p.num_heads + hq) * S;
  float M = kNegInf;
  for (int s = 0; s < S; ++s) M = fmaxf(M, p.ws_ml[(row0 + s) * 2]);
  for (int d = threadIdx.x; d < p.head_size; d += blockDim.x) {
    float num = 0.0f, den = 0.0f;
    if (M != kNegInf) {
      for (int s = 0; s < S; ++s) {
        const float m = p.ws_ml[(row0 + s) * 2];
        if (m == kNegInf) continue;
        const float w = exp2f(m - M);
        num += w * p.ws_acc[(row0 + s) * p.head_size + d];
        den += w * p.ws_ml[(row0 + s) * 2 + 1];
      }
    }
    p.out[static_cast<int64_t>(b) * p.out_stride +
          static_cast<int64_t>(hq) * p.head_size + d] =
        __float2bfloat16_rn(den > 0.0f ? num / den : 0.0f);
  }
}

}  // namespace

void launch_combine(const DecodeParams& p, cudaStream_t stream) {
  dim3 grid(p.num_heads, p.batch);
  const int threads = p.head_size < 128 ? 128 : (p.head_size > 256 ? 256 : p.head_size);
  combine_kernel<<<grid, threads, 0, stream>>>(p);
}

size_t generic_smem_bytes(int gqa, int head_size) {
  return static_cast<size_t>(gqa * head_size + gqa * kGenChunk + 3 * gqa) *
         sizeof(float);
}

int launch_decode_generic(const DecodeParams& p, int mode,
                          cudaStream_t stream) {
  if (p.gqa > kGenMaxG || p.head_size > 2 * kGenThreads)
    return set_error(QKV_ERR_UNSUPPORTED,
                     "paged decode: gqa must be <= 16 and head_size <= 256");
  dim3 grid(p.splits_total, p.kvh, p.batch);
  const size_t smem = generic_smem_bytes(p.gqa, p.head_size);
  if (mode == kKiviPages)
    decode_generic_kernel<kKiviPages><<<grid, kGenThreads, smem, stream>>>(p);
  else if (mode == kInt8Pages)
    decode_generic_kernel<kInt8Pages><<<grid, kGenThreads, smem, stream>>>(p);
  else
    decode_generic_kernel<kDense><<<grid, kGenThreads, smem, stream>>>(p);
  QKV_CHECK_LAUNCH("decode_generic_kernel");
  if (p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
