// Geometry-general paged decode kernels (CUDA cores, fp32 math) and the
// split-KV combine kernel.
//
// These kernels serve every geometry the reference accepts (head_size <= 256,
// gqa <= 16, any block/group size). They dequantise each element with the
// reference's fp32 arithmetic of its dequantise-then-attend path:
//   INT8: k = code * aq  (methods/int8_dynamic/attention_backend.py:398-403)
//   KIVI: k = code * scale + mn, mul and add rounded separately
//         (ops/kivi_gather.py:110-136);
//         residual positions read the bf16 window
//         (methods/kivi_int4/attention_backend.py:889-935).
// The production geometries run the page-pipelined tensor-core kernels of
// decode_kivi_tma.cu, decode_int8_tma.cu and decode_fp8_tma.cu.
#include <math_constants.h>

#include <atomic>

#include <cuda_fp8.h>

#include "decode_common.cuh"

namespace qkv {
namespace {

constexpr int kGenThreads = 128;
constexpr int kGenChunk = 128;  // positions per softmax step (one per thread)
constexpr int kGenMaxG = 16;
#define kNegInf (-CUDART_INF_F)

// INT8: the reference's dense dequantisation, code.to(bf16) * aq in bf16
// (methods/int8_dynamic/attention_backend.py:398-401): the exact product
// rounded once to bf16, as the page-pipelined INT8 kernel computes it.
__device__ __forceinline__ float int8_dequant(int8_t code, float aq) {
  return __bfloat162float(__float2bfloat16_rn(__fmul_rn(static_cast<float>(code), aq)));
}

// KIVI: code * scale + min in fp32 (ops/kivi_gather.py), before the
// reference's cast to the query dtype (the page-pipelined KIVI kernel also
// uses these values unrounded).
__device__ __forceinline__ float kivi_dequant(uint32_t code, float scale,
                                              float mn) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), scale), mn);
}

// Stages rows [c, c + n) of K (IS_K) or V into tile[r][d] (fp32): one warp per
// row, the row's source (residual window, dense K/V or a page) resolved once;
// bf16 rows are read with 16-byte loads.
template <int MODE, bool IS_K>
__device__ __forceinline__ void stage_rows(float* tile, int ld, const DecodeParams& p, const TailState& ts,
                                           int b, int h, int64_t kv_base, bool tail, int c, int n,
                                           int warp, int lane) {
  const int D = p.head_size;
  const int64_t kvh = p.kvh;
  for (int r = warp; r < n; r += kGenThreads / 32) {
    const int pos = c + r;
    float* dst = tile + r * ld;
    const __nv_bfloat16* row16 = nullptr;
    if constexpr (MODE == kDense) {
      row16 = (IS_K ? p.dk : p.dv) + ((kv_base + pos) * kvh + h) * D;
    } else if (MODE == kKiviPages && tail && pos >= (IS_K ? ts.k_begin : ts.v_begin)) {
      const int start = IS_K ? ts.k_start : ts.v_start;
      const int begin = IS_K ? ts.k_begin : ts.v_begin;
      const int laneR = (start + (pos - begin)) % p.res_cap;
      row16 = (IS_K ? p.rk : p.rv) + ((static_cast<int64_t>(ts.row) * p.res_cap + laneR) * kvh + h) * D;
    }
    if (row16 != nullptr) {
      if ((D & 7) == 0 && (reinterpret_cast<uintptr_t>(row16) & 15u) == 0) {
        for (int i = lane; i < D / 8; i += 32) {
          const uint4 raw = reinterpret_cast<const uint4*>(row16)[i];
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(h2[k]);
            dst[8 * i + 2 * k] = f.x;
            dst[8 * i + 2 * k + 1] = f.y;
          }
        }
      } else {
        for (int d = lane; d < D; d += 32) dst[d] = __bfloat162float(row16[d]);
      }
      continue;
    }
    if constexpr (MODE != kDense) {
      int64_t page = -1;
      if (lane == 0) page = page_of(p, b, pos);
      page = __shfl_sync(0xffffffffu, page, 0);
      if (page < 0) {
        for (int d = lane; d < D; d += 32) dst[d] = 0.0f;
        continue;
      }
      const int off = pos % p.blk;
      if constexpr (MODE == kKiviPages) {
        if (IS_K) {
          const int64_t chan0 = (page * kvh + h) * D;
          for (int d = lane; d < D; d += 32) {
            const int64_t chan = chan0 + d;
            const uint32_t w = static_cast<uint32_t>(p.kq[chan * (p.blk >> 3) + (off >> 3)]);
            const int64_t si = chan * (p.blk / p.group) + off / p.group;
            dst[d] = kivi_dequant((w >> (4 * (off & 7))) & 0xFu, p.ks[si], p.km[si]);
          }
        } else {
          const int64_t vrow = (page * p.blk + off) * kvh + h;
          for (int d = lane; d < D; d += 32) {
            const uint32_t w = static_cast<uint32_t>(p.vq[vrow * (D >> 3) + (d >> 3)]);
            const int64_t si = vrow * (D / p.group) + d / p.group;
            dst[d] = kivi_dequant((w >> (4 * (d & 7))) & 0xFu, p.vs[si], p.vm[si]);
          }
        }
      } else if constexpr (MODE == kFp8Pages) {
        // E4M3 codes [NB, blk, KVH, D] and one fp32 scale per (token, head)
        const int64_t rowi = (page * p.blk + off) * kvh + h;
        const uint8_t* row8 = reinterpret_cast<const uint8_t*>(IS_K ? p.kc : p.vc) + rowi * D;
        const float sc8 = (IS_K ? p.ks : p.vs)[rowi];
        for (int d = lane; d < D; d += 32) {
          const __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(row8[d]), __NV_E4M3);
          dst[d] = __fmul_rn(__half2float(__half(hr)), sc8);
        }
      } else {
        const int8_t* row8 = (IS_K ? p.kc : p.vc) + ((page * p.blk + off) * kvh + h) * D;
        const __nv_bfloat16* aq = (IS_K ? p.k_aq : p.v_aq) + static_cast<int64_t>(h) * D;
        for (int d = lane; d < D; d += 32) dst[d] = int8_dequant(row8[d], __bfloat162float(aq[d]));
      }
    }
  }
}

// One CTA per (split, kv head, query row). Each step stages 128 positions of
// dequantised K (then V) in shared memory with coalesced loads, a padded row
// stride keeping the per-position dot products conflict-free.
template <int MODE>
__global__ void __launch_bounds__(kGenThreads)
decode_generic_kernel(const DecodeParams p) {
  constexpr bool KIVI = MODE == kKiviPages;
  constexpr bool DENSE = MODE == kDense;
  extern __shared__ float smem[];
  const int G = p.gqa, D = p.head_size;
  const int ld = D + 1;                // padded row stride of the K/V tile
  float* tile = smem;                  // [kGenChunk][D + 1]
  float* qs = tile + kGenChunk * ld;   // [G][D]   q * scale * log2(e)
  float* sc = qs + G * D;              // [G][kGenChunk] scores, then probs
  float* st_m = sc + G * kGenChunk;    // [G] running max (log2 units)
  float* st_l = st_m + G;              // [G] running sum
  float* st_a = st_l + G;              // [G] rescale factor of this step

  const int split = blockIdx.x + p.split_base, h = blockIdx.y, b = blockIdx.z;
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
  const int body_end = min(ts.k_begin, ts.v_begin);
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

  for (int c = t0; c < t1; c += kGenChunk) {
    const int n = min(kGenChunk, t1 - c);
    // ---- stage K rows of positions c .. c+n-1 (thread -> channel)
    stage_rows<MODE, true>(tile, ld, p, ts, b, h, kv_base, tail, c, n, warp, lane);
    __syncthreads();
    // ---- scores: one position per thread
    float dots[kGenMaxG];
#pragma unroll
    for (int j = 0; j < kGenMaxG; ++j) dots[j] = 0.0f;
    const bool valid = tid < n;
    if (valid) {
      const float* kr = tile + tid * ld;
      for (int d = 0; d < D; ++d) {
        const float kd = kr[d];
#pragma unroll
        for (int j = 0; j < kGenMaxG; ++j)
          if (j < G) dots[j] = fmaf(qs[j * D + d], kd, dots[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kGenMaxG; ++j)
      if (j < G) sc[j * kGenChunk + tid] = valid ? dots[j] : kNegInf;
    __syncthreads();

    // ---- online softmax update, one warp per head; V staged meanwhile
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
    stage_rows<MODE, false>(tile, ld, p, ts, b, h, kv_base, tail, c, n, warp, lane);
    __syncthreads();

    // ---- P @ V: thread owns channels tid and tid + 128
#pragma unroll
    for (int dd = 0; dd < 2; ++dd) {
      const int d = tid + dd * kGenThreads;
      if (d >= D) break;
#pragma unroll
      for (int j = 0; j < kGenMaxG; ++j)
        if (j < G) acc[j][dd] *= st_a[j];
      for (int tt = 0; tt < n; ++tt) {
        const float vd = tile[tt * ld + d];
#pragma unroll
        for (int j = 0; j < kGenMaxG; ++j)
          if (j < G) acc[j][dd] = fmaf(sc[j * kGenChunk + tt], vd, acc[j][dd]);
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

// Warp per (request, head) row, 8 rows per CTA. The lanes read the row's
// (max, sum) pairs together and stage the split weights w = exp2(m - max) in
// shared memory; lane l then merges dims 4 l + 128 k .. + 3 with the
// partials of 8 splits in flight, in split order: num += w acc, den += w l,
// out = num / den (splits with m = -inf are skipped: their partial sums may
// never have been written). kVec: 16-byte loads of the partial sums (the
// workspace 16-byte aligned).
constexpr int kCombineRows = 8;
constexpr int kCombineStaged = 128;  // splits whose weights a warp stages
template <bool kVec>
__global__ void __launch_bounds__(kCombineRows * 32) combine_kernel(const DecodeParams p) {
  __shared__ float wts[kCombineRows][kCombineStaged];
  grid_dependency_wait();  // launched behind the decode that wrote the partials
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kCombineRows + warp;
  if (row >= static_cast<int64_t>(p.batch) * p.num_heads) return;
  const int b = static_cast<int>(row / p.num_heads), hq = static_cast<int>(row % p.num_heads);
  const int S = p.splits_total, D = p.head_size;
  const float* ml = p.ws_ml + row * S * 2;
  const float* acc = p.ws_acc + row * S * D;
  float M = kNegInf;
  for (int s = lane; s < S; s += 32) M = fmaxf(M, ml[2 * s]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  const bool staged = S <= kCombineStaged;
  if (staged)
    for (int s = lane; s < S; s += 32) {
      const float m = ml[2 * s];
      wts[warp][s] = (M == kNegInf || m == kNegInf) ? 0.0f : exp2f(m - M);
    }
  __syncwarp();
  __nv_bfloat16* out = p.out + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(hq) * D;
  for (int d0 = 4 * lane; d0 < D; d0 += 128) {
    float num[4] = {0.0f, 0.0f, 0.0f, 0.0f}, den = 0.0f;
    if (M != kNegInf) {
      for (int s0 = 0; s0 < S; s0 += 8) {
        float4 v[8];
        float l[8], m[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int s = s0 + k < S ? s0 + k : S - 1;  // in range: the extra lanes of the batch are unused
          m[k] = ml[2 * s];
          l[k] = ml[2 * s + 1];
          const float* a = acc + static_cast<int64_t>(s) * D + d0;
          v[k] = kVec ? *reinterpret_cast<const float4*>(a) : make_float4(a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (s0 + k >= S || m[k] == kNegInf) continue;
          const float w = staged ? wts[warp][s0 + k] : exp2f(m[k] - M);
          num[0] = fmaf(w, v[k].x, num[0]);
          num[1] = fmaf(w, v[k].y, num[1]);
          num[2] = fmaf(w, v[k].z, num[2]);
          num[3] = fmaf(w, v[k].w, num[3]);
          den = fmaf(w, l[k], den);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) out[d0 + k] = __float2bfloat16_rn(den > 0.0f ? num[k] / den : 0.0f);
  }
}

}  // namespace

// head_size is a multiple of 8 on every decode entry point, so a 16-byte
// aligned workspace gives 16-byte aligned partial rows.
void launch_combine(const DecodeParams& p, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(p.batch) * p.num_heads;
  const unsigned grid = static_cast<unsigned>((rows + kCombineRows - 1) / kCombineRows);
  // a programmatic dependent launch: the combine's launch overlaps the end
  // of the decode it follows, and its CTAs wait for that decode
  // (a failed launch shows in the callers' launch check)
  PdlConfig c(dim3(grid), dim3(kCombineRows * 32), 0, stream, true);
  if ((reinterpret_cast<uintptr_t>(p.ws_acc) & 15u) == 0)
    (void)cudaLaunchKernelEx(&c.cfg, combine_kernel<true>, p);
  else
    (void)cudaLaunchKernelEx(&c.cfg, combine_kernel<false>, p);
}

size_t generic_smem_bytes(int gqa, int head_size) {
  return static_cast<size_t>(kGenChunk * (head_size + 1) + gqa * head_size +
                             gqa * kGenChunk + 3 * gqa) *
         sizeof(float);
}

// Opts every instantiation into more than 48 KB of dynamic shared memory,
// once per device.
int ensure_generic_smem(int mode, size_t bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << ((4 * dev + mode) & 63);
  if (done.load() & bit) return QKV_OK;
  cudaError_t e;
  const int limit = 160 * 1024;
  if (mode == kKiviPages)
    e = cudaFuncSetAttribute(decode_generic_kernel<kKiviPages>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
  else if (mode == kFp8Pages)
    e = cudaFuncSetAttribute(decode_generic_kernel<kFp8Pages>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
  else if (mode == kInt8Pages)
    e = cudaFuncSetAttribute(decode_generic_kernel<kInt8Pages>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
  else
    e = cudaFuncSetAttribute(decode_generic_kernel<kDense>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(decode_generic_kernel)");
  (void)bytes;
  done.fetch_or(bit);
  return QKV_OK;
}

// Runs splits [p.split_base, p.split_base + num_splits) of the plan; the
// combine kernel runs when `combine` is set and the plan has several splits.
int launch_decode_generic_splits(const DecodeParams& p, int mode, int num_splits,
                                 bool combine, cudaStream_t stream) {
  if (p.gqa > kGenMaxG || p.head_size > 2 * kGenThreads)
    return set_error(QKV_ERR_UNSUPPORTED,
                     "paged decode: gqa must be <= 16 and head_size <= 256");
  dim3 grid(num_splits, p.kvh, p.batch);
  const size_t smem = generic_smem_bytes(p.gqa, p.head_size);
  const int rc = ensure_generic_smem(mode, smem);
  if (rc != QKV_OK) return rc;
  if (mode == kKiviPages)
    decode_generic_kernel<kKiviPages><<<grid, kGenThreads, smem, stream>>>(p);
  else if (mode == kFp8Pages)
    decode_generic_kernel<kFp8Pages><<<grid, kGenThreads, smem, stream>>>(p);
  else if (mode == kInt8Pages)
    decode_generic_kernel<kInt8Pages><<<grid, kGenThreads, smem, stream>>>(p);
  else
    decode_generic_kernel<kDense><<<grid, kGenThreads, smem, stream>>>(p);
  QKV_CHECK_LAUNCH("decode_generic_kernel");
  if (combine && p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

int launch_decode_generic(const DecodeParams& p, int mode, cudaStream_t stream) {
  DecodeParams q = p;
  q.split_base = 0;
  return launch_decode_generic_splits(q, mode, p.splits_total, true, stream);
}

}  // namespace qkv
