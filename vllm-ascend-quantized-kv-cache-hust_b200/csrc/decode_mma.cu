// Tensor-core paged decode over INT8 pages (production geometry: head_size
// 128, page size 128, up to 8 query heads per KV head).
//
// One CTA owns (request, kv head, history split); each of its 8 warps walks
// units of 32 tokens (a quarter page) with a private two-stage cp.async ring
// in shared memory, so every warp keeps one unit in flight while it computes
// the previous one. Per unit the warp computes
//     S^T[token][head] = K[token][channel] . Q'^T[channel][head]
//     O^T[dim][head]  += V^T[dim][token]   . P^T[token][head]
// with mma.sync m16n8k16 (fp16 x fp16 -> fp32); the 8 query heads of the KV
// head are the N dimension. int8 -> fp16 in registers: an xor-bias LOP3 turns
// two signed bytes into the fp16 pair 1152 + c and one HSUB2 removes the 1152
// exactly. The per-channel antiquant scales fold into Q' (keys) and into the
// fp32 output (values), so the dequantised values enter exactly.
#include <math_constants.h>

#include <atomic>

#include "decode_common.cuh"

namespace qkv {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kD = 128;     // head size of the tensor-core path
constexpr int kBlk = 128;   // page size of the tensor-core path
constexpr int kHeads = 8;   // N of the MMA: query heads per KV head (padded)

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                         uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::);
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;\n" ::);
}
__device__ __forceinline__ void cp_async_wait0() {
  asm volatile("cp.async.wait_group 0;\n" ::);
}

// ------------------------------------------------------------ INT8 stage

constexpr int kUnit8 = 32;  // tokens per INT8 unit (a quarter page)

// One INT8 unit: 32 token rows of K and of V (128 bytes each). K rows keep
// their 16-byte chunk c at c ^ (4 * (r & 1)) (each 8-lane phase of the 16-byte
// fragment loads then covers all 8 bank groups) and V rows their word w at
// w ^ (8 * ((r >> 1) & 3)) (the 32 lanes of a 4-byte load hit 32 banks).
struct Int8Stage {
  uint32_t k[kUnit8][32];
  uint32_t v[kUnit8][32];
};
constexpr int kInt8StageBytes = sizeof(Int8Stage);

__device__ __forceinline__ int k8_chunk(int r, int c) { return c ^ ((r & 1) << 2); }
__device__ __forceinline__ int v8_word(int r, int w) { return w ^ (((r >> 1) & 3) << 3); }

// int8 byte pairs (bytes 0 and 2 of x) -> fp16 pair 1152 + c
__device__ __forceinline__ uint32_t i8_pair(uint32_t x) {
  uint32_t y;
  asm("lop3.b32 %0, %1, 0x00FF00FF, 0x64806480, 0x6A;\n" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t hsub2_1152(uint32_t x) {
  uint32_t y;
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(y) : "r"(x), "r"(0x64806480u));
  return y;
}

__device__ __forceinline__ void int8_issue(Int8Stage& st, const DecodeParams& p,
                                           int64_t page, int quarter, int h,
                                           int lane) {
  const int64_t kv = p.kvh;
  const int64_t tok0 = page * kBlk + quarter * kUnit8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane + 32 * i;  // 256 chunks: 32 rows x 8 chunks
    const int r = c >> 3, part = c & 7;
    const int64_t off = ((tok0 + r) * kv + h) * kD + 16 * part;
    cp_async16(&st.k[r][4 * k8_chunk(r, part)], p.kc + off);
    cp_async16(&st.v[r][v8_word(r, 4 * part)], p.vc + off);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
int8_decode_mma_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;
  Int8Stage* stages = reinterpret_cast<Int8Stage*>(smem_raw) + warp * 2;

  const int L = max(p.seq_lens[b], 0);
  const int t0 = split * p.split_tokens;
  const int t1 = min(L, t0 + p.split_tokens);
  const int n_units = t1 > t0 ? (t1 - t0 + kUnit8 - 1) / kUnit8 : 0;

  // ---- Q' = q * k_aq * scale * log2(e) for head g, once per CTA.
  // k-step kk uses word m = 4t + kk (kk < 4) or 16 + 4t + kk - 4 of a row:
  // channels 4m (k 2t), 4m + 2 (k 2t+1), 4m + 1 (k 2t+8), 4m + 3 (k 2t+9)
  uint32_t bq[8][2];
  {
    const __nv_bfloat16* qrow =
        p.q + static_cast<int64_t>(b) * p.q_stride + (static_cast<int64_t>(h) * G + g) * kD;
    const __nv_bfloat16* aq = p.k_aq + static_cast<int64_t>(h) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int m = kk < 4 ? 4 * t + kk : 16 + 4 * t + kk - 4;
      float qq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = 4 * m + i;
        qq[i] = g < G ? __bfloat162float(qrow[ch]) * __bfloat162float(aq[ch]) * p.scale_log2 : 0.0f;
      }
      bq[kk][0] = pack_half2(qq[0], qq[2]);
      bq[kk][1] = pack_half2(qq[1], qq[3]);
    }
  }

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_run[2] = {0.0f, 0.0f};

  int64_t pages[2] = {-1, -1};
  auto issue = [&](int u, int slot) {
    const int pos = t0 + u * kUnit8;
    int64_t pg = -1;
    if (lane == 0) pg = page_of(p, b, pos);
    pg = __shfl_sync(0xffffffffu, pg, 0);
    pages[slot] = pg;
    if (pg >= 0) int8_issue(stages[slot], p, pg, (pos / kUnit8) & 3, h, lane);
    cp_async_commit();
  };

  int it = 0;
  if (warp < n_units) issue(warp, 0);
  for (int u = warp; u < n_units; u += kWarps, ++it) {
    const int slot = it & 1;
    if (u + kWarps < n_units) {
      issue(u + kWarps, slot ^ 1);
    } else {
      cp_async_commit();
    }
    cp_async_wait1();
    __syncwarp();
    if (pages[slot] < 0) {
      __syncwarp();
      continue;
    }
    const Int8Stage& st = stages[slot];
    const int pos0 = t0 + u * kUnit8;

    // ---- S'^T = K . Q'^T, m-tile i: rows g -> token 16 i + g, g + 8 -> +8
    float s[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
      const int r0 = 16 * i + g, r1 = r0 + 8;
      uint4 k0[2], k1[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        k0[hh] = *reinterpret_cast<const uint4*>(&st.k[r0][4 * k8_chunk(r0, 4 * hh + t)]);
        k1[hh] = *reinterpret_cast<const uint4*>(&st.k[r1][4 * k8_chunk(r1, 4 * hh + t)]);
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t* w0 = reinterpret_cast<const uint32_t*>(&k0[kk >> 2]);
        const uint32_t* w1 = reinterpret_cast<const uint32_t*>(&k1[kk >> 2]);
        const uint32_t x0 = w0[kk & 3], x1 = w1[kk & 3];
        mma16816(s[i], hsub2_1152(i8_pair(x0)), hsub2_1152(i8_pair(x1)), hsub2_1152(i8_pair(x0 >> 8)),
                 hsub2_1152(i8_pair(x1 >> 8)), bq[kk][0], bq[kk][1]);
      }
    }

    // ---- scores, masking, online softmax (heads 2t, 2t+1)
    float mx[2] = {-CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const bool v0 = pos0 + 16 * i + g < t1, v1 = pos0 + 16 * i + g + 8 < t1;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[i][e] = v0 ? s[i][e] : -CUDART_INF_F;
        s[i][2 + e] = v1 ? s[i][2 + e] : -CUDART_INF_F;
        mx[e] = fmaxf(mx[e], fmaxf(s[i][e], s[i][2 + e]));
      }
    }
    float alpha[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
      const float m_new = fmaxf(m_run[e], mx[e]);
      alpha[e] = (m_new == -CUDART_INF_F) ? 1.0f
                 : (m_run[e] == -CUDART_INF_F ? 0.0f : exp2f(m_run[e] - m_new));
      m_run[e] = m_new;
      l_run[e] *= alpha[e];
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }
    uint32_t pb[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float pr[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        pr[c] = s[i][c] == -CUDART_INF_F ? 0.0f : exp2f(s[i][c] - m_run[c & 1]);
        l_run[c & 1] += pr[c];
      }
      pb[i][0] = movmatrix_t(pack_half2(pr[0], pr[1]));
      pb[i][1] = movmatrix_t(pack_half2(pr[2], pr[3]));
    }

    // ---- O'^T += V^T . P^T, k-step i: k (2t, 2t+1) -> tokens 16 i + 2t, +1;
    // (2t+8, 2t+9) -> 16 i + 8 + 2t, +1. Dim m-tile mt = (wq, jb): rows g ->
    // byte 2 jb of word g + 8 wq, rows g + 8 -> byte 2 jb + 1.
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int ra = 16 * i + 2 * t, rc = ra + 8;
#pragma unroll
      for (int wq = 0; wq < 4; ++wq) {
        const int w = g + 8 * wq;
        const uint32_t va0 = st.v[ra][v8_word(ra, w)], va1 = st.v[ra + 1][v8_word(ra + 1, w)];
        const uint32_t vc0 = st.v[rc][v8_word(rc, w)], vc1 = st.v[rc + 1][v8_word(rc + 1, w)];
#pragma unroll
        for (int jb = 0; jb < 2; ++jb) {
          // bytes (2jb, 2jb+1) of both tokens -> {A_2jb, A_2jb+1, B_2jb, B_2jb+1}
          // {A_2jb, A_2jb+1, B_2jb, B_2jb+1}: bytes 0,2 pair the two tokens at
          // dim 2jb, bytes 1,3 at dim 2jb + 1
          const uint32_t sel = static_cast<uint32_t>((2 * jb) | ((2 * jb + 1) << 4) |
                                                     ((4 + 2 * jb) << 8) | ((5 + 2 * jb) << 12));
          const uint32_t xa = __byte_perm(va0, va1, sel);
          const uint32_t xc = __byte_perm(vc0, vc1, sel);
          mma16816(o[2 * wq + jb], hsub2_1152(i8_pair(xa)), hsub2_1152(i8_pair(xa >> 8)),
                   hsub2_1152(i8_pair(xc)), hsub2_1152(i8_pair(xc >> 8)), pb[i][0], pb[i][1]);
        }
      }
    }
    __syncwarp();
  }
  cp_async_wait0();
  __syncthreads();

#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], off);
  float* mo = reinterpret_cast<float*>(smem_raw);
  float* mm = mo + kWarps * kHeads * kD;
  float* ml = mm + kWarps * kHeads;
  const __nv_bfloat16* vaq = p.v_aq + static_cast<int64_t>(h) * kD;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int wq = mt >> 1, jb = mt & 1;
    const int d_lo = 4 * (g + 8 * wq) + 2 * jb;  // rows g; rows g + 8 -> d_lo + 1
    const float s_lo = __bfloat162float(vaq[d_lo]), s_hi = __bfloat162float(vaq[d_lo + 1]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int head = 2 * t + e;
      mo[(warp * kHeads + head) * kD + d_lo] = o[mt][e] * s_lo;
      mo[(warp * kHeads + head) * kD + d_lo + 1] = o[mt][2 + e] * s_hi;
    }
  }
  if (g == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mm[warp * kHeads + 2 * t + e] = m_run[e];
      ml[warp * kHeads + 2 * t + e] = l_run[e];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHeads * kD; i += kThreads) {
    const int head = i / kD, d = i % kD;
    if (head >= G) continue;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w * kHeads + head]);
    float acc = 0.0f, l = 0.0f;
    if (M != -CUDART_INF_F) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = mm[w * kHeads + head];
        if (mw == -CUDART_INF_F) continue;
        const float sc = exp2f(mw - M);
        acc = fmaf(sc, mo[(w * kHeads + head) * kD + d], acc);
        l = fmaf(sc, ml[w * kHeads + head], l);
      }
    }
    store_partial(p, b, h * G + head, split, d, acc, M, l);
  }
}

constexpr size_t kInt8Smem = static_cast<size_t>(kInt8StageBytes) * 2 * kWarps;
static_assert(kInt8Smem >= sizeof(float) * (kWarps * kHeads * kD + 2 * kWarps * kHeads),
              "merge buffers must fit in the stage memory");

}  // namespace

bool decode_mma_supported(const DecodeParams& p, bool kivi) {
  if (kivi) return false;  // KIVI runs the page-pipelined kernel (decode_kivi_tma.cu)
  return p.head_size == kD && p.blk == kBlk && p.gqa >= 1 && p.gqa <= kHeads &&
         (reinterpret_cast<uintptr_t>(p.kc) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.vc) & 15u) == 0;
}

int launch_decode_mma(const DecodeParams& p, bool kivi, cudaStream_t stream) {
  if (kivi) return set_error(QKV_ERR_UNSUPPORTED, "launch_decode_mma: INT8 pages only");
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr8{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr8.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(
        int8_decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kInt8Smem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(int8_decode_mma_kernel)");
    attr8.fetch_or(bit);
  }
  dim3 grid(p.num_hist_splits, p.kvh, p.batch);
  int8_decode_mma_kernel<<<grid, kThreads, kInt8Smem, stream>>>(p);
  QKV_CHECK_LAUNCH("int8_decode_mma_kernel");
  if (p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
