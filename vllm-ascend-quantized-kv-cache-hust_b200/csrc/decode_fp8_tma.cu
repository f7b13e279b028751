// FP8 per-token-head paged decode, page-pipelined (head 128, page 128, up to
// 8 query heads per KV head): the read path of the fp8_per_token_head method
// (methods/fp8_per_token_head/: E4M3 codes + one fp32 scale per (token,
// head); the reference stores them but has no read path).
//
// Same skeleton as the INT8 kernel: one CTA of 4 warps owns (request, kv head,
// split) and streams the split's pages through a 2-stage shared-memory ring;
// thread 0 issues the page's K and V rows of this head with two TMA copies
// (128-byte swizzle) and every thread copies its token's two scales with
// cp.async, all completing on the stage's "full" mbarrier. Warp w computes
// tokens [32w, 32w + 32) of every page with mma.sync m16n8k16 (fp16 x fp16 ->
// fp32), the query heads of the KV head as N:
//     S^T[token][head] = k_scale[token] * (K[token][channel] . Q'^T)
//     O^T[dim][head]  += V^T[dim][token] . (v_scale[token] * P^T[token][head])
// with Q' = q * softmax_scale * log2(e); the softmax sum uses the unscaled P.
// E4M3 -> fp16 is exact: one cvt.rn.f16x2.e4m3x2 per byte pair.
//
// Rows of an m-tile: row g (and g + 8) of m-tile i of warp w is page token
// 32 w + 16 i + perm(g) (+ 8), perm = 0 4 3 7 5 1 6 2, which keeps the
// swizzled key (16-byte) and value (4-byte) loads free of bank conflicts.
#include <math_constants.h>

#include <atomic>

#include "decode_common.cuh"
#include "tma_common.cuh"

namespace qkv {

namespace {

using namespace tma;

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kD = 128;
constexpr int kBlk = 128;
constexpr int kHeads = 8;
constexpr int kTokW = kBlk / kWarps;
constexpr int kMaxPages = 64;
constexpr int kStages = 2;
constexpr float kLazy = 4.0f;            // log2 headroom of the running max
constexpr uint32_t kPerm8 = 0x26157340u;  // perm(g) = nibble g

struct __align__(1024) Fp8Page {
  unsigned char k[kBlk][kD];  // 128-byte rows, 128-byte swizzle
  unsigned char v[kBlk][kD];
  float ks[kBlk];  // per-token scales of this head
  float vs[kBlk];
};

struct __align__(1024) Fp8Shared {
  Fp8Page st[kStages];
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
  int pid[kMaxPages];
};
constexpr size_t kFp8SmemBytes = sizeof(Fp8Shared) + 1024;  // + base alignment

__device__ __forceinline__ int perm8(int g) { return (kPerm8 >> (4 * g)) & 7; }

// E4M3 bytes (0, 1) and (2, 3) of x -> two exact fp16 pairs
__device__ __forceinline__ void e4m3x4_to_h2(uint32_t x, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n"
      " cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(x));
}
__device__ __forceinline__ uint32_t lds32(const unsigned char* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__global__ void __launch_bounds__(kThreads, 3)
fp8_decode_tma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ unsigned char smem_raw[];
  // the 128-byte swizzle repeats every 1024 bytes: align the ring to that
  const uint32_t raw = smem_u32(smem_raw);
  Fp8Shared& sh = *reinterpret_cast<Fp8Shared*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;

  const int L = max(p.seq_lens[b], 0);
  const int t0 = split * p.split_tokens;
  const int t1 = min(L, t0 + p.split_tokens);
  const int n_pages = t1 > t0 ? min((t1 - t0 + kBlk - 1) / kBlk, kMaxPages) : 0;
  if (n_pages == 0 && p.splits_total > 1) {  // the request ends before this split
    empty_split(p, b, h, split);
    return;
  }

  for (int i = tid; i < n_pages; i += kThreads)
    sh.pid[i] = static_cast<int>(page_of(p, b, t0 + i * kBlk));
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], kThreads + 1);  // TMA bytes + every thread's scale copies
      mbar_init(&sh.empty[s], kWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }

  // ---- Q' = q * scale * log2(e) for head g, once per CTA. k-step kk uses
  // word m = 4t + kk (kk < 4) or 16 + 4t + kk - 4 of a key row: channels
  // 4m, 4m + 1 (k 2t, 2t+1) and 4m + 2, 4m + 3 (k 2t+8, 2t+9)
  uint32_t bq[8][2];
  {
    const __nv_bfloat16* qrow =
        p.q + static_cast<int64_t>(b) * p.q_stride + (static_cast<int64_t>(h) * G + g) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int m = kk < 4 ? 4 * t + kk : 16 + 4 * t + kk - 4;
      float qq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qq[i] = g < G ? __bfloat162float(qrow[4 * m + i]) * p.scale_log2 : 0.0f;
      bq[kk][0] = pack_half2(qq[0], qq[1]);
      bq[kk][1] = pack_half2(qq[2], qq[3]);
    }
  }
  __syncthreads();

  // All threads: thread 0 the two TMA copies (after the stage's "empty"
  // wait, done by the caller), every thread its own token's two scales. A
  // token's scales are read only by the warp that owns the token, which has
  // finished the page this stage held before.
  auto issue = [&](int ii) {
    const int s = ii % kStages;
    const int pg = sh.pid[ii];
    if (pg >= 0) {
      if (tid == 0) {
        mbar_expect_tx(&sh.full[s], static_cast<uint32_t>(2 * kBlk * kD));
        tma_load_3d(&sh.st[s].k[0][0], &tmap_k, 0, h, pg * kBlk, &sh.full[s]);
        tma_load_3d(&sh.st[s].v[0][0], &tmap_v, 0, h, pg * kBlk, &sh.full[s]);
      }
      const int64_t si = (static_cast<int64_t>(pg) * kBlk + tid) * p.kvh + h;
      cp_async_small<4>(&sh.st[s].ks[tid], p.ks + si);
      cp_async_small<4>(&sh.st[s].vs[tid], p.vs + si);
      cp_async_arrive_noinc(&sh.full[s]);
    } else {
      if (tid == 0) mbar_arrive(&sh.full[s]);
      mbar_arrive(&sh.full[s]);
    }
  };
  if (n_pages > 0) issue(0);

  // ---- per-thread swizzled offsets (bytes from the start of a page's rows)
  const int P = perm8(g);
  const int k_row = (kTokW * warp + P) * kD;  // key rows g (m-tile 0); +16 rows per m-tile, +8 for g + 8
  int k_col[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) k_col[hh] = ((4 * hh + t) ^ P) << 4;
  const int R = perm8(2 * t);                 // value rows for k 2t; k 2t+1 uses R ^ 4
  const int v_rowA = (kTokW * warp + R) * kD;
  const int v_rowB = (kTokW * warp + (R ^ 4)) * kD;
  int v_off[4];  // word g + 8 q of a row with (r & 7) = R; rows R ^ 4 use v_off[q ^ 2]
#pragma unroll
  for (int q = 0; q < 4; ++q)
    v_off[q] = ((2 * (q ^ (R >> 1)) + ((g >> 2) ^ (R & 1))) << 4) + 4 * (g & 3);

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_run[2] = {0.0f, 0.0f};
  bool timed_out = false;

  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kStages;
    if (i + 1 < n_pages) {
      // the stage of page i + 1 held page i - 1: all warps must be done with
      // its K/V rows before the TMA refills them
      if (tid == 0 && i + 1 >= kStages &&
          !mbar_wait(&sh.empty[(i + 1) % kStages], static_cast<uint32_t>(((i - 1) / kStages) & 1)))
        timed_out = true;
      issue(i + 1);
    }
    const bool ok = mbar_wait(&sh.full[s], static_cast<uint32_t>((i / kStages) & 1));
    timed_out |= !ok;
    const int pg = sh.pid[i];
    const int pos0 = t0 + i * kBlk;
    const int valid = min(kBlk, t1 - pos0) - kTokW * warp;  // live tokens of this warp
    if (ok && pg >= 0 && valid > 0) {
      const unsigned char* kpage = &sh.st[s].k[0][0];
      const unsigned char* vpage = &sh.st[s].v[0][0];

      // ---- scores: m-tile j, rows g / g + 8 -> tokens 32w + 16j + P (+ 8)
      float sc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
        const unsigned char* r0 = kpage + k_row + 16 * j * kD;
        const unsigned char* r1 = r0 + 8 * kD;
        uint4 k0[2], k1[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          k0[hh] = *reinterpret_cast<const uint4*>(r0 + k_col[hh]);
          k1[hh] = *reinterpret_cast<const uint4*>(r1 + k_col[hh]);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t x0 = reinterpret_cast<const uint32_t*>(&k0[kk >> 2])[kk & 3];
          const uint32_t x1 = reinterpret_cast<const uint32_t*>(&k1[kk >> 2])[kk & 3];
          uint32_t a0, a2, a1, a3;
          e4m3x4_to_h2(x0, a0, a2);
          e4m3x4_to_h2(x1, a1, a3);
          mma16816(sc[j], a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
        }
        // per-token key scales: rows g and g + 8 of m-tile j
        const float kr0 = sh.st[s].ks[kTokW * warp + 16 * j + P];
        const float kr1 = sh.st[s].ks[kTokW * warp + 16 * j + 8 + P];
        sc[j][0] *= kr0;
        sc[j][1] *= kr0;
        sc[j][2] *= kr1;
        sc[j][3] *= kr1;
      }
      if (valid < kTokW) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const bool lo_ok = 16 * j + P < valid, hi_ok = 16 * j + 8 + P < valid;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (!lo_ok) sc[j][e] = -CUDART_INF_F;
            if (!hi_ok) sc[j][2 + e] = -CUDART_INF_F;
          }
        }
      }

      // ---- online softmax over heads 2t, 2t+1, lazy rescale
      float mx[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mx[e] = fmaxf(fmaxf(sc[0][e], sc[0][2 + e]), fmaxf(sc[1][e], sc[1][2 + e]));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
      }
      const bool grow0 = mx[0] > m_run[0] + kLazy, grow1 = mx[1] > m_run[1] + kLazy;
      if (__any_sync(0xffffffffu, grow0 || grow1)) {
        const float a0 = grow0 ? fast_exp2(m_run[0] - mx[0]) : 1.0f;
        const float a1 = grow1 ? fast_exp2(m_run[1] - mx[1]) : 1.0f;
        if (grow0) m_run[0] = mx[0];
        if (grow1) m_run[1] = mx[1];
        l_run[0] *= a0;
        l_run[1] *= a1;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][0] *= a0;
          o[mt][1] *= a1;
          o[mt][2] *= a0;
          o[mt][3] *= a1;
        }
      }
      uint32_t pb[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float pr[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) pr[c] = fast_exp2(sc[j][c] - m_run[c & 1]);
        l_run[0] += pr[0] + pr[2];
        l_run[1] += pr[1] + pr[3];
        // per-token value scales fold into P before P.V
        const float vr0 = sh.st[s].vs[kTokW * warp + 16 * j + P];
        const float vr1 = sh.st[s].vs[kTokW * warp + 16 * j + 8 + P];
        pb[j][0] = movmatrix_t(pack_half2(pr[0] * vr0, pr[1] * vr0));
        pb[j][1] = movmatrix_t(pack_half2(pr[2] * vr1, pr[3] * vr1));
      }

      // ---- O'^T += V^T . P^T; k-step j: k (2t, 2t+1) = rows (A, B) of m-tile
      // j, (2t+8, 2t+9) their + 8; dim m-tile (wq, jb): rows g -> byte 2 jb of
      // word g + 8 wq, rows g + 8 -> byte 2 jb + 1
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const unsigned char* ra = vpage + v_rowA + 16 * j * kD;
        const unsigned char* rb = vpage + v_rowB + 16 * j * kD;
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          const uint32_t va0 = lds32(ra + v_off[wq]), va1 = lds32(rb + v_off[wq ^ 2]);
          const uint32_t vc0 = lds32(ra + 8 * kD + v_off[wq]), vc1 = lds32(rb + 8 * kD + v_off[wq ^ 2]);
#pragma unroll
          for (int jb = 0; jb < 2; ++jb) {
            // bytes (row A, row B) of dim 2 jb, then of dim 2 jb + 1
            const uint32_t sel = static_cast<uint32_t>((2 * jb) | ((4 + 2 * jb) << 4) |
                                                       ((2 * jb + 1) << 8) | ((5 + 2 * jb) << 12));
            uint32_t a0, a1, a2, a3;
            e4m3x4_to_h2(__byte_perm(va0, va1, sel), a0, a1);
            e4m3x4_to_h2(__byte_perm(vc0, vc1, sel), a2, a3);
            mma16816(o[2 * wq + jb], a0, a1, a2, a3, pb[j][0], pb[j][1]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh.empty[s]);
  }
  if (timed_out) record_error(p.err, kErrPipelineTimeout);
  __syncthreads();

  // ---- merge the 4 warps (stage memory reused: every issued page was waited on)
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], off);
  float* mo = reinterpret_cast<float*>(&sh.st[0].k[0][0]);  // [warp][head][dim]
  float* mm = mo + kWarps * kHeads * kD;
  float* ml = mm + kWarps * kHeads;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int wq = mt >> 1, jb = mt & 1;
    const int d_lo = 4 * (g + 8 * wq) + 2 * jb;  // rows g; rows g + 8 -> d_lo + 1
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int head = 2 * t + e;
      mo[(warp * kHeads + head) * kD + d_lo] = o[mt][e];
      mo[(warp * kHeads + head) * kD + d_lo + 1] = o[mt][2 + e];
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
  for (int idx = tid; idx < kHeads * kD; idx += kThreads) {
    const int head = idx / kD, d = idx % kD;
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

static_assert(sizeof(Fp8Page) * kStages >=
                  sizeof(float) * (kWarps * kHeads * kD + 2 * kWarps * kHeads),
              "merge buffers must fit in the stage memory");

// FP8 data pages [NB, block, KVH, D] as a 3-D map {D bytes, KVH, NB * block}
// with the 128-byte swizzle; one box = the 128 token rows of one head of a page.
int encode_fp8_map(const int8_t* base, const DecodeParams& p, CUtensorMap* map) {
  auto enc = encode_fn();
  if (enc == nullptr) return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.kvh),
                              static_cast<cuuint64_t>(p.num_blocks) * kBlk};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kD) * p.kvh};
  const cuuint32_t box[3] = {kD, 1, kBlk};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides,
                         box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled(fp8 pages) failed: " + std::to_string(r));
  return QKV_OK;
}

}  // namespace

bool fp8_tma_geometry(const DecodeParams& p) {
  return p.head_size == kD && p.blk == kBlk && p.gqa >= 1 && p.gqa <= kHeads;
}

bool fp8_tma_supported(const DecodeParams& p) {
  const auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  return fp8_tma_geometry(p) && p.num_blocks > 0 &&
         static_cast<int64_t>(p.num_blocks) * kBlk < (int64_t{1} << 31) && al(p.kc) && al(p.vc) &&
         (reinterpret_cast<uintptr_t>(p.ks) & 3u) == 0 && (reinterpret_cast<uintptr_t>(p.vs) & 3u) == 0;
}

// The INT8 kernel's split plan: same page geometry and 3 CTAs per SM.
SplitPlan plan_int8_tma(int batch, int kvh, int max_seq_len, int sms);
SplitPlan plan_fp8_tma(int batch, int kvh, int max_seq_len, int sms) {
  return plan_int8_tma(batch, kvh, max_seq_len, sms);
}

int launch_fp8_tma(const DecodeParams& p, cudaStream_t stream) {
  CUtensorMap tk, tv;
  int rc = encode_fp8_map(p.kc, p, &tk);
  if (rc != QKV_OK) return rc;
  if ((rc = encode_fp8_map(p.vc, p, &tv)) != QKV_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(fp8_decode_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kFp8SmemBytes));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(fp8_decode_tma_kernel)");
    attr.fetch_or(bit);
  }
  dim3 grid(p.num_hist_splits, p.kvh, p.batch);
  fp8_decode_tma_kernel<<<grid, kThreads, kFp8SmemBytes, stream>>>(p, tk, tv);
  QKV_CHECK_LAUNCH("fp8_decode_tma_kernel");
  if (p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
