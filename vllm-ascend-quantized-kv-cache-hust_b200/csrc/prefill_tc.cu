// Prompt / chunk attention on the fifth-generation tensor core (tcgen05).
//
// Varlen TND layout: q [total_q, Hq, 128] bf16, k / v [total_k, KVH, 128]
// bf16, request r owns query rows [cu_q[r], cu_q[r+1]) and key rows
// [cu_k[r], cu_k[r+1]); causal rows see keys up to (kv_len - q_len) + i, the
// alignment of the reference's prompt attention (FIA TND, sparse_mode 3).
//
// One CTA per SM owns TWO q-tiles of one request and one KV head. A q-tile is
// the G query heads of the KV head times 128 / G tokens: the M = 128 rows of
// an MMA. Per 64-key tile j and q-tile t:
//     S_t[128 x 64]  = Q_t . K_j^T   tcgen05.mma kind::f16, fp32 in TMEM
//     P_t = softmax row pieces       one thread per row (TMEM lane = row)
//     O_t[128 x 128] += P_t . V_j    A = P_t (K-major, shared memory),
//                                    B = V_j (MN-major)
// Warp roles: warps 0-3 run the softmax of q-tile 0, warps 4-7 of q-tile 1,
// warp 8 issues the TMA copies (Q once, K/V tiles into a 3-stage ring), warp 9
// issues the MMAs. The MMA warp ping-pongs: while warpgroup 1 turns S_1(j)
// into P_1(j), the tensor core runs P_0(j).V_j and S_0(j+1), and the other
// way round, so the exponentials of one q-tile overlap the MMAs of the other,
// and each K/V tile read from L2 serves 256 query rows. The running max moves
// lazily (8 log2 units); O is rescaled in TMEM only then. tcgen05.commit
// arrives on mbarriers (S ready, stage free, O final); every wait is bounded,
// and a wait that gives up ends the CTA's loops, drains what is in flight,
// frees TMEM, skips the store and records device error 5.
#include <math_constants.h>

#include <atomic>

#include "decode_common.cuh"
#include "tma_common.cuh"

namespace qkv {

namespace {

using namespace tma;

constexpr int kD = 128;
constexpr int kRows = 128;     // MMA M: q tokens x query heads of one KV head
constexpr int kKTile = 64;     // keys per tile (MMA N of S, K of P.V)
constexpr int kStages = 3;     // K/V ring
constexpr int kSoftmaxThreads = 256;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr float kLazyMax = 8.0f;
constexpr uint32_t kTmemCols = 512;  // S_0 at 0, S_1 at 64, O_0 at 128, O_1 at 256
__host__ __device__ constexpr uint32_t s_col(int t) { return t == 0 ? 0u : 64u; }
__host__ __device__ constexpr uint32_t o_col(int t) { return t == 0 ? 128u : 256u; }

struct __align__(1024) PrefillSmem {
  __nv_bfloat16 q[2][2][kRows][64];        // [q-tile][64-dim block][row][dims], 128-B rows
  __nv_bfloat16 k[kStages][2][kKTile][64];  // [stage][64-dim block][key][dims]
  __nv_bfloat16 v[kStages][2][kKTile][64];  // [stage][64-dim block][key][dims]
  __nv_bfloat16 p[2][kRows][64];            // [q-tile][row][key], 128-B rows
  unsigned long long q_full;
  unsigned long long kv_full[kStages], kv_empty[kStages];
  unsigned long long s_full[2], p_ready[2], o_done[2];
  uint32_t tmem_base;
};
constexpr size_t kPrefillSmem = sizeof(PrefillSmem) + 1024;
static_assert(kPrefillSmem <= 227 * 1024, "shared memory of one CTA");

struct PrefillArgs {
  const int32_t* cu_q;
  const int32_t* cu_k;
  int num_reqs;
  int num_heads, kvh, gqa, tokens_per_tile;
  int causal;
  float scale_log2;
  __nv_bfloat16* out;
  int* err;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void mbar_arrive_local(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tmap_q,
                  const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  const int G = a.gqa, TPT = a.tokens_per_tile;

  // ---- which request and pair of q-tiles (pairs never straddle requests)
  int r = -1, pair = 0;
  {
    int acc = 0;
    for (int i = 0; i < a.num_reqs; ++i) {
      const int ql = a.cu_q[i + 1] - a.cu_q[i];
      const int nt = ql > 0 ? (ql + TPT - 1) / TPT : 0;
      const int np = (nt + 1) / 2;
      if (static_cast<int>(blockIdx.x) < acc + np) {
        r = i;
        pair = blockIdx.x - acc;
        break;
      }
      acc += np;
    }
  }
  if (r < 0) return;  // uniform: past the last pair
  const int q_begin = a.cu_q[r], q_len = a.cu_q[r + 1] - q_begin;
  const int k_begin = a.cu_k[r], k_len = a.cu_k[r + 1] - k_begin;
  const int tile0 = 2 * pair;                        // q-tile index of warpgroup 0
  const bool has1 = (tile0 + 1) * TPT < q_len;       // q-tile 1 holds live queries
  const int off = k_len - q_len;                     // causal alignment
  const int last_qi = min((tile0 + (has1 ? 2 : 1)) * TPT, q_len) - 1;
  const int kv_end = a.causal ? max(0, min(k_len, off + last_qi + 1)) : max(k_len, 0);
  const int n_tiles = (kv_end + kKTile - 1) / kKTile;

  // ---- tensor memory + barriers
  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_ready[t], kSoftmaxThreads / 2);
      mbar_init(&sm.o_done[t], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;
  bool timed_out = false;

  if (warp == kProducerWarp) {
    // ================================================= TMA producer (one lane)
    if (lane == 0 && n_tiles > 0) {
      const int q0 = q_begin + tile0 * TPT;
      mbar_expect_tx(&sm.q_full, static_cast<uint32_t>(sizeof(sm.q[0]) * (has1 ? 2 : 1)));
      for (int t = 0; t < (has1 ? 2 : 1); ++t)
        for (int b = 0; b < 2; ++b)
          tma_load_3d(&sm.q[t][b][0][0], &tmap_q, 64 * b, h * G, q0 + t * TPT, &sm.q_full);
      constexpr uint32_t kKvBytes = 2 * 2 * kKTile * 64 * 2;
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], static_cast<uint32_t>((j / kStages - 1) & 1))) {
          timed_out = true;
          break;
        }
        mbar_expect_tx(&sm.kv_full[s], kKvBytes);
        const int z = k_begin + j * kKTile;
        for (int b = 0; b < 2; ++b) {
          tma_load_3d(&sm.k[s][b][0][0], &tmap_k, 64 * b, h, z, &sm.kv_full[s]);
          tma_load_3d(&sm.v[s][b][0][0], &tmap_v, 64 * b, h, z, &sm.kv_full[s]);
        }
        issued = j + 1;
      }
      // every copy this CTA started lands before the CTA leaves
      for (int j = max(0, issued - kStages); j < issued; ++j)
        if (!mbar_wait(&sm.kv_full[j % kStages], static_cast<uint32_t>((j / kStages) & 1))) timed_out = true;
    }
  } else if (warp == kMmaWarp) {
    // ================================================= MMA issuer (one lane)
    if (lane == 0 && n_tiles > 0) {
      const uint32_t id_qk = tc::idesc_f16(kRows, kKTile, 1, 0, 0);
      const uint32_t id_pv = tc::idesc_f16(kRows, kD, 1, 0, 1);
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = smem_u32(&sm.q[t][0][0][0]);
        const uint32_t k_addr = smem_u32(&sm.k[j % kStages][0][0][0]);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_ss(tbase + s_col(t), tc::smem_desc_sw128(q_addr + kb * 16384 + ks * 32, 16, 1024),
                       tc::smem_desc_sw128(k_addr + kb * 8192 + ks * 32, 16, 1024), id_qk,
                       (kb | ks) != 0 ? 1u : 0u);
        tc::mma_commit(&sm.s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_addr = smem_u32(&sm.v[j % kStages][0][0][0]);
        const uint32_t p_addr = smem_u32(&sm.p[t][0][0]);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_ss(tbase + o_col(t), tc::smem_desc_sw128(p_addr + ks * 32, 16, 1024),
                     tc::smem_desc_sw128(v_addr + ks * 16 * 128, 8192, 1024), id_pv,
                     (j > 0 || ks > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(&sm.q_full, 0) && mbar_wait(&sm.kv_full[0], 0);
      tc::fence_after_sync();
      if (ok) {
        issue_s(0, 0);
        if (has1) issue_s(1, 0);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const bool next = j + 1 < n_tiles;
        // q-tile 0: P_0(j).V_j, then S_0(j + 1) while warpgroup 1 works
        if (!(ok = mbar_wait(&sm.p_ready[0], static_cast<uint32_t>(j & 1)))) break;
        tc::fence_after_sync();
        issue_pv(0, j);
        if (next) {
          const int s1 = (j + 1) % kStages;
          if (!(ok = mbar_wait(&sm.kv_full[s1], static_cast<uint32_t>(((j + 1) / kStages) & 1)))) break;
          tc::fence_after_sync();
          issue_s(0, j + 1);
        }
        if (has1) {
          if (!(ok = mbar_wait(&sm.p_ready[1], static_cast<uint32_t>(j & 1)))) break;
          tc::fence_after_sync();
          issue_pv(1, j);
        }
        tc::mma_commit(&sm.kv_empty[j % kStages]);  // K_j, V_j and both P buffers consumed
        if (has1 && next) issue_s(1, j + 1);
      }
      if (!ok) timed_out = true;
      tc::mma_commit(&sm.o_done[0]);
      if (has1) tc::mma_commit(&sm.o_done[1]);
    }
  } else {
    // ================================================= softmax warpgroups
    const int t = warp >> 2;  // q-tile of this warpgroup
    const int row = tid & 127;
    const bool active = t == 0 || has1;
    const int qi = (tile0 + t) * TPT + row / G;  // query index inside the request
    const int row_end = a.causal ? min(k_len, off + qi + 1) : k_len;  // keys [0, row_end)
    const uint32_t t_row = tbase + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    float m_run = -CUDART_INF_F, l_run = 0.0f;
    for (int j = 0; active && j < n_tiles; ++j) {
      if (!mbar_wait(&sm.s_full[t], static_cast<uint32_t>(j & 1))) {
        timed_out = true;
        break;
      }
      tc::fence_after_sync();
      uint32_t sv[64];
      tc::tmem_ld64(t_row + s_col(t), sv);
      float sc[64];
      float pm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = -CUDART_INF_F;
      const bool tile_full = (j + 1) * kKTile <= row_end;
      if (__all_sync(0xffffffffu, tile_full)) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          sc[c] = __uint_as_float(sv[c]);
          pm[c & 7] = fmaxf(pm[c & 7], sc[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float v = __uint_as_float(sv[c]);
          sc[c] = j * kKTile + c < row_end ? v : -CUDART_INF_F;
          pm[c & 7] = fmaxf(pm[c & 7], sc[c]);
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                       fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      mx *= a.scale_log2;  // the scale is positive: max commutes with it
      const bool grow = mx > m_run + kLazyMax;
      // S_t(j) is complete, so is every earlier MMA of this q-tile: O_t and
      // the P_t buffer are free to touch
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        const float alpha = grow ? fast_exp2(m_run - mx) : 1.0f;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t ov[32];
          tc::tmem_ld32(t_row + o_col(t) + 32 * cb, ov);
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
          tc::tmem_st32(t_row + o_col(t) + 32 * cb, ov);
        }
        tc::tmem_wait_st();
        l_run *= alpha;
      }
      if (grow) m_run = mx;
      const float neg_m = m_run == -CUDART_INF_F ? 0.0f : -m_run;
      uint32_t pk[32];
      float ps[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps[i] = 0.0f;
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = fast_exp2(fmaf(sc[c], a.scale_log2, neg_m));
        const float p1 = fast_exp2(fmaf(sc[c + 1], a.scale_log2, neg_m));
        ps[(c >> 1) & 7] += p0 + p1;
        pk[c >> 1] = pack_bf16x2(p0, p1);
      }
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      // 8 chunks of 16 B; chunk c of row r sits at chunk c ^ (r & 7)
      unsigned char* prow = reinterpret_cast<unsigned char*>(&sm.p[t][0][0]) + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // P visible to the tensor core
      tc::fence_before_sync();
      mbar_arrive_local(&sm.p_ready[t]);
    }
    // ---- epilogue: O / l -> bf16
    if (active && n_tiles > 0) {
      if (!mbar_wait(&sm.o_done[t], 0)) timed_out = true;
      tc::fence_after_sync();
    }
    const int qrow = q_begin + qi;
    const bool live = active && qi < q_len;
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    __nv_bfloat16* orow = a.out + (static_cast<int64_t>(qrow) * a.num_heads + h * G + row % G) * kD;
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t ov[32];
      if (active && n_tiles > 0) {
        tc::tmem_ld32(t_row + o_col(t) + 32 * cb, ov);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) ov[c] = 0u;
      }
      if (live && !timed_out) {
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(ov[c + 2]) * inv, __uint_as_float(ov[c + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(ov[c + 4]) * inv, __uint_as_float(ov[c + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(ov[c + 6]) * inv, __uint_as_float(ov[c + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + 32 * cb + c) = w;
        }
      }
    }
  }
  if (timed_out) record_error(a.err, kErrPipelineTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, kTmemCols);
  }
}

int encode_rows_map(const void* base, int64_t rows, int heads, int box_heads, int box_rows,
                    CUtensorMap* map, const char* what) {
  auto enc = encode_fn();
  if (enc == nullptr) return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(kD) * 2 * heads};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_heads), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult res = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                           box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return set_error(QKV_ERR_CUDA, std::string("cuTensorMapEncodeTiled(") + what + ") failed: " +
                                       std::to_string(res));
  return QKV_OK;
}

}  // namespace

bool prefill_tc_supported(int head_size, int gqa, const void* q, const void* k, const void* v,
                          const void* out) {
  const auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  return head_size == kD && gqa >= 1 && gqa <= 8 && (kRows % gqa) == 0 && al(q) && al(k) && al(v) &&
         al(out);
}

// Launches the tcgen05 prompt attention; q / out [total_q, Hq, 128],
// k / v [total_k, KVH, 128] bf16; tiles_upper >= the q-tile count.
int launch_prefill_tc(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                      const int32_t* cu_q, const int32_t* cu_k, int num_reqs, int total_q, int total_k,
                      int num_heads, int kvh, int causal, float scale, __nv_bfloat16* out,
                      cudaStream_t stream) {
  const int G = num_heads / kvh;
  const int tpt = kRows / G;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = encode_rows_map(q, total_q, num_heads, G, tpt, &tq, "query")) != QKV_OK) return rc;
  if ((rc = encode_rows_map(k, total_k, kvh, 1, kKTile, &tk, "key")) != QKV_OK) return rc;
  if ((rc = encode_rows_map(v, total_k, kvh, 1, kKTile, &tv, "value")) != QKV_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kPrefillSmem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(prefill_tc_kernel)");
    attr.fetch_or(bit);
  }
  PrefillArgs a{};
  a.cu_q = cu_q;
  a.cu_k = cu_k;
  a.num_reqs = num_reqs;
  a.num_heads = num_heads;
  a.kvh = kvh;
  a.gqa = G;
  a.tokens_per_tile = tpt;
  a.causal = causal;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  a.err = device_error_ptr();
  const int pairs_upper = ((total_q + tpt - 1) / tpt + num_reqs + 1) / 2 + num_reqs;
  dim3 grid(pairs_upper, kvh);
  prefill_tc_kernel<<<grid, kThreads, kPrefillSmem, stream>>>(a, tq, tk, tv);
  QKV_CHECK_LAUNCH("prefill_tc_kernel");
  return QKV_OK;
}

}  // namespace qkv
