// Prompt / chunk attention on the fifth-generation tensor core (tcgen05).
//
// Varlen TND layout: q [total_q, Hq, 128] bf16, k / v [total_k, KVH, 128]
// bf16, request r owns query rows [cu_q[r], cu_q[r+1]) and key rows
// [cu_k[r], cu_k[r+1]); causal rows see keys up to (kv_len - q_len) + i, the
// alignment of the reference's prompt attention (FIA TND, sparse_mode 3).
//
// One CTA per SM owns TWO q-tiles of one request and one KV head. A q-tile is
// the G query heads of the KV head times 128 / G tokens: the M = 128 rows of
// an MMA. Per 128-key tile j and q-tile t:
//     S_t[128 x 128] = Q_t . K_j^T   tcgen05.mma kind::f16, A and B from
//                                    shared memory, fp32 in tensor memory
//     P_t = softmax row pieces       one thread per row (TMEM lane = row):
//                                    the row max over the whole tile first,
//                                    then bf16 P written back over the upper
//                                    64 columns of S_t
//     O_t[128 x 128] += P_t . V_j    A = P_t from TENSOR memory, B = V_j
//                                    (MN-major) from shared memory
// Keeping P in tensor memory leaves the tensor core only Q, K and V to read
// from shared memory (about 94 B per cycle at full rate, under the SM's 128);
// a 64-key tile with P in shared memory needed about 190.
// Warp roles: warps 0-3 run the softmax of q-tile 0, warps 4-7 of q-tile 1,
// warp 8 issues the TMA copies (Q once; K and V tiles into separate 2-stage
// rings, so K_{j+2} loads as soon as both S MMAs of tile j are done), warp 9
// issues the MMAs, ping-ponging: while warpgroup 1 turns S_1(j) into P_1(j),
// the tensor core runs P_0(j).V_j and S_0(j+1), and the other way round. A
// CTA's MMAs execute in issue order, so S_t(j+1) may overwrite the columns
// P_t(j).V_j reads. P of keys 64-127 is handed over first, so their P.V runs
// while the warpgroup finishes keys 0-63. The running max moves lazily (8 log2
// units); O is rescaled in TMEM only then, before any P of the tile exists.
// tcgen05.commit arrives on mbarriers; every wait is bounded, and a wait that
// gives up ends the CTA's loops, drains what is in flight, frees TMEM, skips
// the store and records device error 5.
#include <math_constants.h>

#include <atomic>

#include "decode_common.cuh"
#include "tma_common.cuh"

namespace qkv {

namespace {

using namespace tma;

constexpr int kD = 128;
constexpr int kRows = 128;     // MMA M: q tokens x query heads of one KV head
constexpr int kKTile = 128;    // keys per tile (MMA N of S, K of P.V)
constexpr int kStages = 2;     // K ring and V ring
constexpr int kSoftmaxThreads = 256;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr float kLazyMax = 8.0f;
constexpr uint32_t kTmemCols = 512;  // S_t (P_t in its first 64) at 128 t, O_t at 256 + 128 t
__host__ __device__ constexpr uint32_t s_col(int t) { return 128u * t; }
__host__ __device__ constexpr uint32_t o_col(int t) { return 256u + 128u * t; }

struct __align__(1024) PrefillSmem {
  __nv_bfloat16 q[2][2][kRows][64];         // [q-tile][64-dim block][row][dims], 128-B rows
  __nv_bfloat16 k[kStages][2][kKTile][64];  // [stage][64-dim block][key][dims]
  __nv_bfloat16 v[kStages][2][kKTile][64];  // [stage][64-dim block][key][dims]
  unsigned long long q_full;
  unsigned long long k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  unsigned long long s_full[2], p_hi[2], p_ready[2], o_done[2];  // p_hi: P of keys 64-127 written
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

// Packed fp32 pairs (one f32x2 instruction for both lanes).
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// max of three (one instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair of scores on the FMA pipe instead of the SFU. x = n + f with
// n = rint(x): adding 1.5 * 2^23 leaves n in the low mantissa bits of t, and
// f = x - (t - 1.5 * 2^23) lies in [-1/2, 1/2]. 2^f is a cubic in Horner form,
// and n goes into the exponent field as (bits of t) << 23 (the shift constant's
// own bits vanish in that shift). The cubic is a relative-error minimax fit of
// 2^f on [-1/2, 1/2] by Lawson's iteratively reweighted least squares
// (exp2_poly_fit.py beside this file prints these float32 coefficients); its
// largest relative error evaluated in fp32 is 7.5e-5, under the 2^-9 of the bf16
// rounding P goes through next. The softmax's arguments are at most a few
// units above 0 (the lazy running max), so n + 127 stays below 255; below -126
// (masked scores: -inf) the exponent field would wrap, and the result is
// selected to 0 there, as the SFU's flush-to-zero ex2 gives: a row that sees
// no key keeps a zero sum.
constexpr float kExp2C0 = 0.99992806f, kExp2C1 = 0.69326097f, kExp2C2 = 0.24261114f, kExp2C3 = 0.055171669f;
__device__ __forceinline__ void exp2_fma2(unsigned long long x2, float& p0, float& p1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const unsigned long long rnd = f2_pack(kRound, kRound);
  const unsigned long long t = f2_add(x2, rnd);
  const unsigned long long f = f2_sub(x2, f2_sub(t, rnd));
  unsigned long long q = f2_fma(f2_pack(kExp2C3, kExp2C3), f, f2_pack(kExp2C2, kExp2C2));
  q = f2_fma(q, f, f2_pack(kExp2C1, kExp2C1));
  q = f2_fma(q, f, f2_pack(kExp2C0, kExp2C0));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = x0 >= -126.0f ? __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23)) : 0.0f;
  p1 = x1 >= -126.0f ? __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23)) : 0.0f;
}

// Scores at columns >= lim of a 32-column chunk become -inf (causal mask).
__device__ __forceinline__ void mask_scores(uint32_t (&sv)[32], int lim) {
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c >= lim) sv[c] = __float_as_uint(-CUDART_INF_F);
}
// Running maxima of a chunk: 4 chains of 3-input maxima, two scores per step.
__device__ __forceinline__ void max_scores(float (&cm)[4], const uint32_t (&sv)[32]) {
#pragma unroll
  for (int c = 0; c < 32; c += 2)
    cm[(c >> 1) & 3] = max3f(cm[(c >> 1) & 3], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
}
// p = 2^(s * scale * log2(e) - m) for a 32-score chunk, the scaling as one
// f32x2 FMA per pair. The SFU's ex2 takes 15 of the 16 pairs and the FMA pipe
// (exp2_fma2) the last, whose result then does not wait behind the SFU queue
// (measured on config 4: 1168 TFLOP/s against 1140 with every pair on the SFU,
// 1113-1134 with a quarter and 1036-1067 with a half or more on the FMA pipe).
// Sums go to ps2, bf16 pairs to pk.
__device__ __forceinline__ void exp_scores(const uint32_t (&sv)[32], unsigned long long sc2, unsigned long long nm2,
                                           unsigned long long (&ps2)[4], uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const unsigned long long x2 =
        f2_fma(f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), sc2, nm2);
    float p0, p1;
    if (i == 15) {
      exp2_fma2(x2, p0, p1);
    } else {
      float x0, x1;
      f2_unpack(x2, x0, x1);
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    ps2[i & 3] = f2_add(ps2[i & 3], f2_pack(p0, p1));
    pk[i] = pack_bf16x2(p0, p1);
  }
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
  const int h = static_cast<int>(blockIdx.x % a.kvh);
  const int G = a.gqa, TPT = a.tokens_per_tile;

  // ---- which request and pair of q-tiles (pairs never straddle requests).
  // Blocks start in index order: the KV head is the fastest-moving index and
  // each request's pairs are taken last-first (causal: the last pairs see the
  // most keys), so the longest work items start first and the last wave is
  // made of short ones.
  int r = -1, pair = 0;
  {
    const int rank = static_cast<int>(blockIdx.x / a.kvh);
    int acc = 0;
    for (int i = 0; i < a.num_reqs; ++i) {
      const int ql = a.cu_q[i + 1] - a.cu_q[i];
      const int nt = ql > 0 ? (ql + TPT - 1) / TPT : 0;
      const int np = (nt + 1) / 2;
      if (rank < acc + np) {
        r = i;
        pair = np - 1 - (rank - acc);
        break;
      }
      acc += np;
    }
  }
  if (r < 0) return;  // uniform: past the last pair
  const int q_begin = a.cu_q[r], q_len = a.cu_q[r + 1] - q_begin;
  const int k_begin = a.cu_k[r], k_len = a.cu_k[r + 1] - k_begin;
  const int tile0 = 2 * pair;                   // q-tile index of warpgroup 0
  const bool has1 = (tile0 + 1) * TPT < q_len;  // q-tile 1 holds live queries
  const int nq = has1 ? 2 : 1;
  const int off = k_len - q_len;                // causal alignment
  const int last_qi = min((tile0 + nq) * TPT, q_len) - 1;
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
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_hi[t], kSoftmaxThreads / 2);
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
      mbar_expect_tx(&sm.q_full, static_cast<uint32_t>(sizeof(sm.q[0]) * nq));
      for (int t = 0; t < nq; ++t)
        for (int b = 0; b < 2; ++b)
          tma_load_3d(&sm.q[t][b][0][0], &tmap_q, 64 * b, h * G, q0 + t * TPT, &sm.q_full);
      constexpr uint32_t kTileBytes = 2 * kKTile * 64 * 2;
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_tiles && !timed_out; ++j) {
        const int s = j % kStages;
        const uint32_t par = static_cast<uint32_t>((j / kStages - 1) & 1);
        const int z = k_begin + j * kKTile;
        if (j >= kStages && !mbar_wait(&sm.k_empty[s], par)) {
          timed_out = true;
          break;
        }
        mbar_expect_tx(&sm.k_full[s], kTileBytes);
        for (int b = 0; b < 2; ++b) tma_load_3d(&sm.k[s][b][0][0], &tmap_k, 64 * b, h, z, &sm.k_full[s]);
        issued_k = j + 1;
        if (j >= kStages && !mbar_wait(&sm.v_empty[s], par)) {
          timed_out = true;
          break;
        }
        mbar_expect_tx(&sm.v_full[s], kTileBytes);
        for (int b = 0; b < 2; ++b) tma_load_3d(&sm.v[s][b][0][0], &tmap_v, 64 * b, h, z, &sm.v_full[s]);
        issued_v = j + 1;
      }
      // every copy this CTA started lands before the CTA leaves
      for (int j = max(0, issued_k - kStages); j < issued_k; ++j)
        if (!mbar_wait(&sm.k_full[j % kStages], static_cast<uint32_t>((j / kStages) & 1))) timed_out = true;
      for (int j = max(0, issued_v - kStages); j < issued_v; ++j)
        if (!mbar_wait(&sm.v_full[j % kStages], static_cast<uint32_t>((j / kStages) & 1))) timed_out = true;
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
                       tc::smem_desc_sw128(k_addr + kb * 16384 + ks * 32, 16, 1024), id_qk,
                       (kb | ks) != 0 ? 1u : 0u);
        tc::mma_commit(&sm.s_full[t]);
      };
      // P.V over keys 64-127 (hi) or 0-63; the hi half is issued first, so
      // its first step starts O at tile 0
      auto issue_pv = [&](int t, int j, bool hi) {
        const uint32_t v_addr = smem_u32(&sm.v[j % kStages][0][0][0]);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {  // 16 keys per step: 8 columns of packed bf16 P
          const int ks = hi ? 4 + k4 : k4;
          tc::mma_ts(tbase + o_col(t), tbase + s_col(t) + 64 + 8 * ks,
                     tc::smem_desc_sw128(v_addr + ks * 16 * 128, 16384, 1024), id_pv,
                     (j > 0 || ks != 4) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&sm.q_full, 0) && mbar_wait(&sm.k_full[0], 0);
      tc::fence_after_sync();
      if (ok) {
        for (int t = 0; t < nq; ++t) issue_s(t, 0);
        tc::mma_commit(&sm.k_empty[0]);  // K_0 read by both S MMAs
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const bool next = j + 1 < n_tiles;
        if (!(ok = mbar_wait(&sm.v_full[j % kStages], static_cast<uint32_t>((j / kStages) & 1)))) break;
        // q-tile 0: P_0(j).V_j, then S_0(j + 1) while warpgroup 1 works
        if (!(ok = mbar_wait(&sm.p_hi[0], static_cast<uint32_t>(j & 1)))) break;
        tc::fence_after_sync();
        issue_pv(0, j, true);  // while warpgroup 0 turns keys 0-63 into P
        if (!(ok = mbar_wait(&sm.p_ready[0], static_cast<uint32_t>(j & 1)))) break;
        tc::fence_after_sync();
        issue_pv(0, j, false);
        if (next) {
          const int s1 = (j + 1) % kStages;
          if (!(ok = mbar_wait(&sm.k_full[s1], static_cast<uint32_t>(((j + 1) / kStages) & 1)))) break;
          tc::fence_after_sync();
          issue_s(0, j + 1);
        }
        if (has1) {
          if (!(ok = mbar_wait(&sm.p_hi[1], static_cast<uint32_t>(j & 1)))) break;
          tc::fence_after_sync();
          issue_pv(1, j, true);
          if (!(ok = mbar_wait(&sm.p_ready[1], static_cast<uint32_t>(j & 1)))) break;
          tc::fence_after_sync();
          issue_pv(1, j, false);
        }
        tc::mma_commit(&sm.v_empty[j % kStages]);  // V_j read by both P.V MMAs
        if (next) {
          if (has1) issue_s(1, j + 1);
          tc::mma_commit(&sm.k_empty[(j + 1) % kStages]);  // K_{j+1} read by both S MMAs
        }
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
      // Two phases over S_t. (1) The row max over the tile's 128 scores:
      // chunks 0-1, then chunks 2-3, which stay in registers. A row whose max
      // passes the running max by more than kLazyMax (log2 units) rescales O
      // (earlier tiles), once per tile and before any P of the tile exists;
      // after the first tiles of a row that is rare. (2) P for chunks 2-3, then
      // for chunks 0-1 loaded again. bf16 P goes to S_t's upper 64 columns (key
      // k at column 64 + k / 2), whose scores are in registers by then. Only a
      // tile that reaches past some row's causal end masks.
      const bool full_tile = __all_sync(0xffffffffu, (j + 1) * kKTile <= row_end);
      const int lim = row_end - j * kKTile;  // scores at columns >= lim are masked
      const uint32_t s_addr = t_row + s_col(t);
      uint32_t sa[32], sb[32];
      float cm[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
      tc::tmem_ld32_async(s_addr, sa);
      tc::tmem_ld32_async(s_addr + 32, sb);
      tc::tmem_wait_ld_into(sa);
      tc::tmem_wait_ld_into(sb);
      if (!full_tile) {
        mask_scores(sa, lim);
        mask_scores(sb, lim - 32);
      }
      max_scores(cm, sa);
      max_scores(cm, sb);
      tc::tmem_ld32_async(s_addr + 64, sa);
      tc::tmem_ld32_async(s_addr + 96, sb);
      tc::tmem_wait_ld_into(sa);
      tc::tmem_wait_ld_into(sb);
      if (!full_tile) {
        mask_scores(sa, lim - 64);
        mask_scores(sb, lim - 96);
      }
      max_scores(cm, sa);
      max_scores(cm, sb);
      const float cmax = fmaxf(max3f(cm[0], cm[1], cm[2]), cm[3]) * a.scale_log2;
      const bool grow = cmax > m_run + kLazyMax;
      if (__any_sync(0xffffffffu, grow)) {
        // m_run = -inf (nothing seen yet) gives alpha = 0: nothing to keep
        const float alpha = grow ? fast_exp2(m_run - cmax) : 1.0f;
        // S_t(j) is complete, so is every earlier MMA of this q-tile: O_t
        // is free to touch
        if (j > 0) {
#pragma unroll
          for (int cb = 0; cb < 4; ++cb) {
            uint32_t ov[32];
            tc::tmem_ld32(t_row + o_col(t) + 32 * cb, ov);
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tc::tmem_st32(t_row + o_col(t) + 32 * cb, ov);
          }
        }
        l_run *= alpha;
        if (grow) m_run = cmax;
      }
      const float neg_m = m_run == -CUDART_INF_F ? 0.0f : -m_run;
      const unsigned long long sc2 = f2_pack(a.scale_log2, a.scale_log2), nm2 = f2_pack(neg_m, neg_m);
      // row sums as 4 packed pairs (one f32x2 add per pair of scores)
      unsigned long long ps2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[16];
      exp_scores(sa, sc2, nm2, ps2, pk);
      tc::tmem_st16(s_addr + 96, pk);
      tc::tmem_ld32_async(s_addr, sa);  // chunk 0 again (its columns never hold P)
      exp_scores(sb, sc2, nm2, ps2, pk);
      tc::tmem_st16(s_addr + 112, pk);
      tc::tmem_ld32_async(s_addr + 32, sb);
      tc::tmem_wait_ld_into(sa);
      tc::tmem_wait_ld_into(sb);
      if (!full_tile) {
        mask_scores(sa, lim);
        mask_scores(sb, lim - 32);
      }
      exp_scores(sa, sc2, nm2, ps2, pk);
      // P of keys 64-127 (and any O rescale) is in tensor memory: the MMA
      // warp starts their P.V while this thread finishes keys 0-63
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive_local(&sm.p_hi[t]);
      tc::tmem_st16(s_addr + 64, pk);
      exp_scores(sb, sc2, nm2, ps2, pk);
      tc::tmem_st16(s_addr + 80, pk);
      float ps[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) f2_unpack(ps2[i], ps[2 * i], ps[2 * i + 1]);
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      tc::tmem_wait_st();
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
  const int64_t pairs_upper = ((total_q + tpt - 1) / tpt + num_reqs + 1) / 2 + num_reqs;
  if (pairs_upper * kvh > 0x7FFFFFFFll) return set_error(QKV_ERR_INVALID, "qkv_dense_prefill: too many q-tiles");
  dim3 grid(static_cast<unsigned>(pairs_upper * kvh));
  prefill_tc_kernel<<<grid, kThreads, kPrefillSmem, stream>>>(a, tq, tk, tv);
  QKV_CHECK_LAUNCH("prefill_tc_kernel");
  return QKV_OK;
}

}  // namespace qkv
