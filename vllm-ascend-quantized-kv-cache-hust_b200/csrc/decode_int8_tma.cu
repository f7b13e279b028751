// INT8 paged decode, page-pipelined (head 128, page 128, up to 8 query heads
// per KV head).
//
// One CTA of 4 warps owns (request, kv head, split) and streams the split's
// pages through a 2-stage shared-memory ring (a ring of 4 half-page stages
// measured 11 % slower: more ring bookkeeping, one m-tile per warp per
// stage). Thread 0 issues each page with two TMA tensor copies (the page's K
// and V rows of this head, 128 tokens x 128 B each, written with the 128-byte
// swizzle) that complete on the stage's "full" mbarrier; every warp arrives
// on the stage's "empty" mbarrier when it is done with it, and thread 0
// waits for that before refilling the stage. Warp w computes tokens
// [32w, 32w + 32) of every page:
//     S^T[token][head] = K[token][channel] . Q'^T[channel][head]
//     O^T[dim][head]  += V^T[dim][token]   . P^T[token][head]
// with mma.sync m16n8k16 (bf16 x bf16 -> fp32), the query heads of the KV head
// as N. The operands are the reference's dequantised values: its dense
// dequantisation (methods/int8_dynamic/attention_backend.py:398-401) computes
// code.to(bf16) * (1 / inv) in bf16, i.e. bf16(code * aq) with one rounding,
// and that is what enters both MMAs here (i8_bf16_neg: four instructions per
// pair of codes, the per-channel aq pairs held in registers). The query is
// the MMA's other operand as is (bf16, exact); softmax_scale * log2(e)
// multiplies the fp32 scores. P enters the PV MMA as two bf16 operands
// (hi + lo, ~16 significant bits).
//
// Both dequantised operands are produced negated (it saves an instruction per
// pair); the query fragments are negated to match and the output is negated
// once at the end.
//
// Rows of an m-tile: row g (and g + 8) of m-tile i of warp w is page token
// 32 w + 16 i + perm(g) (+ 8), perm = 0 4 3 7 5 1 6 2. With the TMA's 128-byte
// swizzle (16-byte chunk c of row r stored at chunk c ^ (r & 7)), this order
// makes the key loads (16 bytes) and the value loads (4 bytes) free of bank
// conflicts; every swizzled offset is precomputed per thread.
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
constexpr int kStageTok = 128;                // tokens per ring stage (one page)
constexpr int kHalves = kBlk / kStageTok;     // stages per page
constexpr int kTokW = kStageTok / kWarps;     // tokens per warp per stage
constexpr int kJ = kTokW / 16;                // score m-tiles per warp per stage
constexpr int kMaxPages = 64;
constexpr int kStages = 2;
constexpr float kLazy = 4.0f;            // log2 headroom of the running max
constexpr uint32_t kPerm8 = 0x26157340u;  // perm(g) = nibble g

struct __align__(1024) Int8Stage {
  unsigned char k[kStageTok][kD];  // 128-byte rows, 128-byte swizzle
  unsigned char v[kStageTok][kD];
};
static_assert(kJ >= 1 && kTokW % 16 == 0 && kBlk % kStageTok == 0, "stage geometry");

struct __align__(1024) Int8Shared {
  Int8Stage st[kStages];
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
  int pid[kMaxPages];
};
constexpr size_t kInt8SmemBytes = sizeof(Int8Shared) + 1024;  // + base alignment

__device__ __forceinline__ int perm8(int g) { return (kPerm8 >> (4 * g)) & 7; }

__device__ __forceinline__ uint32_t lds32(const unsigned char* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__global__ void __launch_bounds__(kThreads, 3)
int8_decode_tma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ unsigned char smem_raw[];
  // the 128-byte swizzle repeats every 1024 bytes: align the ring to that
  const uint32_t raw = smem_u32(smem_raw);
  Int8Shared& sh = *reinterpret_cast<Int8Shared*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
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
  const int n_steps = t1 > t0 ? min((t1 - t0 + kStageTok - 1) / kStageTok, kMaxPages * kHalves) : 0;

  for (int i = tid; i < n_pages; i += kThreads)
    sh.pid[i] = static_cast<int>(page_of(p, b, t0 + i * kBlk));
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], kWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }

  // ---- -q for head g and the k_aq pairs of this thread's channels, once per
  // CTA. k-step kk uses word m = 4t + kk (kk < 4) or 16 + 4t + kk - 4 of a key
  // row: channels 4m (k 2t), 4m + 2 (k 2t+1), 4m + 1 (k 2t+8), 4m + 3 (k 2t+9)
  uint32_t bq[8][2], kaq[8][2];
  {
    const uint16_t* qrow = reinterpret_cast<const uint16_t*>(p.q) + static_cast<int64_t>(b) * p.q_stride +
                           (static_cast<int64_t>(h) * G + g) * kD;
    const uint16_t* aq = reinterpret_cast<const uint16_t*>(p.k_aq) + static_cast<int64_t>(h) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int m = kk < 4 ? 4 * t + kk : 16 + 4 * t + kk - 4;
      uint32_t qq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qq[i] = g < G ? static_cast<uint32_t>(qrow[4 * m + i]) ^ 0x8000u : 0u;
      bq[kk][0] = qq[0] | (qq[2] << 16);
      bq[kk][1] = qq[1] | (qq[3] << 16);
      kaq[kk][0] = static_cast<uint32_t>(aq[4 * m]) | (static_cast<uint32_t>(aq[4 * m + 2]) << 16);
      kaq[kk][1] = static_cast<uint32_t>(aq[4 * m + 1]) | (static_cast<uint32_t>(aq[4 * m + 3]) << 16);
    }
  }
  // v_aq of this thread's dims: m-tile (wq, jb) rows g -> dim 4 (g + 8 wq) + 2 jb,
  // rows g + 8 -> that + 1 (both halves of a pair: the same dim)
  uint32_t vaq[8][2];
  {
    const uint16_t* aq = reinterpret_cast<const uint16_t*>(p.v_aq) + static_cast<int64_t>(h) * kD;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d_lo = 4 * (g + 8 * (mt >> 1)) + 2 * (mt & 1);
      vaq[mt][0] = static_cast<uint32_t>(aq[d_lo]) * 0x00010001u;
      vaq[mt][1] = static_cast<uint32_t>(aq[d_lo + 1]) * 0x00010001u;
    }
  }
  __syncthreads();

  auto issue = [&](int ii) {  // thread 0: half page ii of the split
    const int s = ii % kStages;
    const int pg = sh.pid[ii / kHalves];
    if (pg >= 0) {
      const int row = pg * kBlk + (ii % kHalves) * kStageTok;
      mbar_expect_tx(&sh.full[s], static_cast<uint32_t>(sizeof(Int8Stage)));
      tma_load_3d(&sh.st[s].k[0][0], &tmap_k, 0, h, row, &sh.full[s]);
      tma_load_3d(&sh.st[s].v[0][0], &tmap_v, 0, h, row, &sh.full[s]);
    } else {
      mbar_arrive(&sh.full[s]);
    }
  };
  if (tid == 0)
    for (int ii = 0; ii < kStages - 1 && ii < n_steps; ++ii) issue(ii);

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

  for (int i = 0; i < n_steps; ++i) {
    const int s = i % kStages;
    const int nx = i + kStages - 1;
    if (tid == 0 && nx < n_steps) {
      // the stage of step nx held step nx - kStages = i - 1: all warps must be done with it
      if (nx >= kStages &&
          !mbar_wait(&sh.empty[nx % kStages], static_cast<uint32_t>((nx / kStages - 1) & 1)))
        timed_out = true;
      issue(nx);
    }
    const bool ok = mbar_wait(&sh.full[s], static_cast<uint32_t>((i / kStages) & 1));
    timed_out |= !ok;
    const int pg = sh.pid[i / kHalves];
    const int pos0 = t0 + i * kStageTok;
    const int valid = min(kStageTok, t1 - pos0) - kTokW * warp;  // live tokens of this warp
    if (ok && pg >= 0 && valid > 0) {
      const unsigned char* kpage = &sh.st[s].k[0][0];
      const unsigned char* vpage = &sh.st[s].v[0][0];

      // ---- scores (unscaled): m-tile j, rows g / g + 8 -> tokens 16 (kJ w + j) + P (+ 8)
      float sc[kJ][4];
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
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
          mma16816_bf16(sc[j], i8_bf16_neg(x0, kaq[kk][0]), i8_bf16_neg(x1, kaq[kk][0]),
                        i8_bf16_neg(x0 >> 8, kaq[kk][1]), i8_bf16_neg(x1 >> 8, kaq[kk][1]), bq[kk][0],
                        bq[kk][1]);
        }
      }
      if (valid < kTokW) {
#pragma unroll
        for (int j = 0; j < kJ; ++j) {
          const bool lo_ok = 16 * j + P < valid, hi_ok = 16 * j + 8 + P < valid;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (!lo_ok) sc[j][e] = -CUDART_INF_F;
            if (!hi_ok) sc[j][2 + e] = -CUDART_INF_F;
          }
        }
      }

      // ---- online softmax over heads 2t, 2t+1 in log2 units (scores times
      // softmax_scale * log2 e, folded into the exponent's FMA), lazy rescale
      float mx[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mx[e] = fmaxf(sc[0][e], sc[0][2 + e]);
#pragma unroll
        for (int j = 1; j < kJ; ++j) mx[e] = fmaxf(mx[e], fmaxf(sc[j][e], sc[j][2 + e]));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
        mx[e] *= p.scale_log2;
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
      uint32_t pb[kJ][2], pl[kJ][2];  // P^T fragments: bf16 hi and lo parts
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
        float pr[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) pr[c] = fast_exp2(fmaf(sc[j][c], p.scale_log2, -m_run[c & 1]));
        l_run[0] += pr[0] + pr[2];
        l_run[1] += pr[1] + pr[3];
        uint32_t h0, l0, h1, l1;
        split_bf162(pr[0], pr[1], h0, l0);
        split_bf162(pr[2], pr[3], h1, l1);
        pb[j][0] = movmatrix_t(h0);
        pb[j][1] = movmatrix_t(h1);
        pl[j][0] = movmatrix_t(l0);
        pl[j][1] = movmatrix_t(l1);
      }

      // ---- O'^T += V^T . P^T; k-step j: k (2t, 2t+1) = rows (A, B) of m-tile
      // j, (2t+8, 2t+9) their + 8; dim m-tile (wq, jb): rows g -> byte 2 jb of
      // word g + 8 wq, rows g + 8 -> byte 2 jb + 1
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const unsigned char* ra = vpage + v_rowA + 16 * j * kD;
        const unsigned char* rb = vpage + v_rowB + 16 * j * kD;
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          const uint32_t va0 = lds32(ra + v_off[wq]), va1 = lds32(rb + v_off[wq ^ 2]);
          const uint32_t vc0 = lds32(ra + 8 * kD + v_off[wq]), vc1 = lds32(rb + 8 * kD + v_off[wq ^ 2]);
#pragma unroll
          for (int jb = 0; jb < 2; ++jb) {
            const uint32_t sel = static_cast<uint32_t>((2 * jb) | ((2 * jb + 1) << 4) |
                                                       ((4 + 2 * jb) << 8) | ((5 + 2 * jb) << 12));
            const uint32_t xa = __byte_perm(va0, va1, sel);
            const uint32_t xc = __byte_perm(vc0, vc1, sel);
            const int mt = 2 * wq + jb;
            const uint32_t a0 = i8_bf16_neg(xa, vaq[mt][0]), a1 = i8_bf16_neg(xa >> 8, vaq[mt][1]);
            const uint32_t a2 = i8_bf16_neg(xc, vaq[mt][0]), a3 = i8_bf16_neg(xc >> 8, vaq[mt][1]);
            mma16816_bf16(o[mt], a0, a1, a2, a3, pb[j][0], pb[j][1]);
            mma16816_bf16(o[mt], a0, a1, a2, a3, pl[j][0], pl[j][1]);
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
      // the value operands were negated
      mo[(warp * kHeads + head) * kD + d_lo] = -o[mt][e];
      mo[(warp * kHeads + head) * kD + d_lo + 1] = -o[mt][2 + e];
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

static_assert(sizeof(Int8Stage) * kStages >=
                  sizeof(float) * (kWarps * kHeads * kD + 2 * kWarps * kHeads),
              "merge buffers must fit in the stage memory");

// INT8 pages [NB, block, KVH, D] as a 3-D map {D bytes, KVH, NB * block} with
// the 128-byte swizzle; one box = the token rows of one ring stage of one head.
int encode_int8_map(const int8_t* base, const DecodeParams& p, CUtensorMap* map) {
  auto enc = encode_fn();
  if (enc == nullptr) return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.kvh),
                              static_cast<cuuint64_t>(p.num_blocks) * kBlk};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kD) * p.kvh};
  const cuuint32_t box[3] = {kD, 1, kStageTok};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides,
                         box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled(int8 pages) failed: " + std::to_string(r));
  return QKV_OK;
}

}  // namespace

bool int8_tma_geometry(const DecodeParams& p) {
  return p.head_size == kD && p.blk == kBlk && p.gqa >= 1 && p.gqa <= kHeads;
}

bool int8_tma_supported(const DecodeParams& p) {
  const auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  return int8_tma_geometry(p) && p.num_blocks > 0 &&
         static_cast<int64_t>(p.num_blocks) * kBlk < (int64_t{1} << 31) && al(p.kc) && al(p.vc);
}

// Split count that best fills the last wave of resident CTAs (3 per SM),
// pages per split <= kMaxPages, a 0.4 % charge per split for the combine.
SplitPlan plan_int8_tma(int batch, int kvh, int max_seq_len, int sms) {
  SplitPlan plan;
  const int pages = max_seq_len > 0 ? (max_seq_len + kBlk - 1) / kBlk : 1;
  const int units = batch * kvh > 0 ? batch * kvh : 1;
  const int resident = sms * 3;
  const int s_min = (pages + kMaxPages - 1) / kMaxPages;
  int s_max = (8 * resident + units - 1) / units;
  s_max = s_max < s_min ? s_min : s_max;
  s_max = s_max > pages ? pages : s_max;
  double best_score = -1.0;
  int best_pps = pages;
  for (int s = s_min; s <= s_max; ++s) {
    const int pps = (pages + s - 1) / s;
    if (pps > kMaxPages) continue;
    const int se = (pages + pps - 1) / pps;
    const long long grid = static_cast<long long>(units) * se;
    const long long waves = (grid + resident - 1) / resident;
    const double eff = static_cast<double>(grid) / static_cast<double>(waves * resident);
    const double score = eff - 0.004 * se;
    if (score > best_score + 1e-9) {
      best_score = score;
      best_pps = pps;
    }
  }
  plan.split_tokens = best_pps * kBlk;
  plan.hist_splits = (pages + best_pps - 1) / best_pps;
  plan.total = plan.hist_splits;
  return plan;
}

int launch_int8_tma(const DecodeParams& p, cudaStream_t stream) {
  CUtensorMap tk, tv;
  int rc = encode_int8_map(p.kc, p, &tk);
  if (rc != QKV_OK) return rc;
  if ((rc = encode_int8_map(p.vc, p, &tv)) != QKV_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(int8_decode_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kInt8SmemBytes));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(int8_decode_tma_kernel)");
    attr.fetch_or(bit);
  }
  dim3 grid(p.num_hist_splits, p.kvh, p.batch);
  int8_decode_tma_kernel<<<grid, kThreads, kInt8SmemBytes, stream>>>(p, tk, tv);
  QKV_CHECK_LAUNCH("int8_decode_tma_kernel");
  if (p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
