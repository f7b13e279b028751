// KIVI paged decode, page-pipelined version (production geometry: head_size
// 128, page size 128, group 64/128, up to 8 query heads per KV head).
//
// One CTA of 4 warps owns (request, kv head, history split) and streams the
// split's pages through an S-stage ring in shared memory. Per page, one lane
// issues the copies with the Tensor Memory Accelerator:
//     k_quant  one box {16 words, 128 channels} (8 KB, 64-byte rows)
//     v_quant  one box {16 words, 1 head, 32 quads, 4} (8 KB, 64-byte rows)
//     k_scale, k_mn  one bulk copy each (contiguous per page and head)
// and the lanes of the same warp (warp = page % 4) copy the v_scale / v_mn of
// 4 tokens each with cp.async; all of it completes on the stage's mbarrier.
// Both code tiles use the 64-byte swizzle. Warp w computes tokens
// [32w, 32w + 32) of every page:
//     S^T[token][head] = K[token][channel] . Q'^T[channel][head]
//     O^T[dim][head]  += V^T[dim][token]   . P'^T[token][head]
// with mma.sync m16n8k16 (fp16 x fp16 -> fp32), the 8 query heads of the KV
// head as N. Q' = q * k_scale * softmax_scale * log2(e) (and the per-head
// constant sum_d q k_mn) depend only on the page and group, so the CTA builds
// them once per page into shared memory, already in B-fragment order.
//
// int4 -> fp16: ldmatrix.trans reads the packed codes as 16-bit elements (4
// nibbles each) and hands every lane the element of two adjacent rows in one
// register, i.e. the (row, k) / (row, k + 1) pair of an A fragment; masking
// nibble i of both halves (one AND) makes fp16 subnormals n * 2^-24 (16 n *
// 2^-24 for nibble 1), which the MMA takes exactly. Nibbles 2 and 3 first
// move down a byte with zeros above (one PRMT per register); nibble 3's rows
// then take the whole byte n2 + 16 n3 unmasked and lose the n2 part
// afterwards (hi_bytes). Scales fold into the other operand:
//     K: S = S' / f + sum_d q[h][d] k_mn[d][group]
//     V: P'[t][h] = p[t][h] * v_scale[t][group],
//        O = O' / f + sum_t p[t][h] v_mn[t][group]
// so the dequantised values enter exactly (code * scale + min in real
// arithmetic), without the bf16 rounding of a dense gather.
//
// Token placement inside a warp's 32 tokens: a 16-bit element of a key row
// holds the 4 tokens 4e .. 4e + 3 of one channel, so score m-tile j, row g is
// token 4g + 2j and row g + 8 token 4g + 2j + 1. The PV k-step j then takes
// tokens {4r + 2j} (k 0..7) and {4r + 2j + 1} (k 8..15). The value tile's TMA
// copy therefore views the page's tokens as [token % 4][token / 4] (a 4-D map
// with the token-in-quad dimension outermost), so each such set is 8
// consecutive 64-byte rows, and the 64-byte swizzle spreads them over all 8
// bank groups (likewise 8 consecutive key channels).
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
constexpr int kTokW = kBlk / kWarps;  // tokens per warp per page
constexpr int kMaxPages = 64;         // pages per split (ids staged in smem)
constexpr int kStages = 2;
// The int4 codes enter the MMAs as fp16 SUBNORMALS: masking a nibble into the
// low mantissa bits of an fp16 half gives n * 2^-24 exactly (n * 16 * 2^-24
// for a high nibble), one AND per pair and no bias to remove. The tensor core
// takes subnormal inputs exactly; the fp32 accumulators are scaled back once.
constexpr float kUnsub = 16777216.0f;        // 2^24: low-nibble rows
constexpr float kUnsubHi = 1048576.0f;       // 2^20: high-nibble rows (2^24 / 16)
__device__ __forceinline__ uint32_t nib_lo_sub(uint32_t x) { return x & 0x000F000Fu; }
__device__ __forceinline__ uint32_t nib_hi_sub(uint32_t x) { return x & 0x00F000F0u; }
// Bytes 1 and 3 of x moved down to bytes 0 and 2, zeros above: each half is
// the whole byte n2 + 16 n3 as an fp16 subnormal, (n2 + 16 n3) * 2^-24. As the
// operand of the rows that want nibble 3 it saves their AND; the n2 part is
// taken off the accumulator afterwards (the rows that want nibble 2 hold
// exactly it, in the same lane and column).
__device__ __forceinline__ uint32_t hi_bytes(uint32_t x) { return __byte_perm(x, 0u, 0x4341u); }
constexpr float kLazy = 4.0f;  // log2 headroom of the running max

template <int NG>
struct __align__(1024) PageStage {
  uint32_t k[kD][16];         // [channel][word], 64-byte swizzle (see koff)
  uint32_t v[kBlk][16];       // [token % 4][token / 4][word], 64-byte swizzle (see voff)
  float ks[kD * NG];          // [channel][group]
  float km[kD * NG];
  float vs[kBlk * NG];        // [token][group]
  float vm[kBlk * NG];
};

template <int NG>
struct __align__(1024) PageShared {
  PageStage<NG> st[kStages];
  uint4 qf[2][NG][kWarps][32];     // Q' B fragments: [buffer][group][k-step pair][lane]
  float cmn[2][NG][kWarps][kHeads];  // partial sum_d q k_mn: [buffer][group][k-step pair][head]
  float vsv[2][kBlk * NG];           // the page's value scales / minima, copied out of the
  float vmv[2][kBlk * NG];           // stage so it can refill while the page is computed
  unsigned long long full[kStages];
  int pid[kMaxPages];
};

// the code tiles of every stage start on 1024-byte boundaries (a multiple of
// the 512-byte period of the 64-byte swizzle)
static_assert(sizeof(PageStage<1>) % 1024 == 0 && sizeof(PageStage<2>) % 1024 == 0, "stage size");
static_assert(offsetof(PageStage<1>, v) % 1024 == 0 && offsetof(PageStage<2>, v) % 1024 == 0 &&
                  offsetof(PageStage<1>, k) == 0 && offsetof(PageStage<2>, k) == 0,
              "code tile alignment");
// dynamic shared memory of one CTA: the struct plus room to round its base up
template <int NG>
constexpr size_t kivi_smem_bytes() {
  return sizeof(PageShared<NG>) + 1024;
}

// The 64-byte swizzle (address bits [4,6) ^= bits [7,9)) on 64-byte rows:
// 16-byte chunk c of row r sits at 64 r + 16 (c ^ ((r >> 1) & 3)).
// Key tile: row = channel, chunk = token quarter (8 tokens per word).
__device__ __forceinline__ uint32_t koff(int ch, int c) {
  return static_cast<uint32_t>(64 * ch + 16 * (c ^ ((ch >> 1) & 3)));
}
// Value tile: row 32 (tok % 4) + tok / 4 for page token tok, chunk = 32 dims.
__device__ __forceinline__ uint32_t voff(int tok, int c) {
  const int row = 32 * (tok & 3) + (tok >> 2);
  return static_cast<uint32_t>(64 * row + 16 * (c ^ ((row >> 1) & 3)));
}

template <int NG>
constexpr uint32_t stage_tx_bytes() {
  return static_cast<uint32_t>(sizeof(uint32_t) * (kD * (kBlk / 8) + kBlk * (kD / 8)) +
                               2 * sizeof(float) * kD * NG);
}

// ------------------------------------------------------------ window tail

constexpr int kTailCtas = 2;    // extra CTAs per (request, kv head) for the window
constexpr int kTailBlock = 32;  // positions per tail step

// Key row `pos` of request b, channels 4 lane .. 4 lane + 3, in fp32: the bf16
// residual window for positions >= k_begin, else the int4 page.
__device__ __forceinline__ float4 tail_key4(const DecodeParams& p, const TailState& ts, int b,
                                           int h, int pos, int lane) {
  const int64_t kvh = p.kvh;
  if (pos >= ts.k_begin) {
    const int slot = (ts.k_start + (pos - ts.k_begin)) % p.res_cap;
    const __nv_bfloat16* row =
        p.rk + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * kD + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2*>(row);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    return make_float4(a.x, a.y, c.x, c.y);
  }
  int64_t page = -1;
  if (lane == 0) page = page_of(p, b, pos);
  page = __shfl_sync(0xffffffffu, page, 0);
  if (page < 0) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int off = pos % kBlk, ng = kBlk / p.group;
  float r[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t chan = (page * kvh + h) * kD + 4 * lane + k;
    const uint32_t w = static_cast<uint32_t>(p.kq[chan * (kBlk / 8) + (off >> 3)]);
    const int64_t si = chan * ng + off / p.group;
    r[k] = __fadd_rn(__fmul_rn(static_cast<float>((w >> (4 * (off & 7))) & 0xFu), p.ks[si]), p.km[si]);
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

// Value row `pos` of request b, dims 4 lane .. 4 lane + 3, in fp32 (window
// for positions >= v_begin, else the int4 page).
__device__ __forceinline__ float4 tail_value4(const DecodeParams& p, const TailState& ts, int b,
                                             int h, int pos, int lane) {
  const int64_t kvh = p.kvh;
  if (pos >= ts.v_begin) {
    const int slot = (ts.v_start + (pos - ts.v_begin)) % p.res_cap;
    const __nv_bfloat16* row =
        p.rv + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * kD + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2*>(row);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    return make_float4(a.x, a.y, c.x, c.y);
  }
  int64_t page = -1;
  if (lane == 0) page = page_of(p, b, pos);
  page = __shfl_sync(0xffffffffu, page, 0);
  if (page < 0) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int64_t vrow = (page * kBlk + pos % kBlk) * kvh + h;
  const uint32_t w = static_cast<uint32_t>(p.vq[vrow * (kD / 8) + (lane >> 1)]);
  const int64_t si = vrow * (kD / p.group) + (4 * lane) / p.group;  // 4 dims share a group
  const float sc = p.vs[si], mn = p.vm[si];
  float r[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t code = (w >> (4 * (4 * (lane & 1) + k))) & 0xFu;
    r[k] = __fadd_rn(__fmul_rn(static_cast<float>(code), sc), mn);
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

constexpr int kTailLd = kD + 4;  // padded fp32 row of the staged keys


// One tail CTA: positions [body_end, L) in blocks of kTailBlock, blocks
// c, c + n_tail, ...; its partial softmax state is split num_hist_splits + c.
// Each block's K and V rows are staged in shared memory (fp32) with
// independent 8-byte loads, then scored and accumulated from there; fp32
// CUDA-core math (the window is < 1% of the bytes).
__device__ __forceinline__ void window_tail(const DecodeParams& p, int c, int n_tail, int h, int b,
                                            unsigned char* smem) {
  grid_dependency_wait();  // the rings may still be written by the launch before (after_ring_write)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.gqa;
  float* kt = reinterpret_cast<float*>(smem);  // [kTailBlock][kTailLd]
  float* vt = kt + kTailBlock * kTailLd;        // [kTailBlock][kD]
  float* sc = vt + kTailBlock * kD;             // [kTailBlock][kHeads] scores, then probs
  float* st_m = sc + kTailBlock * kHeads;       // [kHeads]
  float* st_l = st_m + kHeads;
  float* st_a = st_l + kHeads;
  const int L = max(p.seq_lens[b], 0);
  const TailState ts = load_tail_state(p, b, L);
  const int body_end = min(ts.k_begin, ts.v_begin);
  if (body_end + kTailBlock * c >= L && p.splits_total > 1) {  // no block for this CTA
    empty_split(p, b, h, p.num_hist_splits + c);
    return;
  }

  // q * scale * log2(e), channels 4 lane .. 4 lane + 3 of every head
  float q[kHeads][4];
  const __nv_bfloat16* qrow =
      p.q + static_cast<int64_t>(b) * p.q_stride + static_cast<int64_t>(h) * G * kD + 4 * lane;
#pragma unroll
  for (int hd = 0; hd < kHeads; ++hd)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      q[hd][k] = hd < G ? __bfloat162float(qrow[hd * kD + k]) * p.scale_log2 : 0.0f;
  if (tid < kHeads) {
    st_m[tid] = -CUDART_INF_F;
    st_l[tid] = 0.0f;
  }
  float acc[kHeads];
#pragma unroll
  for (int hd = 0; hd < kHeads; ++hd) acc[hd] = 0.0f;
  // after the butterfly, lane holds the sum of head bit4 * 4 + bit3 * 2 + bit2
  const int my_head = (((lane >> 4) & 1) << 2) | (((lane >> 3) & 1) << 1) | ((lane >> 2) & 1);
  const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;

  for (int blk = c; body_end + kTailBlock * blk < L; blk += n_tail) {
    const int p0 = body_end + kTailBlock * blk;
    const int n = min(kTailBlock, L - p0);
    // ---- stage rows 8 warp .. 8 warp + 7 of K and V
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 8 * warp + i;
      float4 k4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), v4 = k4;
      if (r < n) {
        k4 = tail_key4(p, ts, b, h, p0 + r, lane);
        v4 = tail_value4(p, ts, b, h, p0 + r, lane);
      }
      *reinterpret_cast<float4*>(&kt[r * kTailLd + 4 * lane]) = k4;
      *reinterpret_cast<float4*>(&vt[r * kD + 4 * lane]) = v4;
    }
    __syncthreads();
    // ---- scores: warp w, positions 8 w .. 8 w + 7 of the block
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int r = 8 * warp + i;
      const float4 k4 = *reinterpret_cast<const float4*>(&kt[r * kTailLd + 4 * lane]);
      float part[kHeads];
#pragma unroll
      for (int hd = 0; hd < kHeads; ++hd)
        part[hd] = fmaf(q[hd][0], k4.x, fmaf(q[hd][1], k4.y, fmaf(q[hd][2], k4.z, q[hd][3] * k4.w)));
      // transpose-reduce the 8 head sums over the 32 lanes (9 shuffles)
      float h4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float keep = b4 ? part[k + 4] : part[k];
        const float send = b4 ? part[k] : part[k + 4];
        h4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
      float h2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float keep = b3 ? h4[k + 2] : h4[k];
        const float send = b3 ? h4[k] : h4[k + 2];
        h2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      float v;
      {
        const float keep = b2 ? h2[1] : h2[0];
        const float send = b2 ? h2[0] : h2[1];
        v = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      if ((lane & 3) == 0) sc[r * kHeads + my_head] = r < n ? v : -CUDART_INF_F;
    }
    __syncthreads();
    // ---- online softmax: warp w owns heads 2w, 2w + 1; lanes = positions
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hd = 2 * warp + e;
      const float v = sc[lane * kHeads + hd];
      float mx = v;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = st_m[hd];
      const float m_new = fmaxf(m_old, mx);
      const float pr = v == -CUDART_INF_F ? 0.0f : exp2f(v - m_new);
      float sum = pr;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sc[lane * kHeads + hd] = pr;
      __syncwarp();
      if (lane == 0) {
        const float alpha =
            m_new == -CUDART_INF_F ? 1.0f : (m_old == -CUDART_INF_F ? 0.0f : exp2f(m_old - m_new));
        st_m[hd] = m_new;
        st_l[hd] = st_l[hd] * alpha + sum;
        st_a[hd] = alpha;
      }
    }
    __syncthreads();
    // ---- P V: thread = dim
#pragma unroll
    for (int hd = 0; hd < kHeads; ++hd) acc[hd] *= st_a[hd];
    for (int j = 0; j < n; ++j) {
      const float v = vt[j * kD + tid];
      const float4 pa = *reinterpret_cast<const float4*>(&sc[j * kHeads]);
      const float4 pb = *reinterpret_cast<const float4*>(&sc[j * kHeads + 4]);
      acc[0] = fmaf(pa.x, v, acc[0]);
      acc[1] = fmaf(pa.y, v, acc[1]);
      acc[2] = fmaf(pa.z, v, acc[2]);
      acc[3] = fmaf(pa.w, v, acc[3]);
      acc[4] = fmaf(pb.x, v, acc[4]);
      acc[5] = fmaf(pb.y, v, acc[5]);
      acc[6] = fmaf(pb.z, v, acc[6]);
      acc[7] = fmaf(pb.w, v, acc[7]);
    }
    __syncthreads();
  }
  const int split = p.num_hist_splits + c;
#pragma unroll
  for (int hd = 0; hd < kHeads; ++hd)
    if (hd < G) store_partial(p, b, h * G + hd, split, tid, acc[hd], st_m[hd], st_l[hd]);
}

static_assert(sizeof(float) * (kTailBlock * (kTailLd + kD + kHeads) + 3 * kHeads) <=
                  sizeof(PageShared<1>),
              "tail staging must fit in the kernel's shared memory");

// ------------------------------------------------------------ the kernel

// Two schedules of the same page pipeline:
//  kEarly = false (large decodes): 5 CTAs per SM for group 128 (4 for group
//   64, shared memory); a page's stage refills after the page is computed,
//   so one page is in flight while another is computed.
//  kEarly = true (small decodes, where one page in flight per CTA leaves DRAM
//   idle): 4 CTAs per SM; a page's code fragments go to registers (ldmatrix)
//   and its value scales to a small side buffer before the CTA barrier, so
//   its stage refills at once and both stages are in flight while the page
//   is computed (32 more registers per thread).
template <int NG, bool kEarly>
__global__ void __launch_bounds__(kThreads, (NG == 1 && !kEarly) ? 5 : 4)
kivi_decode_tma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ unsigned char smem_dyn[];
  const uint32_t raw = smem_u32(smem_dyn);
  unsigned char* smem_raw = smem_dyn + (((raw + 1023u) & ~1023u) - raw);
  PageShared<NG>& sh = *reinterpret_cast<PageShared<NG>*>(smem_raw);
  const int n_tail = p.splits_total - p.num_hist_splits;  // window CTAs come first
  // grid (kv head, request, split) or, with split_mid (early schedule only),
  // (kv head, split, request): the heads of one (request, split) are
  // consecutive CTAs (see the launch)
  const bool mid = kEarly && p.split_mid;
  const int h = blockIdx.x;
  const int b = mid ? blockIdx.z : blockIdx.y, xs = mid ? blockIdx.y : blockIdx.z;
  if (xs < n_tail) {
    window_tail(p, xs, n_tail, h, b, smem_raw);
    return;
  }
  const int split = xs - n_tail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;
  const int kvh = p.kvh;

  // ---- the split's history range [t0, t1): positions before the window.
  // The block-table entry of page tid of the split is read alongside the
  // request's length and window state (it does not depend on them; kMaxPages
  // <= kThreads), and checked once the page count is known.
  static_assert(kMaxPages <= kThreads, "one block-table entry per thread");
  const int t0 = split * p.split_tokens;
  const int col = t0 / kBlk + tid;
  // past the table row: INT32_MAX, which fails the block-range check below
  // with the same error as an entry past the last block (this kernel takes
  // num_blocks * kvh * 128 < 2^31)
  const int32_t pg_raw = tid >= kMaxPages      ? -1
                         : col < p.bt_stride   ? p.bt[static_cast<int64_t>(b) * p.bt_stride + col]
                                               : 0x7fffffff;
  const int L = max(p.seq_lens[b], 0);
  const TailState ts = load_tail_state(p, b, L);
  const int body_end = min(ts.k_begin, ts.v_begin);
  const int t1 = min(body_end, t0 + p.split_tokens);
  const int n_pages = t1 > t0 ? min((t1 - t0 + kBlk - 1) / kBlk, kMaxPages) : 0;
  if (n_pages == 0 && p.splits_total > 1) {  // the request ends before this split
    empty_split(p, b, h, split);
    return;
  }

  if (tid < n_pages) {  // page_of's checks and errors on the entry read above
    int pg = -1;
    if (pg_raw < 0 || pg_raw >= p.num_blocks) {
      record_error(p.err, pg_raw < 0 ? kErrNegativeBlock : kErrBlock);
    } else {
      pg = static_cast<int>(pg_raw);
    }
    sh.pid[tid] = pg;
  }
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&sh.full[s], 32 + 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }

  // q of the Q' entries this thread builds: head g, channels
  // 16 (2 warp + e) + qch(r), qch = 2t, 2t + 1, 2t + 8, 2t + 9 (the B
  // fragment of k-steps 2 warp and 2 warp + 1)
  const auto qch = [t](int r) { return 2 * t + (r & 1) + 8 * (r >> 1); };
  float qv[8];
  {
    const __nv_bfloat16* qrow =
        p.q + static_cast<int64_t>(b) * p.q_stride + (static_cast<int64_t>(h) * G + g) * kD;
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int r = 0; r < 4; ++r)
        qv[4 * e + r] =
            g < G ? __bfloat162float(qrow[16 * (2 * warp + e) + qch(r)]) * p.scale_log2 : 0.0f;
  }
  __syncthreads();

  // Issues the copies of page ii into stage ii % kStages: warp ii % 4 only
  // (the stage's barrier counts its 32 lanes plus the expect-tx arrival).
  auto issue = [&](int ii) {
    if (warp != (ii & (kWarps - 1))) return;
    const int s = ii % kStages;
    PageStage<NG>& st = sh.st[s];
    const int pg = sh.pid[ii];
    if (pg >= 0) {
      if (lane == 0) {
        mbar_expect_tx(&sh.full[s], stage_tx_bytes<NG>());
        tma_load_2d(&st.k[0][0], &tmap_k, 0, (pg * kvh + h) * kD, &sh.full[s]);
        tma_load_4d(&st.v[0][0], &tmap_v, 0, h, pg * (kBlk / 4), 0, &sh.full[s]);
        const int64_t soff = (static_cast<int64_t>(pg) * kvh + h) * kD * NG;
        bulk_load(st.ks, p.ks + soff, sizeof(float) * kD * NG, &sh.full[s]);
        bulk_load(st.km, p.km + soff, sizeof(float) * kD * NG, &sh.full[s]);
      }
#pragma unroll
      for (int k = 0; k < kBlk / 32; ++k) {
        const int tk = lane + 32 * k;
        const int64_t so = ((static_cast<int64_t>(pg) * kBlk + tk) * kvh + h) * NG;
        cp_async_small<4 * NG>(&st.vs[tk * NG], p.vs + so);
        cp_async_small<4 * NG>(&st.vm[tk * NG], p.vm + so);
      }
      cp_async_arrive_noinc(&sh.full[s]);
    } else {
      if (lane == 0) mbar_arrive(&sh.full[s]);
      mbar_arrive(&sh.full[s]);
    }
  };

  constexpr int kAhead = kEarly ? kStages : kStages - 1;  // pages issued before the loop
#pragma unroll
  for (int i = 0; i < kAhead; ++i)
    if (i < n_pages) issue(i);

  // ---- per-warp running state: heads 2t, 2t+1 of this thread
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_run[2] = {0.0f, 0.0f};
  float mn_acc[2][NG];
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int gg = 0; gg < NG; ++gg) mn_acc[e][gg] = 0.0f;

  // token placement (see the file comment)
  int tok_j[2];  // local token of row g in m-tile j (row g + 8: + 1)
#pragma unroll
  for (int j = 0; j < 2; ++j) tok_j[j] = 4 * g + 2 * j;
  // ldmatrix rows of this lane: key channel 32 kp + lane (chunk = warp), value
  // token 4 (lane & 7) + (lane >> 3) of the warp's 32 (matrix lane >> 3 = token
  // set {4r + (lane >> 3)}), one offset per 32-dim block
  uint32_t kro[4], vro[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    kro[i] = koff(32 * i + lane, warp);
    vro[i] = voff(kTokW * warp + 4 * (lane & 7) + (lane >> 3), i);
  }
  const int grp = NG == 2 ? (warp >> 1) : 0;  // key group of this warp's tokens

  int consumed = 0;
  bool aborted = false;
  // late schedule: two pages per unrolled iteration make the stage and
  // buffer indices constants (2.4 % faster on config 5)
#pragma unroll(kEarly ? 1 : 2)
  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kStages;
    const uint32_t parity = static_cast<uint32_t>((i / kStages) & 1);
    const bool ok = mbar_wait(&sh.full[s], parity);
    const PageStage<NG>& st = sh.st[s];
    const int pg = sh.pid[i];
    const int qb = i & 1;
    // the page's key / value code fragments of this lane: matrices m = 0..3
    // of key block kp are channels 32 kp + 8 m .. + 7 (rows) x token quads
    // (columns); value block db is tokens {4r + d} x 32 dims of dim block db
    uint32_t kx[4][4], vx[4][4];
    const auto load_frags = [&]() {
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {
        ldsm_x4_t(kx[kp], reinterpret_cast<const unsigned char*>(&st.k[0][0]) + kro[kp]);
        ldsm_x4_t(vx[kp], reinterpret_cast<const unsigned char*>(&st.v[0][0]) + vro[kp]);
      }
    };
    if (pg >= 0 && ok) {
      if constexpr (kEarly) {
        load_frags();
        for (int e = tid; e < kBlk * NG; e += kThreads) {
          sh.vsv[qb][e] = st.vs[e];
          sh.vmv[qb][e] = st.vm[e];
        }
      }
      // Q' entries of k-steps 2 warp, 2 warp + 1 (lane = fragment owner):
      // channels qch(r) = 2t, 2t + 1, 2t + 8, 2t + 9 are two adjacent pairs,
      // so each pair's scales (and minima) of both groups come in one load
      float c[NG];
      uint32_t f[NG][4];
#pragma unroll
      for (int gq = 0; gq < NG; ++gq) c[gq] = 0.0f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int ch0 = 16 * (2 * warp + e) + 2 * t;
        float ks_[4][NG], km_[4][NG];  // [r][group]
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          const int ch = ch0 + 8 * hp;
          if constexpr (NG == 1) {
            const float2 a = *reinterpret_cast<const float2*>(&st.ks[ch]);
            const float2 m = *reinterpret_cast<const float2*>(&st.km[ch]);
            ks_[2 * hp][0] = a.x;
            ks_[2 * hp + 1][0] = a.y;
            km_[2 * hp][0] = m.x;
            km_[2 * hp + 1][0] = m.y;
          } else {
            const float4 a = *reinterpret_cast<const float4*>(&st.ks[ch * NG]);
            const float4 m = *reinterpret_cast<const float4*>(&st.km[ch * NG]);
            ks_[2 * hp][0] = a.x;
            ks_[2 * hp][NG - 1] = a.y;
            ks_[2 * hp + 1][0] = a.z;
            ks_[2 * hp + 1][NG - 1] = a.w;
            km_[2 * hp][0] = m.x;
            km_[2 * hp][NG - 1] = m.y;
            km_[2 * hp + 1][0] = m.z;
            km_[2 * hp + 1][NG - 1] = m.w;
          }
        }
#pragma unroll
        for (int gq = 0; gq < NG; ++gq) {
          float qq[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            qq[r] = qv[4 * e + r] * ks_[r][gq];
            c[gq] = fmaf(qv[4 * e + r], km_[r][gq], c[gq]);
          }
          f[gq][2 * e] = pack_half2(qq[0], qq[1]);
          f[gq][2 * e + 1] = pack_half2(qq[2], qq[3]);
        }
      }
#pragma unroll
      for (int gq = 0; gq < NG; ++gq) {
        sh.qf[qb][gq][warp][lane] = make_uint4(f[gq][0], f[gq][1], f[gq][2], f[gq][3]);
        float cc = c[gq];
        cc += __shfl_xor_sync(0xffffffffu, cc, 1);
        cc += __shfl_xor_sync(0xffffffffu, cc, 2);
        if (t == 0) sh.cmn[qb][gq][warp][g] = cc;
      }
    }
    if (!__syncthreads_and(ok ? 1 : 0)) {  // uniform: every thread leaves here
      if (tid == 0) record_error(p.err, kErrPipelineTimeout);
      aborted = true;
      consumed = i;
      break;
    }
    consumed = i + 1;
    // early: every warp holds page i in registers, so its stage refills now;
    // otherwise the stage of page i - 1 does
    if (i + kAhead < n_pages) issue(i + kAhead);
    if (pg < 0) continue;
    const int pos0 = t0 + i * kBlk;
    const int valid = min(kBlk, t1 - pos0) - kTokW * warp;  // live tokens of this warp
    if (valid <= 0) continue;

    // ---- B fragments of Q' and the per-head constants
    uint32_t bq[8][2];
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
      const uint4 v = sh.qf[qb][grp][kp][lane];
      bq[2 * kp][0] = v.x;
      bq[2 * kp][1] = v.y;
      bq[2 * kp + 1][0] = v.z;
      bq[2 * kp + 1][1] = v.w;
    }
    float cmn[2];
    {
      float2 c = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {
        const float2 v = *reinterpret_cast<const float2*>(&sh.cmn[qb][grp][kp][2 * t]);
        c.x += v.x;
        c.y += v.y;
      }
      cmn[0] = c.x;
      cmn[1] = c.y;
    }

    // ---- S'^T = K . Q'^T for the warp's two m-tiles
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
      if constexpr (!kEarly)  // late schedule: fragments straight from the stage, next to their use
        ldsm_x4_t(kx[kp], reinterpret_cast<const unsigned char*>(&st.k[0][0]) + kro[kp]);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kk = 2 * kp + e;
        const uint32_t x0 = kx[kp][2 * e], x1 = kx[kp][2 * e + 1];
        mma16816(sc[0], nib_lo_sub(x0), nib_hi_sub(x0), nib_lo_sub(x1), nib_hi_sub(x1), bq[kk][0], bq[kk][1]);
        const uint32_t y0 = hi_bytes(x0), y1 = hi_bytes(x1);
        mma16816(sc[1], nib_lo_sub(y0), y0, nib_lo_sub(y1), y1, bq[kk][0], bq[kk][1]);
      }
    }
    // m-tile 1's rows g + 8 took whole bytes (n2 + 16 n3): remove the n2 part
    sc[1][2] -= sc[1][0];
    sc[1][3] -= sc[1][1];
    // scores in log2 units: [j][0..1] low-nibble token, heads 2t, 2t+1; [j][2..3] its +1
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[j][e] = fmaf(sc[j][e], kUnsub, cmn[e]);
        sc[j][2 + e] = fmaf(sc[j][2 + e], kUnsubHi, cmn[e]);
      }
    const bool partial = valid < kTokW;
    if (partial) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const bool lo_ok = tok_j[j] < valid, hi_ok = tok_j[j] + 1 < valid;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (!lo_ok) sc[j][e] = -CUDART_INF_F;
          if (!hi_ok) sc[j][2 + e] = -CUDART_INF_F;
        }
      }
    }

    // ---- online softmax over heads 2t, 2t+1 (max over the warp's tokens)
    float mx[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mx[e] = fmaxf(fmaxf(sc[0][e], sc[0][2 + e]), fmaxf(sc[1][e], sc[1][2 + e]));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
    }
    // lazy rescale: the running max only moves when a score passes it by more
    // than kLazy (log2 units), so p <= 2^kLazy and P' stays far from fp16
    // overflow; o, l and the v_mn sums share the stale max, so the result is
    // unchanged. The first live page always sets it (m_run = -inf).
    const bool grow0 = mx[0] > m_run[0] + kLazy, grow1 = mx[1] > m_run[1] + kLazy;
    if (__any_sync(0xffffffffu, grow0 || grow1)) {
      float alpha[2];
      alpha[0] = grow0 ? fast_exp2(m_run[0] - mx[0]) : 1.0f;
      alpha[1] = grow1 ? fast_exp2(m_run[1] - mx[1]) : 1.0f;
      if (grow0) m_run[0] = mx[0];
      if (grow1) m_run[1] = mx[1];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l_run[e] *= alpha[e];
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) mn_acc[e][gg] *= alpha[e];
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= alpha[0];
        o[mt][1] *= alpha[1];
        o[mt][2] *= alpha[0];
        o[mt][3] *= alpha[1];
      }
    }

    // ---- probabilities -> P'^T B fragments (per value group), v_mn terms
    uint32_t pb[2][NG][2];
    const float* vsw = kEarly ? &sh.vsv[qb][kTokW * warp * NG] : &st.vs[kTokW * warp * NG];
    const float* vmw = kEarly ? &sh.vmv[qb][kTokW * warp * NG] : &st.vm[kTokW * warp * NG];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float pr[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) pr[c] = fast_exp2(sc[j][c] - m_run[c & 1]);
      l_run[0] += pr[0] + pr[2];
      l_run[1] += pr[1] + pr[3];
      float sl[NG], sh_[NG], ml[NG], mh[NG];
      if (NG == 1) {
        const float2 s2 = *reinterpret_cast<const float2*>(vsw + tok_j[j]);
        const float2 m2 = *reinterpret_cast<const float2*>(vmw + tok_j[j]);
        sl[0] = s2.x;
        sh_[0] = s2.y;
        ml[0] = m2.x;
        mh[0] = m2.y;
      } else {
        const float4 s4 = *reinterpret_cast<const float4*>(vsw + 2 * tok_j[j]);
        const float4 m4 = *reinterpret_cast<const float4*>(vmw + 2 * tok_j[j]);
        sl[0] = s4.x;
        sl[NG - 1] = s4.y;
        sh_[0] = s4.z;
        sh_[NG - 1] = s4.w;
        ml[0] = m4.x;
        ml[NG - 1] = m4.y;
        mh[0] = m4.z;
        mh[NG - 1] = m4.w;
      }
      if (partial) {
        // dead tokens contribute nothing, whatever their (stale) scales hold
        const bool lo_ok = tok_j[j] < valid, hi_ok = tok_j[j] + 1 < valid;
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          sl[gg] = lo_ok ? sl[gg] : 0.0f;
          ml[gg] = lo_ok ? ml[gg] : 0.0f;
          sh_[gg] = hi_ok ? sh_[gg] : 0.0f;
          mh[gg] = hi_ok ? mh[gg] : 0.0f;
        }
      }
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        mn_acc[0][gg] = fmaf(pr[0], ml[gg], fmaf(pr[2], mh[gg], mn_acc[0][gg]));
        mn_acc[1][gg] = fmaf(pr[1], ml[gg], fmaf(pr[3], mh[gg], mn_acc[1][gg]));
        pb[j][gg][0] = movmatrix_t(pack_half2(pr[0] * sl[gg], pr[1] * sl[gg]));
        pb[j][gg][1] = movmatrix_t(pack_half2(pr[2] * sh_[gg], pr[3] * sh_[gg]));
      }
    }

    // ---- O'^T += V^T . P'^T over 32-dim blocks db (dim half db >> 1, chunk
    // db & 1): matrix d = tokens {4r + d} x 32 dims; k-step j takes matrices
    // 2j (k 0..7) and 2j + 1 (k 8..15). m-tile 2 db + s: rows g / g + 8 =
    // dims 32 db + 4g + 2s and + 1.
#pragma unroll
    for (int db = 0; db < 4; ++db) {
      if constexpr (!kEarly) ldsm_x4_t(vx[db], reinterpret_cast<const unsigned char*>(&st.v[0][0]) + vro[db]);
      const int gg = NG == 2 ? (db >> 1) : 0;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t x0 = vx[db][2 * j], x1 = vx[db][2 * j + 1];
        mma16816(o[2 * db], nib_lo_sub(x0), nib_hi_sub(x0), nib_lo_sub(x1), nib_hi_sub(x1), pb[j][gg][0],
                 pb[j][gg][1]);
        const uint32_t y0 = hi_bytes(x0), y1 = hi_bytes(x1);
        mma16816(o[2 * db + 1], nib_lo_sub(y0), y0, nib_lo_sub(y1), y1, pb[j][gg][0],
                 pb[j][gg][1]);
      }
    }
  }

  if (aborted) {
    // let the copies still in flight land before the shared memory is reused
    if (tid == 0)
      for (int i = consumed; i < min(n_pages, consumed + kAhead); ++i)
        (void)mbar_wait(&sh.full[i % kStages], static_cast<uint32_t>((i / kStages) & 1));
  }
  __syncthreads();

  // ---- merge the 4 warps: sum l and mn over the 8 row groups first
#pragma unroll
  for (int e = 0; e < 2; ++e) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], off);
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) mn_acc[e][gg] += __shfl_xor_sync(0xffffffffu, mn_acc[e][gg], off);
    }
  }
  float* mo = reinterpret_cast<float*>(smem_raw);  // [warp][head][dim]
  float* mm = mo + kWarps * kHeads * kD;            // [warp][head]
  float* ml = mm + kWarps * kHeads;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d_lo = 32 * (mt >> 1) + 4 * g + 2 * (mt & 1);
    const int gg = NG == 2 ? (mt >> 2) : 0;
    if (mt & 1) {  // rows g + 8 of the odd m-tiles took whole bytes (n2 + 16 n3)
      o[mt][2] -= o[mt][0];
      o[mt][3] -= o[mt][1];
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int head = 2 * t + e;
      mo[(warp * kHeads + head) * kD + d_lo] = fmaf(o[mt][e], kUnsub, mn_acc[e][gg]);
      mo[(warp * kHeads + head) * kD + d_lo + 1] = fmaf(o[mt][2 + e], kUnsubHi, mn_acc[e][gg]);
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
  // per head: the maximum over the warps, each warp's weight exp2(m_w - M)
  // (-1: the warp saw nothing) and the weighted sum of l, once
  float* mw8 = ml + kWarps * kHeads;  // [warp][head] weights
  float* hmax = mw8 + kWarps * kHeads;
  float* hsum = hmax + kHeads;
  if (tid < kHeads) {
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w * kHeads + tid]);
    float l = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = mm[w * kHeads + tid];
      const bool live = M != -CUDART_INF_F && mw != -CUDART_INF_F;
      const float sc = live ? exp2f(mw - M) : -1.0f;
      mw8[w * kHeads + tid] = sc;
      if (live) l = fmaf(sc, ml[w * kHeads + tid], l);
    }
    hmax[tid] = M;
    hsum[tid] = l;
  }
  __syncthreads();
  for (int idx = tid; idx < kHeads * kD; idx += kThreads) {
    const int head = idx / kD, d = idx % kD;
    if (head >= G) continue;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float sc = mw8[w * kHeads + head];
      if (sc >= 0.0f) acc = fmaf(sc, mo[(w * kHeads + head) * kD + d], acc);
    }
    store_partial(p, b, h * G + head, split, d, acc, hmax[head], hsum[head]);
  }
}

static_assert(sizeof(PageStage<1>) * kStages >=
                  sizeof(float) * (kWarps * kHeads * kD + 3 * kWarps * kHeads + 2 * kHeads),
              "merge buffers must fit in the stage memory");

// ------------------------------------------------------------ host side

int encode_maps(const DecodeParams& p, CUtensorMap* tk, CUtensorMap* tv) {
  auto enc = encode_fn();
  if (enc == nullptr) return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  {
    // k_quant as [NB * KVH * D rows][B/8 words]; one (page, head) block is one
    // box of 64-byte rows with the 64-byte swizzle (see koff)
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kBlk / 8),
                                static_cast<cuuint64_t>(p.num_blocks) * p.kvh * kD};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kBlk / 8) * 4};
    const cuuint32_t box[2] = {kBlk / 8, kD};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(tk, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(p.kq), dims,
                           strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled(k_quant) failed: " + std::to_string(r));
  }
  {
    // v_quant [NB * B tokens][KVH][D/8 words] viewed as
    // [token % 4][token / 4][KVH][D/8 words]: the box {16 words, 1 head, B/4
    // quads, 4} lands as [token % 4][token / 4][16 words], 64-byte rows with
    // the 64-byte swizzle (see voff)
    const cuuint64_t row = static_cast<cuuint64_t>(kD / 8) * 4 * p.kvh;  // bytes per token
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD / 8), static_cast<cuuint64_t>(p.kvh),
                                static_cast<cuuint64_t>(p.num_blocks) * (kBlk / 4), 4};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD / 8) * 4, 4 * row, row};
    const cuuint32_t box[4] = {kD / 8, 1, kBlk / 4, 4};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = enc(tv, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, const_cast<int32_t*>(p.vq), dims,
                           strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return set_error(QKV_ERR_CUDA, "cuTensorMapEncodeTiled(v_quant) failed: " + std::to_string(r));
  }
  return QKV_OK;
}

template <int NG, bool kEarly>
int set_smem_attr() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> done{0};
  const uint64_t bit = 1ull << (dev & 63);
  if ((done.load() & bit) == 0) {
    const cudaError_t e = cudaFuncSetAttribute(kivi_decode_tma_kernel<NG, kEarly>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kivi_smem_bytes<NG>()));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(kivi_decode_tma_kernel)");
    done.fetch_or(bit);
  }
  return QKV_OK;
}

}  // namespace

bool kivi_tma_geometry(const DecodeParams& p) {
  return p.head_size == kD && p.blk == kBlk && (p.group == 64 || p.group == 128) && p.gqa >= 1 &&
         p.gqa <= kHeads;
}

bool kivi_tma_supported(const DecodeParams& p) {
  const auto al = [](const void* x, uintptr_t a) { return (reinterpret_cast<uintptr_t>(x) & (a - 1)) == 0; };
  return kivi_tma_geometry(p) && p.num_blocks > 0 &&
         static_cast<int64_t>(p.num_blocks) * p.kvh * kD < (int64_t{1} << 31) && al(p.kq, 16) && al(p.vq, 16) && al(p.ks, 16) &&
         al(p.km, 16) && al(p.vs, 8) && al(p.vm, 8);
}

// Unit-pages (requests x kv heads x pages per request) up to which the early
// refill schedule runs: measured on config 5's shapes with the current page
// loop (late: unrolled by two), it wins at 8192 (0.0469 vs 0.0490 ms) and on
// config 2 (3968; 35.1 vs 36.9 us), and loses at 16384 (0.0800 vs 0.0780) and
// 32768 (0.149 vs 0.137).
constexpr long long kEarlyMaxUnitPages = 12288;

bool kivi_early(long long units, long long pages) { return units * pages <= kEarlyMaxUnitPages; }

// CTAs of the page-pipelined kernel resident per SM: the launch bounds (5 for
// group 128 on the late schedule, else 4) or shared memory, whichever is lower.
int kivi_tma_ctas_per_sm(int group, bool early) {
  constexpr int kSmemPerSm = 228 * 1024, kReservedPerCta = 1024;
  const int per = static_cast<int>(group == 128 ? kivi_smem_bytes<1>() : kivi_smem_bytes<2>()) +
                  kReservedPerCta;
  const int by_smem = kSmemPerSm / per, by_regs = (group == 128 && !early) ? 5 : 4;
  return by_smem < by_regs ? by_smem : by_regs;
}

// Splits chosen for whole waves: among split counts that keep each split
// within kMaxPages pages, the one whose grid (window CTAs included) best
// fills its last wave, with a small charge per split for the partial-state
// traffic of the combine.
SplitPlan plan_kivi_tma(int batch, int kvh, int group, int max_seq_len, int sms) {
  SplitPlan plan;
  const int pages = max_seq_len > 0 ? (max_seq_len + kBlk - 1) / kBlk : 1;
  const int units = batch * kvh > 0 ? batch * kvh : 1;
  const int resident = sms * kivi_tma_ctas_per_sm(group, kivi_early(units, pages));
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
    // the window CTAs are short but take their slots when the grid starts
    const long long grid = static_cast<long long>(units) * (se + kTailCtas);
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
  plan.total = plan.hist_splits + kTailCtas;
  return plan;
}

constexpr int kSplitMidBatch = 8;

int launch_kivi_tma(const DecodeParams& p0, cudaStream_t stream, bool combine, int* splits_used) {
  DecodeParams p = p0;
  // window CTAs only when there is a window; the partial count shrinks to match
  if (p.res_state == nullptr) p.splits_total = p.num_hist_splits;
  if (splits_used != nullptr) *splits_used = p.splits_total;
  CUtensorMap tk, tv;
  int rc = encode_maps(p, &tk, &tv);
  if (rc != QKV_OK) return rc;
  // the split index moves slowest, so the CTAs an SM receives come from
  // different splits rather than neighbouring splits of few requests (config
  // 5 0.245 -> 0.240 ms, one GPU's N = 8 share 0.0468 -> 0.0450, config 4's
  // decode rows 0.104 -> 0.100). Batches of up to kSplitMidBatch requests
  // order (kv head, split, request) instead: config 2 (8 requests) 0.0367 ->
  // 0.0329-0.0344 ms, where that order costs config 4's rows (30 requests)
  // and the N = 8 share (32) 3-4 %.
  // (the late schedule keeps the first order: its kernel reads no flag).
  // The plan's pages per request: history splits x pages per split.
  const bool early = kivi_early(static_cast<long long>(p.batch) * p.kvh,
                                static_cast<long long>(p.num_hist_splits) * (p.split_tokens / kBlk));
  p.split_mid = early && p.batch <= kSplitMidBatch ? 1 : 0;
  const dim3 grid = p.split_mid ? dim3(p.kvh, p.splits_total, p.batch) : dim3(p.kvh, p.batch, p.splits_total);
#define QKV_KIVI_LAUNCH(NG, EARLY)                                                      \
  do {                                                                                  \
    if ((rc = set_smem_attr<NG, EARLY>()) != QKV_OK) return rc;                         \
    PdlConfig c_(grid, dim3(kThreads), kivi_smem_bytes<NG>(), stream, p.after_ring_write != 0); \
    const cudaError_t le_ = cudaLaunchKernelEx(&c_.cfg, kivi_decode_tma_kernel<NG, EARLY>, p, tk, tv); \
    if (le_ != cudaSuccess) return cuda_error(le_, "kivi_decode_tma_kernel");                          \
  } while (0)
  if (p.group == 128) {
    if (early) QKV_KIVI_LAUNCH(1, true); else QKV_KIVI_LAUNCH(1, false);
  } else {
    if (early) QKV_KIVI_LAUNCH(2, true); else QKV_KIVI_LAUNCH(2, false);
  }
#undef QKV_KIVI_LAUNCH
  QKV_CHECK_LAUNCH("kivi_decode_tma_kernel");
  if (p.splits_total > 1 && combine) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
