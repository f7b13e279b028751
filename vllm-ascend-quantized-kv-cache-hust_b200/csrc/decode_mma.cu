// Tensor-core paged decode kernels (production geometry: head_size 128,
// page size 128, group 64/128, up to 8 query heads per KV head).
//
// One CTA owns (request, kv head, history split); each of its 8 warps walks
// "units" of 64 tokens (half a page) with a private two-stage cp.async ring in
// shared memory, so every warp keeps one unit in flight while it computes the
// previous one. Per unit the warp computes
//     S^T[token][head] = K[token][channel] . Q'^T[channel][head]
//     O^T[dim][head]  += V^T[dim][token]   . P'^T[token][head]
// with mma.sync m16n8k16 (fp16 x fp16 -> fp32). The 8 query heads of the KV
// head are the N dimension, so no MMA lane is padding for GQA 8.
//
// int4 -> fp16 in registers: PRMT gathers byte j of two 32-bit words (two
// channels of K, or two tokens of V) into the low bytes of each half, and one
// LOP3 ((x & 0x000F000F) | 0x6400_6400) yields the fp16 pair 1024 + n; the
// high nibble ((x & 0x00F000F0) | ...) yields 1024 + 16 n, so no shift is ever
// needed; one HSUB2 removes the 1024 exactly, so the MMA sees the codes n (or
// 16 n) and accumulates only the signal. Token rows / dim rows built from high
// nibbles carry a factor 16 that is divided out of the fp32 result. Scales fold
// into the other operand:
//     K: Q'[h][d] = q[h][d] * k_scale[d][group] * softmax_scale * log2(e)
//        S = S' / f + sum_d q[h][d] k_mn[d][group]
//     V: P'[t][h] = p[t][h] * v_scale[t][group]
//        O = O' / f + sum_t p[t][h] * v_mn[t][group]
// The dequantised values are thus used exactly (code * scale + min in real
// arithmetic), without the bf16 rounding a dense gather would add.
// The bf16 residual window (the "tail" split) is handled by the generic
// kernel, which writes the same partial-softmax format.
#include <math_constants.h>

#include <atomic>

#include "decode_common.cuh"

namespace qkv {

int launch_decode_generic_splits(const DecodeParams& p, int mode, int num_splits,
                                 bool combine, cudaStream_t stream);

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kD = 128;     // head size of the tensor-core path
constexpr int kBlk = 128;   // page size of the tensor-core path
constexpr int kUnit = 64;   // tokens per unit (half a page)
constexpr int kHeads = 8;   // N of the MMA: query heads per KV head (padded)
constexpr float kLog2Inv16 = 0.0625f;

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

__device__ __forceinline__ float2 unpack_half2(uint32_t x) {
  return __half22float2(*reinterpret_cast<const __half2*>(&x));
}

__device__ __forceinline__ uint32_t hsub2_1024(uint32_t x) {
  uint32_t y;
  asm("sub.f16x2 %0, %1, %2;\n" : "=r"(y) : "r"(x), "r"(0x64006400u));
  return y;
}

// fp16 pairs of the low / high nibbles of bytes 0 and 2 of x
__device__ __forceinline__ uint32_t nib_lo(uint32_t x) {
  return (x & 0x000F000Fu) | 0x64006400u;
}
__device__ __forceinline__ uint32_t nib_hi(uint32_t x) {
  return (x & 0x00F000F0u) | 0x64006400u;
}
// byte j of a -> byte 0, byte j of b -> byte 2
__device__ __forceinline__ uint32_t pair_bytes(uint32_t a, uint32_t b, int j) {
  return __byte_perm(a, b, static_cast<uint32_t>(j | ((4 + j) << 8)));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
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

// ------------------------------------------------------------ KIVI stage

// One unit (64 tokens of one page, one KV head) in shared memory.
struct KiviStage {
  uint32_t k[kD][8];      // words 8*half .. 8*half+7 of every channel
  float ks[kD * 2];       // k_scale rows of the page (both groups when g = 64)
  float km[kD * 2];       // k_mn
  uint32_t v[kUnit][16];  // value words, swizzled (see v_row / v_word)
  float vs[kUnit * 2];    // v_scale of the unit's tokens (D/g per token)
  float vm[kUnit * 2];    // v_mn
};
constexpr int kKiviStageBytes = sizeof(KiviStage);

// Value rows are swizzled so the 4 token rows one PV load instruction touches
// (local tokens 16t + 2j, t = 0..3) hit distinct banks: token r lives in row
// r ^ ((r >> 4) & 1), and its word w at w ^ (8 * ((r >> 5) & 1)).
__device__ __forceinline__ int v_row(int r) { return r ^ ((r >> 4) & 1); }
__device__ __forceinline__ int v_word(int r, int w) { return w ^ (((r >> 5) & 1) << 3); }

// Issues the cp.async copies of unit (page, half) into `st`; all 32 lanes.
__device__ __forceinline__ void kivi_issue(KiviStage& st, const DecodeParams& p,
                                           int64_t page, int half, int h,
                                           int lane, int ngk, int ngv) {
  const int64_t kv = p.kvh;
  // keys: 128 channels x 32 bytes
  const int32_t* kbase = p.kq + ((page * kv + h) * kD) * (kBlk / 8) + 8 * half;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane + 32 * i;  // 256 chunks of 16 B
    const int ch = c >> 1, part = c & 1;
    cp_async16(&st.k[ch][4 * part], kbase + ch * (kBlk / 8) + 4 * part);
  }
  // key scales / mins: 128 * ngk floats each, contiguous
  const float* ksrc = p.ks + (page * kv + h) * kD * ngk;
  const float* msrc = p.km + (page * kv + h) * kD * ngk;
  for (int c = lane; c < kD * ngk / 4; c += 32) {
    cp_async16(&st.ks[4 * c], ksrc + 4 * c);
    cp_async16(&st.km[4 * c], msrc + 4 * c);
  }
  // values: 64 tokens x 64 bytes (token stride kvh * 64 B)
  const int64_t tok0 = page * kBlk + half * kUnit;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = lane + 32 * i;
    const int r = c >> 2, part = c & 3;
    const int32_t* src = p.vq + ((tok0 + r) * kv + h) * (kD / 8) + 4 * part;
    cp_async16(&st.v[v_row(r)][v_word(r, 4 * part)], src);
  }
  // value scales / mins: ngv floats per token
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = lane + 32 * i;
    const int64_t off = ((tok0 + r) * kv + h) * ngv;
    if (ngv == 1) {
      cp_async4(&st.vs[r], p.vs + off);
      cp_async4(&st.vm[r], p.vm + off);
    } else {
      cp_async8(&st.vs[2 * r], p.vs + off);
      cp_async8(&st.vm[2 * r], p.vm + off);
    }
  }
}

template <int NGV>  // value groups per token: 1 (g = 128) or 2 (g = 64)
__global__ void __launch_bounds__(kThreads, 1)
kivi_decode_mma_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.gqa;
  const int ngk = kBlk / p.group;  // key groups per page (1 or 2)
  constexpr int ngv = NGV;

  KiviStage* stages = reinterpret_cast<KiviStage*>(smem_raw) + warp * 2;

  // ---- history range of this split: [t0, t1), t1 <= first window position
  const int L = max(p.seq_lens[b], 0);
  const TailState ts = load_tail_state(p, b, L);
  const int body_end = min(ts.k_begin, ts.v_begin);
  const int t0 = split * p.split_tokens;
  const int t1 = min(body_end, t0 + p.split_tokens);
  const int n_units = t1 > t0 ? (t1 - t0 + kUnit - 1) / kUnit : 0;

  // ---- q of head g (zero for padding heads), channels of this thread:
  // k-step kk, slot i -> channel 16*kk + 4*i + t
  float qv[8][4];
  {
    const __nv_bfloat16* qrow =
        p.q + static_cast<int64_t>(b) * p.q_stride + (static_cast<int64_t>(h) * G + g) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qv[kk][i] = g < G ? __bfloat162float(qrow[16 * kk + 4 * i + t]) * p.scale_log2 : 0.0f;
  }

  float o[8][4];  // O^T fragments of dim m-tiles (j', h') = (mt & 3, mt >> 2)
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};  // heads 2t, 2t+1
  float l_run[2] = {0.0f, 0.0f};                    // this thread's share
  float mn_acc[2][NGV];                             // sum_t p * v_mn per head, group
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int gg = 0; gg < NGV; ++gg) mn_acc[i][gg] = 0.0f;

  // units of this warp: warp, warp + 8, ...
  int64_t pages[2] = {-1, -1};
  auto unit_page = [&](int u) -> int64_t {
    const int pos = t0 + u * kUnit;
    int64_t pg = -1;
    if (lane == 0) pg = page_of(p, b, pos);
    return __shfl_sync(0xffffffffu, pg, 0);
  };
  auto issue = [&](int u, int slot) {
    const int64_t pg = unit_page(u);
    pages[slot] = pg;
    if (pg >= 0) kivi_issue(stages[slot], p, pg, ((t0 + u * kUnit) / kUnit) & 1, h, lane, ngk, ngv);
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
    const KiviStage& st = stages[slot];
    const int pos0 = t0 + u * kUnit;         // first position of the unit
    const int half = (pos0 / kUnit) & 1;
    const int kgrp = ngk == 2 ? half : 0;

    // ---- Q' = q * k_scale (fp16) and sum_d q * k_mn, head g
    uint32_t bq[8][2];
    float smn = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      float qq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = 16 * kk + 4 * i + t;
        qq[i] = qv[kk][i] * st.ks[ch * ngk + kgrp];
        smn = fmaf(qv[kk][i], st.km[ch * ngk + kgrp], smn);
      }
      bq[kk][0] = pack_half2(qq[0], qq[1]);
      bq[kk][1] = pack_half2(qq[2], qq[3]);
    }
    smn += __shfl_xor_sync(0xffffffffu, smn, 1);
    smn += __shfl_xor_sync(0xffffffffu, smn, 2);
    // per-head constant of this thread's score columns (heads 2t, 2t+1)
    float cmn[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) cmn[e] = __shfl_sync(0xffffffffu, smn, (2 * t + e) << 2);

    // ---- S'^T = K . Q'^T: m-tile j = byte j of word g (rows g: low nibble,
    // rows g + 8: high nibble) -> tokens 8 g + 2 j (+1)
    float s[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t w0 = st.k[16 * kk + t][g];
      const uint32_t w1 = st.k[16 * kk + 4 + t][g];
      const uint32_t w2 = st.k[16 * kk + 8 + t][g];
      const uint32_t w3 = st.k[16 * kk + 12 + t][g];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t x01 = pair_bytes(w0, w1, j);
        const uint32_t x23 = pair_bytes(w2, w3, j);
        mma16816(s[j], hsub2_1024(nib_lo(x01)), hsub2_1024(nib_hi(x01)), hsub2_1024(nib_lo(x23)),
                 hsub2_1024(nib_hi(x23)), bq[kk][0], bq[kk][1]);
      }
    }

    // ---- scores (log2 units), masking, online softmax over heads 2t, 2t+1
    float mx[2] = {-CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tok_lo = 8 * g + 2 * j;  // local token of rows g; +1 for rows g+8
      const bool v_lo = pos0 + tok_lo < t1, v_hi = pos0 + tok_lo + 1 < t1;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float lo = s[j][e] + cmn[e];
        const float hi = fmaf(s[j][2 + e], kLog2Inv16, cmn[e]);
        s[j][e] = v_lo ? lo : -CUDART_INF_F;
        s[j][2 + e] = v_hi ? hi : -CUDART_INF_F;
        mx[e] = fmaxf(mx[e], fmaxf(s[j][e], s[j][2 + e]));
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
#pragma unroll
      for (int gg = 0; gg < NGV; ++gg) mn_acc[e][gg] *= alpha[e];
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }

    // ---- probabilities -> P'^T B fragments (per value group), mn terms
    uint32_t pb[4][NGV][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float pr[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int e = c & 1;
        pr[c] = s[j][c] == -CUDART_INF_F ? 0.0f : exp2f(s[j][c] - m_run[e]);
        l_run[e] += pr[c];
      }
      const int tok_lo = 8 * g + 2 * j;
#pragma unroll
      for (int gg = 0; gg < NGV; ++gg) {
        const float sl = st.vs[tok_lo * NGV + gg], sh = st.vs[(tok_lo + 1) * NGV + gg];
        const float ml = st.vm[tok_lo * NGV + gg], mh = st.vm[(tok_lo + 1) * NGV + gg];
        // masked tokens contribute nothing, whatever their (stale) scales hold
        const float f0 = pr[0] > 0.0f ? pr[0] * sl : 0.0f, f1 = pr[1] > 0.0f ? pr[1] * sl : 0.0f;
        const float f2 = pr[2] > 0.0f ? pr[2] * sh : 0.0f, f3 = pr[3] > 0.0f ? pr[3] * sh : 0.0f;
        if (pr[0] > 0.0f) mn_acc[0][gg] = fmaf(pr[0], ml, mn_acc[0][gg]);
        if (pr[1] > 0.0f) mn_acc[1][gg] = fmaf(pr[1], ml, mn_acc[1][gg]);
        if (pr[2] > 0.0f) mn_acc[0][gg] = fmaf(pr[2], mh, mn_acc[0][gg]);
        if (pr[3] > 0.0f) mn_acc[1][gg] = fmaf(pr[3], mh, mn_acc[1][gg]);
        pb[j][gg][0] = movmatrix_t(pack_half2(f0, f1));  // rows 0..7 (low nibble tokens)
        pb[j][gg][1] = movmatrix_t(pack_half2(f2, f3));  // rows 8..15 (high nibble tokens)
      }
    }

    // ---- O'^T += V^T . P'^T: k-step j = m-tile j of the scores. k positions
    // (2t, 2t+1) are tokens 16t + 2j and 16t + 8 + 2j, (2t+8, 2t+9) their +1.
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ra = 16 * t + 2 * j, rb = ra + 8;
      uint32_t wa[2][2], wb[2][2];  // [token +0/+1][dim half h']
#pragma unroll
      for (int d1 = 0; d1 < 2; ++d1) {
        const int r0 = ra + d1, r1 = rb + d1;
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          wa[d1][hp] = st.v[v_row(r0)][v_word(r0, 8 * hp + g)];
          wb[d1][hp] = st.v[v_row(r1)][v_word(r1, 8 * hp + g)];
        }
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int jp = mt & 3, hp = mt >> 2;
        const uint32_t x0 = pair_bytes(wa[0][hp], wb[0][hp], jp);
        const uint32_t x1 = pair_bytes(wa[1][hp], wb[1][hp], jp);
        const int gg = NGV == 2 ? hp : 0;
        mma16816(o[mt], hsub2_1024(nib_lo(x0)), hsub2_1024(nib_hi(x0)), hsub2_1024(nib_lo(x1)),
                 hsub2_1024(nib_hi(x1)), pb[j][gg][0], pb[j][gg][1]);
      }
    }
    __syncwarp();
  }
  cp_async_wait0();
  __syncthreads();

  // ---- per-warp finalisation: sum l and mn over the 8 row groups
#pragma unroll
  for (int e = 0; e < 2; ++e) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run[e] += __shfl_xor_sync(0xffffffffu, l_run[e], off);
#pragma unroll
      for (int gg = 0; gg < NGV; ++gg) mn_acc[e][gg] += __shfl_xor_sync(0xffffffffu, mn_acc[e][gg], off);
    }
  }
  // merge buffers (reuse the stages): O [warp][head][dim], m/l [warp][head]
  float* mo = reinterpret_cast<float*>(smem_raw);
  float* mm = mo + kWarps * kHeads * kD;
  float* ml = mm + kWarps * kHeads;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int jp = mt & 3, hp = mt >> 2;
    const int d_lo = 8 * (8 * hp + g) + 2 * jp;  // rows g; rows g + 8 -> d_lo + 1
    const int gg = NGV == 2 ? hp : 0;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int head = 2 * t + e;
      mo[(warp * kHeads + head) * kD + d_lo] = o[mt][e] + mn_acc[e][gg];
      mo[(warp * kHeads + head) * kD + d_lo + 1] = fmaf(o[mt][2 + e], kLog2Inv16, mn_acc[e][gg]);
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

constexpr size_t kKiviSmem = static_cast<size_t>(kKiviStageBytes) * 2 * kWarps;
static_assert(kKiviSmem >= sizeof(float) * (kWarps * kHeads * kD + 2 * kWarps * kHeads),
              "merge buffers must fit in the stage memory");

}  // namespace

bool decode_mma_supported(const DecodeParams& p, bool kivi) {
  if (!kivi)
    return p.head_size == kD && p.blk == kBlk && p.gqa >= 1 && p.gqa <= kHeads &&
           (reinterpret_cast<uintptr_t>(p.kc) & 15u) == 0 &&
           (reinterpret_cast<uintptr_t>(p.vc) & 15u) == 0;
  return p.head_size == kD && p.blk == kBlk && (p.group == 64 || p.group == 128) &&
         p.gqa >= 1 && p.gqa <= kHeads &&
         (reinterpret_cast<uintptr_t>(p.kq) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.ks) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.km) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.vq) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.vs) & 7u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.vm) & 7u) == 0;
}

int launch_decode_mma(const DecodeParams& p, bool kivi, cudaStream_t stream) {
  if (!kivi) {
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
  // the residual-window tail split runs on the generic kernel first
  if (p.splits_total > p.num_hist_splits) {
    DecodeParams tail = p;
    tail.split_base = p.num_hist_splits;
    const int rc = launch_decode_generic_splits(tail, kKiviPages,
                                                p.splits_total - p.num_hist_splits, false, stream);
    if (rc != QKV_OK) return rc;
  }
  dim3 grid(p.num_hist_splits, p.kvh, p.batch);
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr_set{0};  // bit (2 * device + variant)
  const int variant = p.group == 128 ? 0 : 1;
  const uint64_t bit = 1ull << ((2 * dev + variant) & 63);
  if ((attr_set.load() & bit) == 0) {
    const cudaError_t e = variant == 0
        ? cudaFuncSetAttribute(kivi_decode_mma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kKiviSmem))
        : cudaFuncSetAttribute(kivi_decode_mma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kKiviSmem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(kivi_decode_mma_kernel)");
    attr_set.fetch_or(bit);
  }
  if (variant == 0)
    kivi_decode_mma_kernel<1><<<grid, kThreads, kKiviSmem, stream>>>(p);
  else
    kivi_decode_mma_kernel<2><<<grid, kThreads, kKiviSmem, stream>>>(p);
  QKV_CHECK_LAUNCH("kivi_decode_mma_kernel");
  if (p.splits_total > 1) {
    launch_combine(p, stream);
    QKV_CHECK_LAUNCH("combine_kernel");
  }
  return QKV_OK;
}

}  // namespace qkv
