// KIVI gather: dense bf16 K/V of whole requests from the int4 pages and the
// bf16 residual windows — the reference's kivi_dequant_gather_cache
// (ops/kivi_gather.py:36-156) followed by its residual overwrite
// (methods/kivi_int4/attention_backend.py:849-935), in one pass.
//
// Element (position t of request r, head h, channel d):
//   key:   t >= k_begin(r) ? window_k[row][(k_start + t - k_begin) % cap][h][d]
//                          : bf16(code * k_scale + k_mn)     (fp32, rounded once)
//   value: the same with the value window and v_scale / v_mn.
// One thread writes 8 consecutive channels (16 bytes) of one (token, head);
// geometries the tiled kernel below does not take use this generic form.
#include "decode_common.cuh"

namespace qkv {

namespace {

__device__ __forceinline__ float kivi_value(uint32_t code, float scale, float mn) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), scale), mn);
}

// The same value without an int -> float conversion: `field` holds the code
// at bits 19..22, so f = 16 + code exactly (1.0 * 2^4 plus code ulps of
// 2^-19), and fma(f, scale, -16 scale) = RN(code * scale): the product f *
// scale is exact inside the FMA and -16 scale is exact, so the sum is code *
// scale exactly before its one rounding. Valid while 16 |scale| is finite
// (|scale| < 2^124); callers take kivi_value beyond kBigScale.
constexpr float kBigScale = 0x1p120f;
__device__ __forceinline__ float kivi_value_field(uint32_t field, float scale, float neg16_scale, float mn) {
  const float f = __uint_as_float((field & 0x00780000u) | 0x41800000u);
  return __fadd_rn(__fmaf_rn(f, scale, neg16_scale), mn);
}
// rotates the nibble at bits 4 k .. 4 k + 3 of w to bits 19..22
__device__ __forceinline__ uint32_t nibble_field(uint32_t w, int k) {
  return __funnelshift_l(w, w, (19 - 4 * k) & 31);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// grid.x over (token, head, word) triples of all requests
__global__ void kivi_gather_kernel(const DecodeParams p, const int32_t* cu_k, int total_k,
                                   __nv_bfloat16* dense_k, __nv_bfloat16* dense_v) {
  const int words = p.head_size / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t per_token = static_cast<int64_t>(p.kvh) * words;
  if (idx >= static_cast<int64_t>(total_k) * per_token) return;
  const int tok = static_cast<int>(idx / per_token);
  const int h = static_cast<int>((idx / words) % p.kvh);
  const int w = static_cast<int>(idx % words);
  // request of this dense row: the last r with cu_k[r] <= tok
  int lo = 0, hi = p.num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_k[mid] <= tok) lo = mid; else hi = mid - 1;
  }
  const int r = lo;
  const int t = tok - cu_k[r];
  const int L = max(p.seq_lens[r], 0);
  const TailState ts = load_tail_state(p, r, L);
  const int64_t kvh = p.kvh;
  const int D = p.head_size;
  uint32_t outk[4], outv[4];
  // ---- key
  if (t >= ts.k_begin) {
    const int slot = (ts.k_start + (t - ts.k_begin)) % p.res_cap;
    const uint4 raw = *reinterpret_cast<const uint4*>(
        p.rk + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * D + 8 * w);
    outk[0] = raw.x; outk[1] = raw.y; outk[2] = raw.z; outk[3] = raw.w;
  } else {
    const int64_t page = page_of(p, r, t);
    float v[8];
    if (page < 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    } else {
      const int off = t % p.blk;
      const int ngk = p.blk / p.group;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t chan = (page * kvh + h) * D + 8 * w + i;
        const uint32_t word = static_cast<uint32_t>(p.kq[chan * (p.blk >> 3) + (off >> 3)]);
        const int64_t si = chan * ngk + off / p.group;
        v[i] = kivi_value((word >> (4 * (off & 7))) & 0xFu, p.ks[si], p.km[si]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) outk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  }
  // ---- value
  if (t >= ts.v_begin) {
    const int slot = (ts.v_start + (t - ts.v_begin)) % p.res_cap;
    const uint4 raw = *reinterpret_cast<const uint4*>(
        p.rv + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * D + 8 * w);
    outv[0] = raw.x; outv[1] = raw.y; outv[2] = raw.z; outv[3] = raw.w;
  } else {
    const int64_t page = page_of(p, r, t);
    float v[8];
    if (page < 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    } else {
      const int64_t vrow = (page * p.blk + t % p.blk) * kvh + h;
      const uint32_t word = static_cast<uint32_t>(p.vq[vrow * (D >> 3) + w]);
      const int64_t si = vrow * (D / p.group) + (8 * w) / p.group;  // 8 dims share a group
      const float sc = p.vs[si], mn = p.vm[si];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = kivi_value((word >> (4 * i)) & 0xFu, sc, mn);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) outv[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  }
  const int64_t o = (static_cast<int64_t>(tok) * kvh + h) * D + 8 * w;
  *reinterpret_cast<uint4*>(dense_k + o) = make_uint4(outk[0], outk[1], outk[2], outk[3]);
  *reinterpret_cast<uint4*>(dense_v + o) = make_uint4(outv[0], outv[1], outv[2], outv[3]);
}

// Tiled form: one CTA per (chunk of `ch` positions of one request, KV head).
// The key codes are channel-major in the pages ([D][blk / 8] words per page
// and head), the dense rows token-major, so the chunk's code words and group
// scales are staged in shared memory transposed (word-major, channel-minor;
// rows padded by 4 words so both the staging stores and the 16-byte reads
// are conflict-free) and every thread then writes 16 contiguous bytes of one
// token row. Values are token-major already and are read directly. `ch`
// divides the block size and is a multiple or a divisor of the group, so a
// chunk lies in one page and its groups do not straddle chunks.
// kD / kG / kCh: the head size, group and chunk as constants (0: from the
// arguments), so the per-element index arithmetic is shifts.
template <int kD, int kG, int kCh>
__global__ void __launch_bounds__(256) kivi_gather_tiled_kernel(const DecodeParams p, const int32_t* cu_k, int ch_arg,
                                                                __nv_bfloat16* dense_k, __nv_bfloat16* dense_v) {
  const int ch = kCh ? kCh : ch_arg;
  const int group = kG ? kG : p.group;
  extern __shared__ __align__(16) uint32_t gsm[];
  // ---- chunk -> (request, first position): chunks never straddle requests
  int b = -1, t0 = 0;
  {
    int acc = 0;
    for (int r = 0; r < p.num_reqs; ++r) {
      const int nc = (max(p.seq_lens[r], 0) + ch - 1) / ch;
      if (static_cast<int>(blockIdx.x) < acc + nc) {
        b = r;
        t0 = (blockIdx.x - acc) * ch;
        break;
      }
      acc += nc;
    }
  }
  if (b < 0) return;  // uniform: past the last chunk
  const int h = blockIdx.y;
  const int L = max(p.seq_lens[b], 0);
  const int n = min(ch, L - t0);
  const int D = kD ? kD : p.head_size, kvh = p.kvh, words = D >> 3;
  const int cw = ch >> 3, pitch = D + 4;
  const int ng = ch >= group ? ch / group : 1;
  uint32_t* codes = gsm;                                          // [cw][pitch]
  float* gscale = reinterpret_cast<float*>(gsm + cw * pitch);     // [ng][D]
  float* gmin = gscale + ng * D;
  float* gneg = gmin + ng * D;                                    // -16 x scale
  const TailState ts = load_tail_state(p, b, L);
  const int64_t page = t0 < ts.k_begin || t0 < ts.v_begin ? page_of(p, b, t0) : -1;
  const int off0 = t0 % p.blk;
  const int g0 = off0 / group;
  if (page >= 0 && t0 < ts.k_begin) {
    const int wpb = p.blk >> 3;
    const int32_t* src = p.kq + (page * kvh + h) * static_cast<int64_t>(D) * wpb + (off0 >> 3);
    for (int i = threadIdx.x; i < D * cw; i += blockDim.x) {
      const int d = i / cw, w = i - d * cw;
      codes[w * pitch + d] = static_cast<uint32_t>(__ldg(src + static_cast<int64_t>(d) * wpb + w));
    }
    const int ngk = p.blk / group;
    const int64_t sb = (page * kvh + h) * static_cast<int64_t>(D) * ngk + g0;
    for (int i = threadIdx.x; i < D * ng; i += blockDim.x) {
      const int d = i / ng, gi = i - d * ng;
      const float sc = __ldg(p.ks + sb + static_cast<int64_t>(d) * ngk + gi);
      gscale[gi * D + d] = sc;
      gneg[gi * D + d] = fabsf(sc) < kBigScale ? __fmul_rn(-16.0f, sc) : __int_as_float(0x7fffffff);
      gmin[gi * D + d] = __ldg(p.km + sb + static_cast<int64_t>(d) * ngk + gi);
    }
  }
  __syncthreads();
  const int64_t row0 = static_cast<int64_t>(cu_k[b]) + t0;
  if constexpr (kD > 0 && kCh > 0 && kG >= kCh) {
    // Constant geometry with one key group per chunk: a thread keeps the same
    // 8 channels (word c) for all its tokens, so their key scales, minima and
    // -16 x scales, and the choice of the fast form, are loop constants, and
    // the row addresses advance by a fixed stride.
    constexpr int kWords = kD / 8;
    static_assert(256 % kWords == 0, "a block covers whole token rows");
    const int c = threadIdx.x % kWords, tl0 = threadIdx.x / kWords;
    constexpr int kStep = 256 / kWords;  // tokens per pass of the block
    float sv[8], mv[8], nv[8];
    bool fast = true;
    const bool staged = page >= 0 && t0 < ts.k_begin;  // the key scales were staged above
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sv[j] = staged ? gscale[8 * c + j] : 0.0f;
      mv[j] = staged ? gmin[8 * c + j] : 0.0f;
      nv[j] = staged ? gneg[8 * c + j] : 0.0f;
      fast = fast && !isnan(nv[j]);  // a NaN -16 x scale marks a scale beyond kBigScale
    }
    const int64_t ostride = static_cast<int64_t>(kStep) * kvh * kD;
    int64_t o = ((row0 + tl0) * kvh + h) * kD + 8 * c;
    // value row of token tl: (page * blk + off0 + tl) * kvh + h
    int64_t vrow = page >= 0 ? (page * p.blk + off0 + tl0) * kvh + h : 0;
    const int vcg = (8 * c) / kG;  // value group of this thread's 8 dims
    for (int tl = tl0; tl < n; tl += kStep, o += ostride, vrow += static_cast<int64_t>(kStep) * kvh) {
      const int t = t0 + tl;
      uint32_t ok[4], ov[4];
      // ---- key
      if (t >= ts.k_begin) {
        const int slot = (ts.k_start + (t - ts.k_begin)) % p.res_cap;
        const uint4 raw = *reinterpret_cast<const uint4*>(
            p.rk + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * kD + 8 * c);
        ok[0] = raw.x; ok[1] = raw.y; ok[2] = raw.z; ok[3] = raw.w;
      } else if (page < 0) {
        ok[0] = ok[1] = ok[2] = ok[3] = 0u;
      } else {
        const uint32_t* cr = codes + (tl >> 3) * pitch + 8 * c;
        const uint4 w0 = *reinterpret_cast<const uint4*>(cr);
        const uint4 w1 = *reinterpret_cast<const uint4*>(cr + 4);
        const int k = tl & 7;
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        if (fast) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ok[j] = pack_bf16x2(kivi_value_field(nibble_field(wv[2 * j], k), sv[2 * j], nv[2 * j], mv[2 * j]),
                                kivi_value_field(nibble_field(wv[2 * j + 1], k), sv[2 * j + 1], nv[2 * j + 1],
                                                 mv[2 * j + 1]));
        } else {
          const int sh = 4 * k;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ok[j] = pack_bf16x2(kivi_value((wv[2 * j] >> sh) & 0xFu, sv[2 * j], mv[2 * j]),
                                kivi_value((wv[2 * j + 1] >> sh) & 0xFu, sv[2 * j + 1], mv[2 * j + 1]));
        }
      }
      // ---- value (token-major in the pages)
      if (t >= ts.v_begin) {
        const int slot = (ts.v_start + (t - ts.v_begin)) % p.res_cap;
        const uint4 raw = *reinterpret_cast<const uint4*>(
            p.rv + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * kD + 8 * c);
        ov[0] = raw.x; ov[1] = raw.y; ov[2] = raw.z; ov[3] = raw.w;
      } else if (page < 0) {
        ov[0] = ov[1] = ov[2] = ov[3] = 0u;
      } else {
        const uint32_t word = static_cast<uint32_t>(__ldg(p.vq + vrow * kWords + c));
        const int64_t si = vrow * (kD / kG) + vcg;
        const float sc = __ldg(p.vs + si), mn = __ldg(p.vm + si);
        if (fabsf(sc) < kBigScale) {
          const float n16 = __fmul_rn(-16.0f, sc);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ov[j] = pack_bf16x2(kivi_value_field(nibble_field(word, 2 * j), sc, n16, mn),
                                kivi_value_field(nibble_field(word, 2 * j + 1), sc, n16, mn));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ov[j] = pack_bf16x2(kivi_value((word >> (8 * j)) & 0xFu, sc, mn),
                                kivi_value((word >> (8 * j + 4)) & 0xFu, sc, mn));
        }
      }
      *reinterpret_cast<uint4*>(dense_k + o) = make_uint4(ok[0], ok[1], ok[2], ok[3]);
      *reinterpret_cast<uint4*>(dense_v + o) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
    }
    return;
  }
  for (int i = threadIdx.x; i < n * words; i += blockDim.x) {
    const int tl = i / words, c = i - tl * words;
    const int t = t0 + tl;
    uint32_t ok[4], ov[4];
    // ---- key
    if (t >= ts.k_begin) {
      const int slot = (ts.k_start + (t - ts.k_begin)) % p.res_cap;
      const uint4 raw = *reinterpret_cast<const uint4*>(
          p.rk + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * D + 8 * c);
      ok[0] = raw.x; ok[1] = raw.y; ok[2] = raw.z; ok[3] = raw.w;
    } else if (page < 0) {
      ok[0] = ok[1] = ok[2] = ok[3] = 0u;
    } else {
      const uint32_t* cr = codes + (tl >> 3) * pitch + 8 * c;
      const uint4 w0 = *reinterpret_cast<const uint4*>(cr);
      const uint4 w1 = *reinterpret_cast<const uint4*>(cr + 4);
      const int gi = (off0 + tl) / group - g0;
      const float4 s0 = *reinterpret_cast<const float4*>(gscale + gi * D + 8 * c);
      const float4 s1 = *reinterpret_cast<const float4*>(gscale + gi * D + 8 * c + 4);
      const float4 m0 = *reinterpret_cast<const float4*>(gmin + gi * D + 8 * c);
      const float4 m1 = *reinterpret_cast<const float4*>(gmin + gi * D + 8 * c + 4);
      const float4 n0 = *reinterpret_cast<const float4*>(gneg + gi * D + 8 * c);
      const float4 n1 = *reinterpret_cast<const float4*>(gneg + gi * D + 8 * c + 4);
      const int k = tl & 7;
      const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      const float nv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
      // a NaN -16 x scale marks a scale beyond kBigScale (or not finite)
      const bool fast = !(isnan(nv[0]) || isnan(nv[1]) || isnan(nv[2]) || isnan(nv[3]) || isnan(nv[4]) ||
                          isnan(nv[5]) || isnan(nv[6]) || isnan(nv[7]));
      if (fast) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ok[j] = pack_bf16x2(kivi_value_field(nibble_field(wv[2 * j], k), sv[2 * j], nv[2 * j], mv[2 * j]),
                              kivi_value_field(nibble_field(wv[2 * j + 1], k), sv[2 * j + 1], nv[2 * j + 1],
                                               mv[2 * j + 1]));
      } else {
        const int sh = 4 * k;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ok[j] = pack_bf16x2(kivi_value((wv[2 * j] >> sh) & 0xFu, sv[2 * j], mv[2 * j]),
                              kivi_value((wv[2 * j + 1] >> sh) & 0xFu, sv[2 * j + 1], mv[2 * j + 1]));
      }
    }
    // ---- value (token-major in the pages)
    if (t >= ts.v_begin) {
      const int slot = (ts.v_start + (t - ts.v_begin)) % p.res_cap;
      const uint4 raw = *reinterpret_cast<const uint4*>(
          p.rv + ((static_cast<int64_t>(ts.row) * p.res_cap + slot) * kvh + h) * D + 8 * c);
      ov[0] = raw.x; ov[1] = raw.y; ov[2] = raw.z; ov[3] = raw.w;
    } else if (page < 0) {
      ov[0] = ov[1] = ov[2] = ov[3] = 0u;
    } else {
      const int64_t vrow = (page * p.blk + off0 + tl) * kvh + h;
      const uint32_t word = static_cast<uint32_t>(__ldg(p.vq + vrow * words + c));
      const int64_t si = vrow * (D / group) + (8 * c) / group;
      const float sc = __ldg(p.vs + si), mn = __ldg(p.vm + si);
      if (fabsf(sc) < kBigScale) {
        const float n16 = __fmul_rn(-16.0f, sc);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ov[j] = pack_bf16x2(kivi_value_field(nibble_field(word, 2 * j), sc, n16, mn),
                              kivi_value_field(nibble_field(word, 2 * j + 1), sc, n16, mn));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ov[j] = pack_bf16x2(kivi_value((word >> (8 * j)) & 0xFu, sc, mn),
                              kivi_value((word >> (8 * j + 4)) & 0xFu, sc, mn));
      }
    }
    const int64_t o = ((row0 + tl) * kvh + h) * D + 8 * c;
    *reinterpret_cast<uint4*>(dense_k + o) = make_uint4(ok[0], ok[1], ok[2], ok[3]);
    *reinterpret_cast<uint4*>(dense_v + o) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
  }
}

// Chunk length of the tiled kernel for this geometry, or 0 (generic kernel).
int tiled_chunk(int blk, int group) {
  const int ch = blk % 64 == 0 ? 64 : blk;
  if (ch > 128 || ch % 8 != 0) return 0;
  if (ch % group != 0 && group % ch != 0) return 0;
  return ch;
}

}  // namespace

int launch_kivi_gather(const DecodeParams& p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                       __nv_bfloat16* dense_v, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(total_k) * p.kvh * (p.head_size / 8);
  if (threads <= 0) return QKV_OK;
  const int ch = tiled_chunk(p.blk, p.group);
  const int ng = ch >= p.group ? ch / p.group : 1;
  const size_t smem = ch > 0 ? (static_cast<size_t>(ch / 8) * (p.head_size + 4) + 3 * ng * p.head_size) * 4 : 0;
  if (ch > 0 && smem <= 48 * 1024) {
    const int64_t chunks = (static_cast<int64_t>(total_k) + ch - 1) / ch + p.num_reqs;  // upper bound
    if (chunks > 0x7FFFFFFFll) return set_error(QKV_ERR_INVALID, "qkv_kivi_dequant_gather: too many chunks");
    const dim3 grid(static_cast<unsigned>(chunks), p.kvh);
    if (p.head_size == 128 && ch == 64 && p.group == 64)
      kivi_gather_tiled_kernel<128, 64, 64><<<grid, 256, smem, stream>>>(p, cu_k, ch, dense_k, dense_v);
    else if (p.head_size == 128 && ch == 64 && p.group == 128)
      kivi_gather_tiled_kernel<128, 128, 64><<<grid, 256, smem, stream>>>(p, cu_k, ch, dense_k, dense_v);
    else
      kivi_gather_tiled_kernel<0, 0, 0><<<grid, 256, smem, stream>>>(p, cu_k, ch, dense_k, dense_v);
    QKV_CHECK_LAUNCH("kivi_gather_tiled_kernel");
    return QKV_OK;
  }
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  if (grid > 0x7FFFFFFFll) return set_error(QKV_ERR_INVALID, "qkv_kivi_dequant_gather: too many elements");
  kivi_gather_kernel<<<static_cast<unsigned>(grid), block, 0, stream>>>(p, cu_k, total_k, dense_k, dense_v);
  QKV_CHECK_LAUNCH("kivi_gather_kernel");
  return QKV_OK;
}

}  // namespace qkv
