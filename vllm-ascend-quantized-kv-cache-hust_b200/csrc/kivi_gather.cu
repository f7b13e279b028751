// KIVI gather: dense bf16 K/V of whole requests from the int4 pages and the
// bf16 residual windows — the reference's kivi_dequant_gather_cache
// (ops/kivi_gather.py:36-156) followed by its residual overwrite
// (methods/kivi_int4/attention_backend.py:849-935), in one pass.
//
// Element (position t of request r, head h, channel d):
//   key:   t >= k_begin(r) ? window_k[row][(k_start + t - k_begin) % cap][h][d]
//                          : bf16(code * k_scale + k_mn)     (fp32, rounded once)
//   value: the same with the value window and v_scale / v_mn.
// One thread writes 8 consecutive channels (16 bytes) of one (token, head).
#include "decode_common.cuh"

namespace qkv {

namespace {

__device__ __forceinline__ float kivi_value(uint32_t code, float scale, float mn) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), scale), mn);
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

}  // namespace

int launch_kivi_gather(const DecodeParams& p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                       __nv_bfloat16* dense_v, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(total_k) * p.kvh * (p.head_size / 8);
  if (threads <= 0) return QKV_OK;
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  if (grid > 0x7FFFFFFFll) return set_error(QKV_ERR_INVALID, "qkv_kivi_dequant_gather: too many elements");
  kivi_gather_kernel<<<static_cast<unsigned>(grid), block, 0, stream>>>(p, cu_k, total_k, dense_k, dense_v);
  QKV_CHECK_LAUNCH("kivi_gather_kernel");
  return QKV_OK;
}

}  // namespace qkv
