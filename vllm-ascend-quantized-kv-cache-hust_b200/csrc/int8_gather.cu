// INT8 gather: dense bf16 K/V of whole requests from the int8 pages — the
// reference's _dequant_int8_paged_kv_to_dense
// (methods/int8_dynamic/attention_backend.py:370-404): gather by block table,
// keep the live tokens, (code - 0) * (1 / inv) in bf16.
//
// Element (position t of request r, head h, channel d):
//   bf16(code[page(t)][t % blk][h][d] * aq[h][d])
// The product of an int8 code and a bf16 scale is exact in fp32, so one
// rounding to bf16 gives the reference's bf16 multiply bit for bit.
// One thread writes 16 consecutive channels (32 bytes) of one (token, head):
// the 16-byte code load and both stores are coalesced along the token row.
#include "decode_common.cuh"

namespace qkv {

namespace {

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 16 int8 codes times 16 bf16 scales -> 16 bf16 (two uint4)
__device__ __forceinline__ void dequant16(uint4 codes, const __nv_bfloat16* aq, uint4& lo, uint4& hi) {
  const uint4 s0 = *reinterpret_cast<const uint4*>(aq);
  const uint4 s1 = *reinterpret_cast<const uint4*>(aq + 8);
  const uint32_t cw[4] = {codes.x, codes.y, codes.z, codes.w};
  const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t word = cw[i >> 1];
    const int sh = (i & 1) * 16;
    const float c0 = static_cast<float>(static_cast<int8_t>((word >> sh) & 0xFFu));
    const float c1 = static_cast<float>(static_cast<int8_t>((word >> (sh + 8)) & 0xFFu));
    const float a0 = __uint_as_float(sw[i] << 16);
    const float a1 = __uint_as_float(sw[i] & 0xFFFF0000u);
    o[i] = pack_bf16x2(c0 * a0, c1 * a1);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

__global__ void int8_gather_kernel(const DecodeParams p, const int32_t* cu_k, int total_k,
                                   __nv_bfloat16* dense_k, __nv_bfloat16* dense_v) {
  const int chunks = p.head_size / 16;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t per_token = static_cast<int64_t>(p.kvh) * chunks;
  if (idx >= static_cast<int64_t>(total_k) * per_token) return;
  const int tok = static_cast<int>(idx / per_token);
  const int hc = static_cast<int>(idx % per_token);  // head * chunks + chunk
  // request of this dense row: the last r with cu_k[r] <= tok
  int lo = 0, hi = p.num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_k[mid] <= tok) lo = mid; else hi = mid - 1;
  }
  const int t = tok - cu_k[lo];
  const int64_t page = page_of(p, lo, t);
  uint4 k0 = make_uint4(0, 0, 0, 0), k1 = k0, v0 = k0, v1 = k0;
  if (page >= 0) {
    const int64_t src = ((page * p.blk + t % p.blk) * p.kvh) * p.head_size + 16 * static_cast<int64_t>(hc);
    const uint4 kc = __ldg(reinterpret_cast<const uint4*>(p.kc + src));
    const uint4 vc = __ldg(reinterpret_cast<const uint4*>(p.vc + src));
    const int64_t sidx = 16 * static_cast<int64_t>(hc);  // [KVH, D] scale row of this chunk
    dequant16(kc, p.k_aq + sidx, k0, k1);
    dequant16(vc, p.v_aq + sidx, v0, v1);
  }
  const int64_t o = static_cast<int64_t>(tok) * p.kvh * p.head_size + 16 * static_cast<int64_t>(hc);
  reinterpret_cast<uint4*>(dense_k + o)[0] = k0;
  reinterpret_cast<uint4*>(dense_k + o)[1] = k1;
  reinterpret_cast<uint4*>(dense_v + o)[0] = v0;
  reinterpret_cast<uint4*>(dense_v + o)[1] = v1;
}

}  // namespace

int launch_int8_gather(const DecodeParams& p, const int32_t* cu_k, int total_k, __nv_bfloat16* dense_k,
                       __nv_bfloat16* dense_v, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(total_k) * p.kvh * (p.head_size / 16);
  if (threads <= 0) return QKV_OK;
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  if (grid > 0x7FFFFFFFll) return set_error(QKV_ERR_INVALID, "qkv_int8_dequant_gather: too many elements");
  int8_gather_kernel<<<static_cast<unsigned>(grid), block, 0, stream>>>(p, cu_k, total_k, dense_k, dense_v);
  QKV_CHECK_LAUNCH("int8_gather_kernel");
  return QKV_OK;
}

}  // namespace qkv
