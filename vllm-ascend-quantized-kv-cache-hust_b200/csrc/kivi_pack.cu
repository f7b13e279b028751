// KIVI INT4 pack kernels: full-precision K/V -> the paged int4 views.
//
// Bit-exact restatement of the reference pack arithmetic
// (ops/triton/kivi_pack.py:61-131 value kernel, :134-226 key kernel; the CPU
// contract is KiviInt4Semantics.group_scale / quantize_group / pack_int4,
// methods/kivi_int4/semantics.py:76-111):
//   scale = max((mx - mn) / 15, 1e-6)                 fp32, IEEE division
//   code  = clamp(floor((x - mn) / scale + 0.5), 0, 15)
//   word  = OR_L (code_L & 0xF) << 4L                 lane L at bits 4L
// Every operation is written with explicit round-to-nearest intrinsics so the
// compiler cannot contract or reassociate it.
#include <type_traits>

#include "qkv_common.cuh"

namespace qkv {
namespace {

__device__ __forceinline__ float group_scale(float mn, float mx) {
  return fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 15.0f), 1.0e-6f);
}

__device__ __forceinline__ uint32_t quantize_code(float x, float mn,
                                                  float scale) {
  float q = floorf(__fadd_rn(__fdiv_rn(__fsub_rn(x, mn), scale), 0.5f));
  q = fminf(fmaxf(q, 0.0f), 15.0f);
  return static_cast<uint32_t>(static_cast<int>(q)) & 0xFu;
}

// Loads 8 consecutive elements starting at p (8-element aligned) as fp32.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p,
                                                     float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// ------------------------------------------------------------------ values

// One thread per (token, head, 8-dim word). The D/8 threads of a
// (token, head) row are a power-of-two aligned run inside one warp, and a
// quant group is an aligned run of g/8 of them, so the group min/max is an
// xor-shuffle reduction. Every lane takes part in the shuffles; only lanes
// with a valid slot store.
// Where a packed token's row comes from: token t of `value` (dense), or, with
// `src`, ring lane src[t] >= 0 of `ring` / new token -1 - src[t] of `fresh`
// (a window plan's flush sources, read in place).
template <typename T>
struct RowSource {
  const int64_t* src;
  const T* ring;
  const T* fresh;
  int64_t ring_lanes, n_new;
};

template <typename T>
__global__ void __launch_bounds__(256)
pack_value_kernel(const T* __restrict__ value, const void* __restrict__ slots,
                  int slot_dtype, int64_t num_tokens, int kvh, int head_size,
                  int group_size, int64_t num_slots, int32_t* __restrict__ v_quant,
                  float* __restrict__ v_scale, float* __restrict__ v_mn, int* err,
                  RowSource<T> rs) {
  const int words = head_size >> 3;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = num_tokens * kvh * words;
  const bool in_range = tid < total;
  const int64_t t_idx = in_range ? tid : 0;
  const int w = static_cast<int>(t_idx % words);
  const int64_t row = t_idx / words;  // token * kvh + head
  const int64_t token = row / kvh;
  const int head = static_cast<int>(row % kvh);

  int64_t slot = -1;
  if (in_range) slot = load_index(slots, slot_dtype, token);
  bool valid = in_range && slot >= 0;
  if (valid && slot >= num_slots) {
    record_error(err, kErrSlot);
    valid = false;
  }

  float v[8];
  const T* rowp = value + row * head_size;
  if (rs.src != nullptr && in_range) {
    const int64_t sidx = rs.src[token];
    const int64_t tok_row = static_cast<int64_t>(kvh) * head_size;
    if (sidx >= 0 && sidx < rs.ring_lanes) {
      rowp = rs.ring + sidx * tok_row + static_cast<int64_t>(head) * head_size;
    } else if (sidx < 0 && -1 - sidx < rs.n_new) {
      rowp = rs.fresh + (-1 - sidx) * tok_row + static_cast<int64_t>(head) * head_size;
    } else {
      if (w == 0) record_error(err, kErrWindowSource);
      valid = false;
      rowp = nullptr;
    }
  }
  if (in_range && rowp != nullptr) {
    load8<T>(rowp + w * 8, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  const int gw = group_size >> 3;  // words per group (power of two)
  for (int off = 1; off < gw; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  if (!valid) return;
  const float scale = group_scale(mn, mx);
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) word |= quantize_code(v[i], mn, scale) << (4 * i);
  const int64_t dst_row = slot * kvh + head;  // [NB*B, KVH] flattened
  v_quant[dst_row * words + w] = static_cast<int32_t>(word);
  if ((w & (gw - 1)) == 0) {
    const int groups = head_size / group_size;
    const int64_t s = dst_row * groups + w / gw;
    v_scale[s] = scale;
    v_mn[s] = mn;
  }
}

// Generic value packer for head sizes whose word count is not a power of two
// up to 32: one thread per (token, head, group).
template <typename T>
__global__ void pack_value_generic_kernel(
    const T* __restrict__ value, const void* __restrict__ slots, int slot_dtype,
    int64_t num_tokens, int kvh, int head_size, int group_size, int64_t num_slots,
    int32_t* __restrict__ v_quant, float* __restrict__ v_scale,
    float* __restrict__ v_mn, int* err) {
  const int groups = head_size / group_size;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid >= num_tokens * kvh * groups) return;
  const int grp = static_cast<int>(tid % groups);
  const int64_t row = tid / groups;
  const int64_t token = row / kvh;
  const int head = static_cast<int>(row % kvh);
  const int64_t slot = load_index(slots, slot_dtype, token);
  if (slot < 0) return;
  if (slot >= num_slots) {
    record_error(err, kErrSlot);
    return;
  }
  const T* src = value + row * head_size + grp * group_size;
  float mn = to_f32(src[0]), mx = mn;
  for (int i = 1; i < group_size; ++i) {
    const float x = to_f32(src[i]);
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
  }
  const float scale = group_scale(mn, mx);
  const int64_t dst_row = slot * kvh + head;
  for (int wbase = 0; wbase < group_size; wbase += 8) {
    uint32_t word = 0;
    for (int i = 0; i < 8; ++i)
      word |= quantize_code(to_f32(src[wbase + i]), mn, scale) << (4 * i);
    v_quant[dst_row * (head_size >> 3) + (grp * group_size + wbase) / 8] =
        static_cast<int32_t>(word);
  }
  v_scale[dst_row * groups + grp] = scale;
  v_mn[dst_row * groups + grp] = mn;
}

// -------------------------------------------------------------------- keys

// One thread per (token group, head, channel). The group's g tokens of this
// channel are reduced to mn/mx, then re-read (L1/L2 hit) and packed 8 tokens
// per int32 word; the g/8 words of a channel are contiguous in k_quant
// ([NB, KVH, D, B/8]) and are stored as 16-byte vectors when aligned.
template <typename T, int GW>
__global__ void __launch_bounds__(128)
pack_key_kernel(const T* __restrict__ key, const void* __restrict__ slots,
                int slot_dtype, int64_t num_groups, int kvh, int head_size,
                int block_size, int64_t num_blocks, int32_t* __restrict__ k_quant,
                float* __restrict__ k_scale, float* __restrict__ k_mn, int* err,
                bool vector_store) {
  constexpr int kGroup = GW * 8;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid >= num_groups * kvh * head_size) return;
  const int d = static_cast<int>(tid % head_size);
  const int64_t gh = tid / head_size;
  const int head = static_cast<int>(gh % kvh);
  const int64_t gi = gh / kvh;

  const int64_t first_slot = load_index(slots, slot_dtype, gi * kGroup);
  if (first_slot < 0) return;  // the reference kernel skips such groups
  const int64_t blk = first_slot / block_size;
  const int off = static_cast<int>(first_slot - blk * block_size);
  if (blk >= num_blocks || (off % kGroup) != 0 || off + kGroup > block_size) {
    record_error(err, kErrSlot);
    return;
  }

  const int64_t row_stride = static_cast<int64_t>(kvh) * head_size;
  const T* src = key + gi * kGroup * row_stride + head * head_size + d;
  float mn = to_f32(src[0]), mx = mn;
#pragma unroll 8
  for (int t = 1; t < kGroup; ++t) {
    const float x = to_f32(src[t * row_stride]);
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
  }
  const float scale = group_scale(mn, mx);

  uint32_t words[GW];
#pragma unroll
  for (int j = 0; j < GW; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int l = 0; l < 8; ++l)
      word |= quantize_code(to_f32(src[(j * 8 + l) * row_stride]), mn, scale)
              << (4 * l);
    words[j] = word;
  }
  const int64_t chan = (blk * kvh + head) * static_cast<int64_t>(head_size) + d;
  int32_t* dst = k_quant + chan * (block_size >> 3) + (off >> 3);
  if (GW % 4 == 0 && vector_store) {
#pragma unroll
    for (int j = 0; j + 3 < GW; j += 4)
      reinterpret_cast<uint4*>(dst)[j / 4] =
          make_uint4(words[j], words[j + 1], words[j + 2], words[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < GW; ++j) dst[j] = static_cast<int32_t>(words[j]);
  }
  const int64_t s = chan * (block_size / kGroup) + off / kGroup;
  k_scale[s] = scale;
  k_mn[s] = mn;
}

// Tiled key packer for group_size in {32, 64, 128}: one CTA per
// (token group, head) stages the group's [g x D] slice in shared memory with
// 16-byte coalesced loads, then thread d quantises channel d from there.
template <typename T, int GW>
__global__ void __launch_bounds__(128)
pack_key_tiled_kernel(const T* __restrict__ key, const void* __restrict__ slots,
                      int slot_dtype, int kvh, int head_size, int block_size,
                      int64_t num_blocks, int32_t* __restrict__ k_quant,
                      float* __restrict__ k_scale, float* __restrict__ k_mn,
                      int* err) {
  constexpr int kGroup = GW * 8;
  extern __shared__ __align__(16) unsigned char tile_raw[];
  T* tile = reinterpret_cast<T*>(tile_raw);  // [kGroup][head_size]
  const int head = blockIdx.y;
  const int64_t gi = blockIdx.x;
  const int64_t first_slot = load_index(slots, slot_dtype, gi * kGroup);
  if (first_slot < 0) return;
  const int64_t blk = first_slot / block_size;
  const int off = static_cast<int>(first_slot - blk * block_size);
  if (blk >= num_blocks || (off % kGroup) != 0 || off + kGroup > block_size) {
    if (threadIdx.x == 0) record_error(err, kErrSlot);
    return;
  }
  const int64_t row_stride = static_cast<int64_t>(kvh) * head_size;
  const T* src = key + gi * kGroup * row_stride + static_cast<int64_t>(head) * head_size;
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte load
  const int vec_per_row = head_size / kVec;
  for (int i = threadIdx.x; i < kGroup * vec_per_row; i += blockDim.x) {
    const int r = i / vec_per_row, c = i % vec_per_row;
    reinterpret_cast<uint4*>(tile + r * head_size)[c] =
        reinterpret_cast<const uint4*>(src + r * row_stride)[c];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < head_size; d += blockDim.x) {
    float mn = to_f32(tile[d]), mx = mn;
#pragma unroll 8
    for (int r = 1; r < kGroup; ++r) {
      const float x = to_f32(tile[r * head_size + d]);
      mn = fminf(mn, x);
      mx = fmaxf(mx, x);
    }
    const float scale = group_scale(mn, mx);
    uint32_t words[GW];
#pragma unroll
    for (int j = 0; j < GW; ++j) {
      uint32_t word = 0;
#pragma unroll
      for (int l = 0; l < 8; ++l)
        word |= quantize_code(to_f32(tile[(j * 8 + l) * head_size + d]), mn, scale) << (4 * l);
      words[j] = word;
    }
    const int64_t chan = (blk * kvh + head) * static_cast<int64_t>(head_size) + d;
    int32_t* dst = k_quant + chan * (block_size >> 3) + (off >> 3);
#pragma unroll
    for (int j = 0; j < GW; j += 4)
      reinterpret_cast<uint4*>(dst)[j / 4] = make_uint4(words[j], words[j + 1], words[j + 2], words[j + 3]);
    const int64_t s = chan * (block_size / kGroup) + off / kGroup;
    k_scale[s] = scale;
    k_mn[s] = mn;
  }
}

// ------------------------------------------------ fast path (bf16, head 128)
//
// The same codes, scales and minima as the kernels above, without an IEEE
// division per element and without branches. For a group with minimum mn and
// scale s (computed exactly as above) and inv = RN(1/s), each element takes
//   d  = RN(x - mn)                   the reference's first operation
//   q0 = RN(d * inv)                  quotient estimate
//   r  = RN(d - q0 * s)               (one FMA) the remainder, exact
//   q  = RN(q0 + r * inv)             (one FMA) = RN(d / s), the reference's
//                                     IEEE quotient (Markstein's correction
//                                     step, 1990)
//   t  = RN(q + 0.5)                  the reference's second rounding
//   k  = floor(t): RM(t + 1.5 2^23)   rounding toward -inf leaves 1.5 2^23 +
//                                     floor(t), so k sits in the low mantissa
//                                     bits
// k needs no clamp: 0 <= d <= mx - mn, so q <= 15 (1 + 2^-23) and t <= 15.5.
// The correction step was checked against exact rational arithmetic on
// 600 000 quotients: random ones, every element of bf16 groups (which hit
// exact half-integer quotients often), quotients next to float32 rounding
// midpoints, and the hardest case fp32 operands allow (a quotient 1/B of an
// ulp from a midpoint, B the divisor's 24-bit significand); no mismatch. The
// fp32 pairs run as packed f32x2 instructions (two lanes per instruction).
// Non-finite inputs give codes outside the contract (the reference's cast of
// a NaN to an integer is undefined as well).
namespace fastq {

using u64 = unsigned long long;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ u64 pack2(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(u64 r, uint32_t& a, uint32_t& b) {
  asm("mov.b64 {%0, %1}, %2;\n" : "=r"(a), "=r"(b) : "l"(r));
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 add2_rm(u64 a, u64 b) {
  u64 r;
  asm("add.rm.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint32_t bmin2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// The group constants of one lane pair: minima, reciprocal and negated scale.
struct Group2 {
  float mn0, mn1;
  u64 inv, neg_s;
};
__device__ __forceinline__ Group2 group2(float mn0, float s0, float mn1, float s1) {
  return Group2{mn0, mn1, pack2(__frcp_rn(s0), __frcp_rn(s1)), pack2(-s0, -s1)};
}

// RN(x - mn) for the bf16 halves of w in one mixed-precision subtraction
// each (the bf16 operand enters exactly; one rounding, as x.float() - mn).
__device__ __forceinline__ u64 sub_bf16x2(uint32_t w, float mn0, float mn1) {
  float d0, d1;
  asm("{\n .reg .b16 lo, hi;\n mov.b32 {lo, hi}, %2;\n"
      " sub.rn.f32.bf16 %0, lo, %3;\n sub.rn.f32.bf16 %1, hi, %4;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "r"(w), "f"(mn0), "f"(mn1));
  return pack2(d0, d1);
}

// Codes of the two bf16 values of w (low half: lane 0 of the group pair),
// returned in the low byte of r0 / r1.
__device__ __forceinline__ void quant2(uint32_t w, const Group2& g, uint32_t& r0, uint32_t& r1) {
  const u64 d = sub_bf16x2(w, g.mn0, g.mn1);
  const u64 q0 = mul2(d, g.inv);
  const u64 q = fma2(fma2(q0, g.neg_s, d), g.inv, q0);
  const u64 k = add2_rm(add2(q, pack2(0.5f, 0.5f)), pack2(kMagic, kMagic));
  unpack2(k, r0, r1);
}

// 8 codes (low bytes of c[0..7], each < 16) -> one int4 word, lane L at bits 4L.
__device__ __forceinline__ uint32_t pack8(const uint32_t (&c)[8]) {
  const uint32_t e = __byte_perm(__byte_perm(c[0], c[2], 0x0040), __byte_perm(c[4], c[6], 0x0040), 0x5410);
  const uint32_t o = __byte_perm(__byte_perm(c[1], c[3], 0x0040), __byte_perm(c[5], c[7], 0x0040), 0x5410);
  return e | (o << 4);
}

}  // namespace fastq

// Keys: one CTA of 256 threads per (token group, head). Thread t owns the
// channel pair cp = t % 64 and the token quarter t / 64 of the group: it
// loads the pair for its G / 4 tokens (a warp's loads are 128 contiguous
// bytes of a token row), reduces min / max in bf16 pairs (exact), the four
// quarters meet in shared memory, and each thread quantises and stores its
// own G / 32 words per channel. (Eighths of the group over channel halves,
// twice the CTAs with half the tokens each, measured 19 % slower: the
// per-thread setup weighs more.)
template <int G>
__device__ __forceinline__ void pack_key_fast_tile(const __nv_bfloat16* __restrict__ key,
                                                   const void* __restrict__ slots, int slot_dtype, int kvh,
                                                   int block_size, int64_t num_blocks, int32_t* __restrict__ k_quant,
                                                   float* __restrict__ k_scale, float* __restrict__ k_mn, int* err,
                                                   int64_t gi, int head) {
  using namespace fastq;
  constexpr int kD = 128, kChunks = 4, kTok = G / kChunks, kWords = kTok / 8;
  __shared__ uint32_t s_mn[kChunks][64], s_mx[kChunks][64];
  const int64_t first_slot = load_index(slots, slot_dtype, gi * G);
  if (first_slot < 0) return;  // the reference kernel skips such groups
  // (32-bit division whenever the slot fits: one per thread, on every lane)
  const int64_t blk = first_slot < 0x7FFFFFFF
                          ? static_cast<int64_t>(static_cast<uint32_t>(first_slot) / static_cast<uint32_t>(block_size))
                          : first_slot / block_size;
  const int off = static_cast<int>(first_slot - blk * block_size);
  if (blk >= num_blocks || (off % G) != 0 || off + G > block_size) {
    if (threadIdx.x == 0) record_error(err, kErrSlot);
    return;
  }
  const int tc = threadIdx.x >> 6, lane = threadIdx.x & 63;
  const int cp = lane;
  const int64_t row_words = static_cast<int64_t>(kvh) * (kD / 2);
  const uint32_t* src =
      reinterpret_cast<const uint32_t*>(key) + (gi * G + tc * kTok) * row_words + head * (kD / 2) + cp;
  uint32_t v[kTok];
#pragma unroll
  for (int i = 0; i < kTok; ++i) v[i] = __ldg(src + i * row_words);
  uint32_t mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < kTok; ++i) {
    mn = bmin2(mn, v[i]);
    mx = bmax2(mx, v[i]);
  }
  s_mn[tc][lane] = mn;
  s_mx[tc][lane] = mx;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    mn = bmin2(mn, s_mn[j][lane]);
    mx = bmax2(mx, s_mx[j][lane]);
  }
  const float mn0 = bf_lo(mn), mn1 = bf_hi(mn);
  const float sc0 = group_scale(mn0, bf_lo(mx)), sc1 = group_scale(mn1, bf_hi(mx));
  const Group2 g2 = group2(mn0, sc0, mn1, sc1);
  uint32_t w0[kWords], w1[kWords];
#pragma unroll
  for (int j = 0; j < kWords; ++j) {
    uint32_t c0[8], c1[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) quant2(v[8 * j + l], g2, c0[l], c1[l]);
    w0[j] = pack8(c0);
    w1[j] = pack8(c1);
  }
  const int64_t chan0 = (blk * kvh + head) * static_cast<int64_t>(kD) + 2 * cp;
  const int64_t wpc = block_size >> 3;  // words per channel and page
  int32_t* dst0 = k_quant + chan0 * wpc + (off >> 3) + tc * kWords;
  int32_t* dst1 = dst0 + wpc;
  if constexpr (kWords == 4) {
    *reinterpret_cast<uint4*>(dst0) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    *reinterpret_cast<uint4*>(dst1) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  } else {
    static_assert(kWords == 2, "group 64 or 128");
    *reinterpret_cast<uint2*>(dst0) = make_uint2(w0[0], w0[1]);
    *reinterpret_cast<uint2*>(dst1) = make_uint2(w1[0], w1[1]);
  }
  if (tc == 0) {
    const int gpb = block_size / G;
    const int64_t s0 = chan0 * gpb + off / G;
    k_scale[s0] = sc0;
    k_mn[s0] = mn0;
    k_scale[s0 + gpb] = sc1;
    k_mn[s0 + gpb] = mn1;
  }
}

template <int G>
__global__ void __launch_bounds__(256)
pack_key_fast_kernel(const __nv_bfloat16* __restrict__ key, const void* __restrict__ slots, int slot_dtype,
                     int kvh, int block_size, int64_t num_blocks, int32_t* __restrict__ k_quant,
                     float* __restrict__ k_scale, float* __restrict__ k_mn, int* err) {
  pack_key_fast_tile<G>(key, slots, slot_dtype, kvh, block_size, num_blocks, k_quant, k_scale, k_mn, err,
                        blockIdx.x, blockIdx.y);
}

// Values: two threads per (token, head) row of 128 dims, 64 contiguous dims
// (eight 16-byte loads) each, so a warp covers 16 rows; at group 128 the two
// halves combine min / max with one shuffle. Each thread stores its eight
// words (two 16-byte vectors). Index arithmetic is 32-bit: the launcher
// guarantees num_tokens * kvh * 2 < 2^31.
template <int G>
__device__ __forceinline__ void pack_value_fast_rows(const __nv_bfloat16* __restrict__ value,
                                                     const void* __restrict__ slots, int slot_dtype,
                                                     int num_rows, int kvh, int64_t num_slots,
                                                     int32_t* __restrict__ v_quant, float* __restrict__ v_scale,
                                                     float* __restrict__ v_mn, int* err,
                                                     const RowSource<__nv_bfloat16>& rs, unsigned block) {
  using namespace fastq;
  constexpr int kD = 128, kHalf = kD / 2;
  const unsigned tid = block * blockDim.x + threadIdx.x;
  const unsigned row = tid >> 1;  // token * kvh + head
  const int part = static_cast<int>(tid & 1);
  const bool in_range = row < static_cast<unsigned>(num_rows);
  const unsigned token = in_range ? row / static_cast<unsigned>(kvh) : 0u;
  const int head = static_cast<int>(row - token * static_cast<unsigned>(kvh));
  int64_t slot = -1;
  if (in_range) slot = load_index(slots, slot_dtype, token);
  bool valid = in_range && slot >= 0;
  if (valid && slot >= num_slots) {
    record_error(err, kErrSlot);
    valid = false;
  }
  const __nv_bfloat16* rowp = in_range ? value + static_cast<int64_t>(row) * kD : nullptr;
  if (rs.src != nullptr && in_range) {
    const int64_t sidx = rs.src[token];
    const int64_t tok_row = static_cast<int64_t>(kvh) * kD;
    if (sidx >= 0 && sidx < rs.ring_lanes) {
      rowp = rs.ring + sidx * tok_row + static_cast<int64_t>(head) * kD;
    } else if (sidx < 0 && -1 - sidx < rs.n_new) {
      rowp = rs.fresh + (-1 - sidx) * tok_row + static_cast<int64_t>(head) * kD;
    } else {
      if (part == 0) record_error(err, kErrWindowSource);
      valid = false;
      rowp = nullptr;
    }
  }
  uint32_t v[kHalf / 2];
  if (rowp != nullptr) {
#pragma unroll
    for (int i = 0; i < kHalf / 8; ++i) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(rowp + kHalf * part) + i);
      v[4 * i] = a.x;
      v[4 * i + 1] = a.y;
      v[4 * i + 2] = a.z;
      v[4 * i + 3] = a.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kHalf / 2; ++i) v[i] = 0u;
  }
  uint32_t mnp = v[0], mxp = v[0];
#pragma unroll
  for (int i = 1; i < kHalf / 2; ++i) {
    mnp = bmin2(mnp, v[i]);
    mxp = bmax2(mxp, v[i]);
  }
  float mn = fminf(bf_lo(mnp), bf_hi(mnp)), mx = fmaxf(bf_lo(mxp), bf_hi(mxp));
  if constexpr (G == kD) {  // the row is one group: combine the halves
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  }
  if (!valid) return;
  const float sc = group_scale(mn, mx);
  const Group2 g2 = group2(mn, sc, mn, sc);
  uint32_t w[kHalf / 8];
#pragma unroll
  for (int j = 0; j < kHalf / 8; ++j) {
    uint32_t c[8];
#pragma unroll
    for (int l = 0; l < 4; ++l) quant2(v[4 * j + l], g2, c[2 * l], c[2 * l + 1]);
    w[j] = pack8(c);
  }
  const int64_t dst_row = slot * kvh + head;
  uint4* dst = reinterpret_cast<uint4*>(v_quant + dst_row * (kD / 8) + part * (kHalf / 8));
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  if (G == kD ? part == 0 : true) {
    const int64_t sidx = dst_row * (kD / G) + (G == kD ? 0 : part);
    v_scale[sidx] = sc;
    v_mn[sidx] = mn;
  }
}

template <int G>
__global__ void __launch_bounds__(256)
pack_value_fast_kernel(const __nv_bfloat16* __restrict__ value, const void* __restrict__ slots, int slot_dtype,
                       int num_rows, int kvh, int64_t num_slots, int32_t* __restrict__ v_quant,
                       float* __restrict__ v_scale, float* __restrict__ v_mn, int* err,
                       RowSource<__nv_bfloat16> rs) {
  pack_value_fast_rows<G>(value, slots, slot_dtype, num_rows, kvh, num_slots, v_quant, v_scale, v_mn, err, rs,
                          blockIdx.x);
}

// Keys and values of the same tokens in one launch: CTAs [0, groups * kvh)
// take the key tiles (group = x / kvh, head = x % kvh), the rest the value
// rows.
template <int G>
__global__ void __launch_bounds__(256)
pack_kv_fast_kernel(const __nv_bfloat16* __restrict__ key, const __nv_bfloat16* __restrict__ value,
                    const void* __restrict__ slots, int slot_dtype, int64_t num_tokens, int kvh, int block_size,
                    int64_t num_blocks, int32_t* __restrict__ k_quant, float* __restrict__ k_scale,
                    float* __restrict__ k_mn, int32_t* __restrict__ v_quant, float* __restrict__ v_scale,
                    float* __restrict__ v_mn, int* err) {
  const unsigned key_ctas = static_cast<unsigned>(num_tokens / G * kvh);
  const unsigned x = blockIdx.x;
  if (x < key_ctas)
    pack_key_fast_tile<G>(key, slots, slot_dtype, kvh, block_size, num_blocks, k_quant, k_scale, k_mn, err,
                          x / static_cast<unsigned>(kvh), static_cast<int>(x % static_cast<unsigned>(kvh)));
  else
    pack_value_fast_rows<G>(value, slots, slot_dtype, static_cast<int>(num_tokens * kvh), kvh,
                            num_blocks * block_size, v_quant, v_scale, v_mn, err,
                            RowSource<__nv_bfloat16>{nullptr, nullptr, nullptr, 0, 0}, x - key_ctas);
}

template <typename T>
int launch_pack_key(const void* key, const void* slots, int slot_dtype,
                    int64_t num_tokens, int kvh, int head_size, int group_size,
                    int block_size, int64_t num_blocks, int32_t* kq, float* ks,
                    float* km, cudaStream_t stream) {
  const int64_t groups = num_tokens / group_size;
  const int64_t threads = groups * kvh * head_size;
  const int block = 128;
  const int64_t grid = (threads + block - 1) / block;
  const T* k = static_cast<const T*>(key);
  int* err = device_error_ptr();
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    // bf16 at head 128, group 64 / 128: the division-free kernel
    const uintptr_t qa = reinterpret_cast<uintptr_t>(kq);
    if (head_size == 128 && (group_size == 64 || group_size == 128) &&
        (reinterpret_cast<uintptr_t>(key) & 3u) == 0 && (qa & (group_size == 128 ? 15u : 7u)) == 0) {
      dim3 fgrid(static_cast<unsigned>(groups), kvh);
      if (group_size == 128)
        pack_key_fast_kernel<128><<<fgrid, 256, 0, stream>>>(k, slots, slot_dtype, kvh, block_size, num_blocks,
                                                             kq, ks, km, err);
      else
        pack_key_fast_kernel<64><<<fgrid, 256, 0, stream>>>(k, slots, slot_dtype, kvh, block_size, num_blocks,
                                                            kq, ks, km, err);
      QKV_CHECK_LAUNCH("pack_key_fast_kernel");
      return QKV_OK;
    }
  }
  // 16-byte stores need a 16-byte aligned k_quant base and rows of whole
  // 16-byte units; group offsets are multiples of g/8 words (a multiple of 4
  // whenever the vector path is taken)
  const bool vec = (reinterpret_cast<uintptr_t>(kq) & 15u) == 0 &&
                   ((block_size / 8) % 4) == 0;
  // the tiled kernel: 16-byte aligned rows and a tile that fits in 48 KB
  const size_t tile_bytes = static_cast<size_t>(group_size) * head_size * sizeof(T);
  const bool tiled = vec && (reinterpret_cast<uintptr_t>(key) & 15u) == 0 &&
                     (head_size * sizeof(T)) % 16 == 0 && tile_bytes <= 48 * 1024 &&
                     (group_size == 32 || group_size == 64 || group_size == 128);
  if (tiled) {
    dim3 tgrid(static_cast<unsigned>(groups), kvh);
    const int threads = head_size < 128 ? 64 : 128;
    if (group_size == 128)
      pack_key_tiled_kernel<T, 16><<<tgrid, threads, tile_bytes, stream>>>(
          k, slots, slot_dtype, kvh, head_size, block_size, num_blocks, kq, ks, km, err);
    else if (group_size == 64)
      pack_key_tiled_kernel<T, 8><<<tgrid, threads, tile_bytes, stream>>>(
          k, slots, slot_dtype, kvh, head_size, block_size, num_blocks, kq, ks, km, err);
    else
      pack_key_tiled_kernel<T, 4><<<tgrid, threads, tile_bytes, stream>>>(
          k, slots, slot_dtype, kvh, head_size, block_size, num_blocks, kq, ks, km, err);
    QKV_CHECK_LAUNCH("pack_key_tiled_kernel");
    return QKV_OK;
  }
#define QKV_PACK_KEY_CASE(GW)                                                  \
  case GW:                                                                     \
    pack_key_kernel<T, GW><<<grid, block, 0, stream>>>(                        \
        k, slots, slot_dtype, groups, kvh, head_size, block_size, num_blocks, \
        kq, ks, km, err, vec);                                                 \
    break;
  switch (group_size / 8) {
    QKV_PACK_KEY_CASE(1)
    QKV_PACK_KEY_CASE(2)
    QKV_PACK_KEY_CASE(3)
    QKV_PACK_KEY_CASE(4)
    QKV_PACK_KEY_CASE(6)
    QKV_PACK_KEY_CASE(8)
    QKV_PACK_KEY_CASE(12)
    QKV_PACK_KEY_CASE(16)
    QKV_PACK_KEY_CASE(24)
    QKV_PACK_KEY_CASE(32)
    default:
      return set_error(QKV_ERR_UNSUPPORTED,
                       "qkv_kivi_pack_key: group_size " +
                           std::to_string(group_size) +
                           " is not one of 8,16,24,32,48,64,96,128,192,256");
  }
#undef QKV_PACK_KEY_CASE
  QKV_CHECK_LAUNCH("pack_key_kernel");
  return QKV_OK;
}

// The division-free value kernel for bf16 rows at head 128, group 64 / 128
// (rows and v_quant 16-byte aligned); false when it does not apply.
bool launch_pack_value_fast(const __nv_bfloat16* v, const void* slots, int slot_dtype, int64_t num_tokens, int kvh,
                            int head_size, int group_size, int64_t num_slots, int32_t* vq, float* vs, float* vm,
                            RowSource<__nv_bfloat16> rs, cudaStream_t stream) {
  const auto al = [](const void* p, unsigned m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
  if (head_size != 128 || (group_size != 64 && group_size != 128) || !al(vq, 15u)) return false;
  if (rs.src == nullptr ? !al(v, 15u) : (!al(rs.ring, 15u) || !al(rs.fresh, 15u))) return false;
  const int64_t threads = num_tokens * kvh * 2;
  if (threads >= (int64_t{1} << 31)) return false;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  const int rows = static_cast<int>(num_tokens * kvh);
  if (group_size == 128)
    pack_value_fast_kernel<128><<<grid, 256, 0, stream>>>(v, slots, slot_dtype, rows, kvh, num_slots, vq, vs, vm,
                                                          device_error_ptr(), rs);
  else
    pack_value_fast_kernel<64><<<grid, 256, 0, stream>>>(v, slots, slot_dtype, rows, kvh, num_slots, vq, vs, vm,
                                                         device_error_ptr(), rs);
  return true;
}

template <typename T>
int launch_pack_value(const void* value, const void* slots, int slot_dtype,
                      int64_t num_tokens, int kvh, int head_size, int group_size,
                      int block_size, int64_t num_blocks, int32_t* vq, float* vs,
                      float* vm, cudaStream_t stream) {
  const int words = head_size / 8;
  const int64_t num_slots = num_blocks * block_size;
  const T* v = static_cast<const T*>(value);
  int* err = device_error_ptr();
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (launch_pack_value_fast(v, slots, slot_dtype, num_tokens, kvh, head_size, group_size, num_slots, vq, vs,
                               vm, RowSource<__nv_bfloat16>{nullptr, nullptr, nullptr, 0, 0}, stream)) {
      QKV_CHECK_LAUNCH("pack_value_fast_kernel");
      return QKV_OK;
    }
  }
  const bool pow2 = (words & (words - 1)) == 0 && words <= 32;
  // the vector path loads 8 elements (16 or 32 bytes) per thread
  const bool aligned = (reinterpret_cast<uintptr_t>(value) & 15u) == 0;
  if (pow2 && aligned) {
    const int64_t threads = num_tokens * kvh * words;
    const int block = 256;
    const int64_t grid = (threads + block - 1) / block;
    pack_value_kernel<T><<<grid, block, 0, stream>>>(
        v, slots, slot_dtype, num_tokens, kvh, head_size, group_size, num_slots,
        vq, vs, vm, err, RowSource<T>{nullptr, nullptr, nullptr, 0, 0});
    QKV_CHECK_LAUNCH("pack_value_kernel");
  } else {
    const int64_t threads = num_tokens * kvh * (head_size / group_size);
    const int block = 128;
    const int64_t grid = (threads + block - 1) / block;
    pack_value_generic_kernel<T><<<grid, block, 0, stream>>>(
        v, slots, slot_dtype, num_tokens, kvh, head_size, group_size, num_slots,
        vq, vs, vm, err);
    QKV_CHECK_LAUNCH("pack_value_generic_kernel");
  }
  return QKV_OK;
}

int check_common(const char* fn, int dtype, int slot_dtype, int64_t num_tokens,
                 int kvh, int head_size, int group_size, int block_size,
                 int64_t num_blocks) {
  const std::string f(fn);
  QKV_CHECK_ARG(dtype == QKV_F32 || dtype == QKV_BF16 || dtype == QKV_F16,
                f + ": unsupported input dtype");
  QKV_CHECK_ARG(slot_dtype == QKV_I32 || slot_dtype == QKV_I64,
                f + ": slot_mapping must be int32/int64");
  QKV_CHECK_ARG(num_tokens >= 0 && kvh > 0 && num_blocks > 0,
                f + ": bad sizes");
  QKV_CHECK_ARG(group_size > 0 && group_size % 8 == 0,
                f + ": group_size must be a positive multiple of 8");
  QKV_CHECK_ARG(head_size > 0 && head_size % 8 == 0 && head_size <= 1024,
                f + ": head_size must be a multiple of 8 (<= 1024)");
  QKV_CHECK_ARG(block_size > 0 && block_size % 8 == 0,
                f + ": block_size must be a multiple of 8");
  return QKV_OK;
}

}  // namespace

// Value pack of a window plan's flushed rows read where they are (ring
// lanes or new tokens, `src` as in qkv_kivi_window_gather), bf16 rings; the
// vector kernel's geometry only (head_size / 8 a power of two up to 32).
int pack_value_from_sources(const __nv_bfloat16* ring, int64_t ring_lanes, const __nv_bfloat16* fresh,
                            int64_t n_new, const int64_t* src, const int64_t* slots, int64_t num_tokens, int kvh,
                            int head_size, int group_size, int block_size, int64_t num_blocks, int32_t* vq,
                            float* vs, float* vm, cudaStream_t stream) {
  if (num_tokens == 0) return QKV_OK;
  const int words = head_size / 8;
  QKV_CHECK_ARG((words & (words - 1)) == 0 && words <= 32 && head_size % group_size == 0 && src && slots,
                "pack_value_from_sources: unsupported geometry");
  if (launch_pack_value_fast(nullptr, slots, QKV_I64, num_tokens, kvh, head_size, group_size,
                             num_blocks * block_size, vq, vs, vm,
                             RowSource<__nv_bfloat16>{src, ring, fresh, ring_lanes, n_new}, stream)) {
    QKV_CHECK_LAUNCH("pack_value_fast_kernel");
    return QKV_OK;
  }
  const int64_t threads = num_tokens * kvh * words;
  const int block = 256;
  pack_value_kernel<__nv_bfloat16><<<(threads + block - 1) / block, block, 0, stream>>>(
      nullptr, slots, QKV_I64, num_tokens, kvh, head_size, group_size, num_blocks * block_size, vq, vs, vm,
      device_error_ptr(), RowSource<__nv_bfloat16>{src, ring, fresh, ring_lanes, n_new});
  QKV_CHECK_LAUNCH("pack_value_kernel");
  return QKV_OK;
}

}  // namespace qkv

extern "C" {

int qkv_kivi_pack_key(const void* key, int key_dtype, const void* slot_mapping,
                      int slot_dtype, int64_t num_tokens, int num_kv_heads,
                      int head_size, int group_size, int block_size,
                      int64_t num_blocks, int32_t* k_quant, float* k_scale,
                      float* k_mn, qkv_stream_t stream) {
  using namespace qkv;
  int rc = check_common("qkv_kivi_pack_key", key_dtype, slot_dtype, num_tokens,
                        num_kv_heads, head_size, group_size, block_size,
                        num_blocks);
  if (rc != QKV_OK) return rc;
  QKV_CHECK_ARG(num_tokens % group_size == 0,
                "qkv_kivi_pack_key: num_tokens must be a whole number of groups");
  QKV_CHECK_ARG(block_size % group_size == 0,
                "qkv_kivi_pack_key: block_size must be divisible by group_size");
  if (num_tokens == 0) return QKV_OK;
  QKV_CHECK_ARG(key && slot_mapping && k_quant && k_scale && k_mn,
                "qkv_kivi_pack_key: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (key_dtype) {
    case QKV_F32:
      return launch_pack_key<float>(key, slot_mapping, slot_dtype, num_tokens,
                                    num_kv_heads, head_size, group_size,
                                    block_size, num_blocks, k_quant, k_scale,
                                    k_mn, s);
    case QKV_BF16:
      return launch_pack_key<__nv_bfloat16>(
          key, slot_mapping, slot_dtype, num_tokens, num_kv_heads, head_size,
          group_size, block_size, num_blocks, k_quant, k_scale, k_mn, s);
    default:
      return launch_pack_key<__half>(key, slot_mapping, slot_dtype, num_tokens,
                                     num_kv_heads, head_size, group_size,
                                     block_size, num_blocks, k_quant, k_scale,
                                     k_mn, s);
  }
}

int qkv_kivi_pack_value(const void* value, int value_dtype,
                        const void* slot_mapping, int slot_dtype,
                        int64_t num_tokens, int num_kv_heads, int head_size,
                        int group_size, int block_size, int64_t num_blocks,
                        int32_t* v_quant, float* v_scale, float* v_mn,
                        qkv_stream_t stream) {
  using namespace qkv;
  int rc = check_common("qkv_kivi_pack_value", value_dtype, slot_dtype,
                        num_tokens, num_kv_heads, head_size, group_size,
                        block_size, num_blocks);
  if (rc != QKV_OK) return rc;
  QKV_CHECK_ARG(head_size % group_size == 0,
                "qkv_kivi_pack_value: head_size must be divisible by group_size");
  if (num_tokens == 0) return QKV_OK;
  QKV_CHECK_ARG(value && slot_mapping && v_quant && v_scale && v_mn,
                "qkv_kivi_pack_value: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (value_dtype) {
    case QKV_F32:
      return launch_pack_value<float>(value, slot_mapping, slot_dtype,
                                      num_tokens, num_kv_heads, head_size,
                                      group_size, block_size, num_blocks,
                                      v_quant, v_scale, v_mn, s);
    case QKV_BF16:
      return launch_pack_value<__nv_bfloat16>(
          value, slot_mapping, slot_dtype, num_tokens, num_kv_heads, head_size,
          group_size, block_size, num_blocks, v_quant, v_scale, v_mn, s);
    default:
      return launch_pack_value<__half>(value, slot_mapping, slot_dtype,
                                       num_tokens, num_kv_heads, head_size,
                                       group_size, block_size, num_blocks,
                                       v_quant, v_scale, v_mn, s);
  }
}

int qkv_kivi_pack_kv(const void* key, const void* value, int dtype, const void* slot_mapping, int slot_dtype,
                     int64_t num_tokens, int num_kv_heads, int head_size, int group_size, int block_size,
                     int64_t num_blocks, int32_t* k_quant, float* k_scale, float* k_mn, int32_t* v_quant,
                     float* v_scale, float* v_mn, qkv_stream_t stream) {
  using namespace qkv;
  int rc = check_common("qkv_kivi_pack_kv", dtype, slot_dtype, num_tokens, num_kv_heads, head_size, group_size,
                        block_size, num_blocks);
  if (rc != QKV_OK) return rc;
  QKV_CHECK_ARG(num_tokens % group_size == 0, "qkv_kivi_pack_kv: num_tokens must be a whole number of groups");
  QKV_CHECK_ARG(block_size % group_size == 0, "qkv_kivi_pack_kv: block_size must be divisible by group_size");
  QKV_CHECK_ARG(head_size % group_size == 0, "qkv_kivi_pack_kv: head_size must be divisible by group_size");
  if (num_tokens == 0) return QKV_OK;
  QKV_CHECK_ARG(key && value && slot_mapping && k_quant && k_scale && k_mn && v_quant && v_scale && v_mn,
                "qkv_kivi_pack_kv: null pointer");
  const auto al = [](const void* p, unsigned m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
  const bool fused = dtype == QKV_BF16 && head_size == 128 && (group_size == 64 || group_size == 128) &&
                     al(key, 3u) && al(k_quant, group_size == 128 ? 15u : 7u) && al(value, 15u) &&
                     al(v_quant, 15u) && num_tokens * num_kv_heads * 2 < (int64_t{1} << 31);
  if (!fused) {
    rc = qkv_kivi_pack_key(key, dtype, slot_mapping, slot_dtype, num_tokens, num_kv_heads, head_size, group_size,
                           block_size, num_blocks, k_quant, k_scale, k_mn, stream);
    if (rc != QKV_OK) return rc;
    return qkv_kivi_pack_value(value, dtype, slot_mapping, slot_dtype, num_tokens, num_kv_heads, head_size,
                               group_size, block_size, num_blocks, v_quant, v_scale, v_mn, stream);
  }
  const int64_t key_ctas = num_tokens / group_size * num_kv_heads;
  const int64_t value_ctas = (num_tokens * num_kv_heads * 2 + 255) / 256;
  const int64_t grid = key_ctas + value_ctas;
  QKV_CHECK_ARG(grid < (int64_t{1} << 31), "qkv_kivi_pack_kv: too many tokens for one launch");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* k = static_cast<const __nv_bfloat16*>(key);
  const auto* v = static_cast<const __nv_bfloat16*>(value);
  if (group_size == 128)
    pack_kv_fast_kernel<128><<<static_cast<unsigned>(grid), 256, 0, s>>>(
        k, v, slot_mapping, slot_dtype, num_tokens, num_kv_heads, block_size, num_blocks, k_quant, k_scale, k_mn,
        v_quant, v_scale, v_mn, device_error_ptr());
  else
    pack_kv_fast_kernel<64><<<static_cast<unsigned>(grid), 256, 0, s>>>(
        k, v, slot_mapping, slot_dtype, num_tokens, num_kv_heads, block_size, num_blocks, k_quant, k_scale, k_mn,
        v_quant, v_scale, v_mn, device_error_ptr());
  QKV_CHECK_LAUNCH("pack_kv_fast_kernel");
  return QKV_OK;
}

}  // extern "C"
