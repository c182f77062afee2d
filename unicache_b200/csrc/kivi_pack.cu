// KIVI grouped quantization, bit-packing, dequantization and fake quantization.
//
// Arithmetic contract (bit-exact with unicache/storage/physical.py:139-201 and
// unicache/operators/builtin.py:31-53): every step is one IEEE fp32 operation
// with round-to-nearest (explicit __fsub_rn/__fdiv_rn/__fmul_rn/__fadd_rn, so
// the compiler cannot contract them into FMAs), rounding to integers is
// round-half-even (rintf), and stores into bf16/fp16 round to nearest even.
// This translation unit must not be compiled with fast-math.
#include <cfloat>
#include <type_traits>

#include "common.cuh"

namespace ucb {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  return Dtype<T>::to_f(*p);
}

__device__ __forceinline__ float quant_scale(float mn, float mx, float max_code) {
  return fmaxf(__fdiv_rn(__fsub_rn(mx, mn), max_code), FLT_EPSILON);
}

__device__ __forceinline__ uint32_t quant_code(float v, float mn, float scale, float max_code) {
  float q = rintf(__fdiv_rn(__fsub_rn(v, mn), scale));
  q = fminf(fmaxf(q, 0.0f), max_code);
  return static_cast<uint32_t>(q);
}

// Codes of two values with the results of quant_code, without a division or
// a float-to-integer conversion per element.  q = RN(d * RN(1/scale)) differs
// from RN(d / scale) by less than 2^-22 q, below 2^-14 because 0 <= q <=
// max_code (1 + 2^-22) < 2^8 for finite inputs (d = RN(v - mn) lies in
// [0, RN(mx - mn)]), so unless q is within 2^-12 of a half-integer both round
// to the same integer.  Adding 1.5 * 2^23 rounds q to an integer, ties to
// even like rintf, in the low mantissa bits: the sum's bit pattern is
// kRoundBits + code, and the clamps of quant_code cannot act.  A product
// within 2^-12 of a half-integer (or not finite) takes quant_code itself.
// Returned as bit patterns kRoundBits + code, which pack_bits folds into a
// word with one shift-add each.
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kRoundBits = 0x4B400000u;

// The exact fallback, out of line: inlined at every pair of the unrolled
// loops its divisions would crowd the instruction cache for a path that is
// almost never taken.
__device__ __noinline__ uint2 quant_exact2(float2 v, float2 mn, float2 sc, float max_code) {
  return make_uint2(kRoundBits + quant_code(v.x, mn.x, sc.x, max_code),
                    kRoundBits + quant_code(v.y, mn.y, sc.y, max_code));
}

__device__ __forceinline__ uint2 quant_bits2(float2 v, float2 mn, float2 sc, float2 inv, float max_code) {
  const float2 d = __fadd2_rn(v, make_float2(-mn.x, -mn.y));
  const float2 q = __fmul2_rn(d, inv);
  const float2 t = __fadd2_rn(q, make_float2(kRound, kRound));
  const float2 c = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 e = __fadd2_rn(q, make_float2(-c.x, -c.y));
  constexpr float kEdge = 0.5f - 0x1p-12f;
  uint2 r = make_uint2(__float_as_uint(t.x), __float_as_uint(t.y));
  if (!(fabsf(e.x) < kEdge && fabsf(e.y) < kEdge)) r = quant_exact2(v, mn, sc, max_code);
  return r;
}

// What N codes of BITS bits, each carried as kRoundBits + code and added
// in at shifts 0, BITS, 2 BITS, ..., leave in a 32-bit word beyond the codes
// (arithmetic modulo 2^32).
template <int BITS, int N>
__host__ __device__ constexpr uint32_t round_bias() {
  uint32_t s = 0;
  for (int j = 0; j < N; ++j) s += kRoundBits << (j * BITS);
  return s;
}

// Element-wise minimum and maximum of two packed pairs of 16-bit values
// (NaN loses to a number, as with fminf / fmaxf; exact, no rounding).
template <typename T>
__device__ __forceinline__ uint32_t min_pair(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <typename T>
__device__ __forceinline__ uint32_t max_pair(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// ---------------------------------------------------------------- key pack
// One CTA per (token group, head); one thread per pair of adjacent channels,
// so a warp reads 64 channels (a full 128-byte line for 16-bit inputs) per
// token row.  Groups run along tokens: a thread reduces two columns of G
// values and emits G*bits/32 words per channel.  Loads are issued 32 rows at
// a time before any reduction, and 16-bit inputs are reduced as packed pairs
// (one min and one max instruction per row for both channels); for G = 32
// the raw words stay in registers for the code pass, larger groups re-read
// them from L1.
template <typename T, int BITS, int G>
__device__ __forceinline__ void pack_key_item(const T* __restrict__ x, int64_t stride_t, int64_t stride_h, int tokens,
                                              int head_dim, uint32_t* __restrict__ codes32,
                                              uint8_t* __restrict__ codes8, T* __restrict__ scale,
                                              T* __restrict__ minimum, int g, int h, int pair) {
  constexpr int CH = 32;
  constexpr bool kPair16 = sizeof(T) == 2;
  using V2 = typename Dtype<T>::vec2;
  const int d = 2 * pair;
  if (d >= head_dim) return;
  const int groups = tokens / G;
  const T* col = x + static_cast<int64_t>(g) * G * stride_t + h * stride_h + d;
  V2 w[CH];
  float mna = INFINITY, mxa = -INFINITY, mnb = INFINITY, mxb = -INFINITY;
#pragma unroll
  for (int c0 = 0; c0 < G; c0 += CH) {
#pragma unroll
    for (int i = 0; i < CH; ++i) w[i] = *reinterpret_cast<const V2*>(col + static_cast<int64_t>(c0 + i) * stride_t);
    if constexpr (kPair16) {
      uint32_t lo = w[0], hi = w[0];
#pragma unroll
      for (int i = 1; i < CH; ++i) {
        lo = min_pair<T>(lo, w[i]);
        hi = max_pair<T>(hi, w[i]);
      }
      mna = fminf(mna, Dtype<T>::lo(lo));
      mnb = fminf(mnb, Dtype<T>::hi(lo));
      mxa = fmaxf(mxa, Dtype<T>::lo(hi));
      mxb = fmaxf(mxb, Dtype<T>::hi(hi));
    } else {
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        mna = fminf(mna, Dtype<T>::lo(w[i]));
        mxa = fmaxf(mxa, Dtype<T>::lo(w[i]));
        mnb = fminf(mnb, Dtype<T>::hi(w[i]));
        mxb = fmaxf(mxb, Dtype<T>::hi(w[i]));
      }
    }
  }
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  const float sca = quant_scale(mna, mxa, kMax), scb = quant_scale(mnb, mxb, kMax);
  const float2 mn = make_float2(mna, mnb), sc = make_float2(sca, scb);
  const float2 inv = make_float2(__frcp_rn(sca), __frcp_rn(scb));
  const int64_t stat = (static_cast<int64_t>(h) * groups + g) * head_dim + d;
  scale[stat] = Dtype<T>::from_f(sca);
  scale[stat + 1] = Dtype<T>::from_f(scb);
  minimum[stat] = Dtype<T>::from_f(mna);
  minimum[stat + 1] = Dtype<T>::from_f(mnb);
#pragma unroll
  for (int c0 = 0; c0 < G; c0 += CH) {
    if (G > CH) {
#pragma unroll
      for (int i = 0; i < CH; ++i) w[i] = *reinterpret_cast<const V2*>(col + static_cast<int64_t>(c0 + i) * stride_t);
    }
    if constexpr (BITS == 8) {
      uint8_t* out = codes8 + (static_cast<int64_t>(h) * tokens + static_cast<int64_t>(g) * G + c0) * head_dim + d;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const uint2 c = quant_bits2(make_float2(Dtype<T>::lo(w[i]), Dtype<T>::hi(w[i])), mn, sc, inv, kMax);
        *reinterpret_cast<uint16_t*>(out + static_cast<int64_t>(i) * head_dim) =
            static_cast<uint16_t>(c.x + (c.y << 8) - round_bias<8, 2>());
      }
    } else {
      constexpr int F = 32 / BITS;
      uint32_t* out = codes32 + (static_cast<int64_t>(h) * (tokens / F) + (static_cast<int64_t>(g) * G + c0) / F) *
                                    head_dim + d;
#pragma unroll
      for (int k = 0; k < CH / F; ++k) {
        uint32_t wa = 0, wb = 0;
#pragma unroll
        for (int j = 0; j < F; ++j) {
          const V2 e = w[k * F + j];
          const uint2 c = quant_bits2(make_float2(Dtype<T>::lo(e), Dtype<T>::hi(e)), mn, sc, inv, kMax);
          wa += c.x << (j * BITS);
          wb += c.y << (j * BITS);
        }
        *reinterpret_cast<uint2*>(out + static_cast<int64_t>(k) * head_dim) =
            make_uint2(wa - round_bias<BITS, F>(), wb - round_bias<BITS, F>());
      }
    }
  }
}

// Group 32 with the two halves of a group on a lane pair: lanes 2p and 2p + 1
// take rows 0-15 and 16-31 of channel pair p, so a thread holds 16 raw pairs;
// the halves' packed minimum and maximum are exchanged with one shuffle, both
// lanes compute the group's statistics (lane 2p stores them) and each writes
// the codes of its own 16 rows (one word per channel for 2-bit codes).  The
// codes and statistics are those of pack_key_item<T, BITS, 32>.  Both lanes of
// a pair must reach this function.
template <int BITS>
__device__ __forceinline__ void pack_key_half_item(const __nv_bfloat16* __restrict__ x, int64_t stride_t,
                                                   int64_t stride_h, int tokens, int head_dim,
                                                   uint32_t* __restrict__ codes32, uint8_t* __restrict__ codes8,
                                                   __nv_bfloat16* __restrict__ scale,
                                                   __nv_bfloat16* __restrict__ minimum, int g, int h, int pair,
                                                   int half) {
  using T = __nv_bfloat16;
  constexpr int G = 32, R = 16;
  const int d = 2 * pair;
  const int groups = tokens / G;
  const T* col = x + (static_cast<int64_t>(g) * G + half * R) * stride_t + h * stride_h + d;
  uint32_t w[R];
#pragma unroll
  for (int i = 0; i < R; ++i) w[i] = *reinterpret_cast<const uint32_t*>(col + static_cast<int64_t>(i) * stride_t);
  uint32_t lo = w[0], hi = w[0];
#pragma unroll
  for (int i = 1; i < R; ++i) {
    lo = min_pair<T>(lo, w[i]);
    hi = max_pair<T>(hi, w[i]);
  }
  const unsigned pair_mask = 3u << ((threadIdx.x & 31) & ~1);
  lo = min_pair<T>(lo, __shfl_xor_sync(pair_mask, lo, 1));
  hi = max_pair<T>(hi, __shfl_xor_sync(pair_mask, hi, 1));
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  const float mna = Dtype<T>::lo(lo), mnb = Dtype<T>::hi(lo);
  const float sca = quant_scale(mna, Dtype<T>::lo(hi), kMax), scb = quant_scale(mnb, Dtype<T>::hi(hi), kMax);
  const float2 mn = make_float2(mna, mnb), sc = make_float2(sca, scb);
  const float2 inv = make_float2(__frcp_rn(sca), __frcp_rn(scb));
  if (half == 0) {
    const int64_t stat = (static_cast<int64_t>(h) * groups + g) * head_dim + d;
    scale[stat] = Dtype<T>::from_f(sca);
    scale[stat + 1] = Dtype<T>::from_f(scb);
    minimum[stat] = Dtype<T>::from_f(mna);
    minimum[stat + 1] = Dtype<T>::from_f(mnb);
  }
  const int64_t row0 = static_cast<int64_t>(g) * G + half * R;
  if constexpr (BITS == 8) {
    uint8_t* out = codes8 + (static_cast<int64_t>(h) * tokens + row0) * head_dim + d;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const uint2 c = quant_bits2(make_float2(Dtype<T>::lo(w[i]), Dtype<T>::hi(w[i])), mn, sc, inv, kMax);
      *reinterpret_cast<uint16_t*>(out + static_cast<int64_t>(i) * head_dim) =
          static_cast<uint16_t>(c.x + (c.y << 8) - round_bias<8, 2>());
    }
  } else {
    constexpr int F = 32 / BITS;
    uint32_t* out = codes32 + (static_cast<int64_t>(h) * (tokens / F) + row0 / F) * head_dim + d;
#pragma unroll
    for (int k = 0; k < R / F; ++k) {
      uint32_t wa = 0, wb = 0;
#pragma unroll
      for (int j = 0; j < F; ++j) {
        const uint32_t e = w[k * F + j];
        const uint2 c = quant_bits2(make_float2(Dtype<T>::lo(e), Dtype<T>::hi(e)), mn, sc, inv, kMax);
        wa += c.x << (j * BITS);
        wb += c.y << (j * BITS);
      }
      *reinterpret_cast<uint2*>(out + static_cast<int64_t>(k) * head_dim) =
          make_uint2(wa - round_bias<BITS, F>(), wb - round_bias<BITS, F>());
    }
  }
}

template <typename T, int BITS, int G>
__global__ void __launch_bounds__(64) pack_key_kernel(const T* __restrict__ x, int64_t stride_t,
                                                      int64_t stride_h, int tokens, int head_dim,
                                                      uint32_t* __restrict__ codes32,
                                                      uint8_t* __restrict__ codes8,
                                                      T* __restrict__ scale, T* __restrict__ minimum) {
  pack_key_item<T, BITS, G>(x, stride_t, stride_h, tokens, head_dim, codes32, codes8, scale, minimum, blockIdx.x,
                            blockIdx.y, threadIdx.x);
}

// ---------------------------------------------------------------- value pack
// One thread per (token row, channel group): it reads the group's G channels
// with 16-byte loads, reduces them locally (16-bit inputs as packed pairs)
// and writes G*bits/32 words and its two statistics.  Consecutive threads
// take consecutive groups of consecutive rows, so a warp reads one
// contiguous span of the input.
template <typename T, int BITS, int D, int G, bool VEC>
__device__ __forceinline__ void pack_value_item(const T* __restrict__ x, int64_t stride_t, int64_t stride_h,
                                                int tokens, int heads, uint32_t* __restrict__ codes32,
                                                uint8_t* __restrict__ codes8, T* __restrict__ scale,
                                                T* __restrict__ minimum, int64_t item) {
  constexpr int NG = D / G;                     // groups per row
  constexpr int EPV = 16 / (int)sizeof(T);      // elements per 16-byte load
  constexpr bool kPair16 = VEC && sizeof(T) == 2;
  const int64_t n_items = static_cast<int64_t>(tokens) * heads * NG;
  if (item >= n_items) return;
  const int gi = static_cast<int>(item % NG);
  const int64_t row = item / NG;
  const int t = static_cast<int>(row / heads), h = static_cast<int>(row % heads);
  const T* src = x + t * stride_t + h * stride_h + gi * G;
  // the group as G/2 pairs: raw 16-bit pairs, or fp32 pairs
  uint32_t r[kPair16 ? G / 2 : 1];
  float v[kPair16 ? 1 : G];
  float mn, mx;
  if constexpr (kPair16) {
#pragma unroll
    for (int c = 0; c < G / 2; c += 4) {
      const uint4 raw = *reinterpret_cast<const uint4*>(src + 2 * c);
      r[c] = raw.x;
      r[c + 1] = raw.y;
      r[c + 2] = raw.z;
      r[c + 3] = raw.w;
    }
    uint32_t lo = r[0], hi = r[0];
#pragma unroll
    for (int j = 1; j < G / 2; ++j) {
      lo = min_pair<T>(lo, r[j]);
      hi = max_pair<T>(hi, r[j]);
    }
    mn = fminf(Dtype<T>::lo(lo), Dtype<T>::hi(lo));
    mx = fmaxf(Dtype<T>::lo(hi), Dtype<T>::hi(hi));
  } else {
    if constexpr (VEC) {  // 16-byte aligned rows
#pragma unroll
      for (int c = 0; c < G; c += EPV) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + c);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int j = 0; j < EPV; ++j) v[c + j] = Dtype<T>::to_f(e[j]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < G; ++c) v[c] = ld(src + c);
    }
    mn = v[0];
    mx = v[0];
#pragma unroll
    for (int j = 1; j < G; ++j) {
      mn = fminf(mn, v[j]);
      mx = fmaxf(mx, v[j]);
    }
  }
  // values 2p and 2p + 1 of the group as fp32
  auto pair_at = [&](int p) {
    if constexpr (kPair16)
      return make_float2(Dtype<T>::lo(r[p]), Dtype<T>::hi(r[p]));
    else
      return make_float2(v[2 * p], v[2 * p + 1]);
  };
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  const float sc = quant_scale(mn, mx, kMax);
  const float inv = __frcp_rn(sc);
  const float2 mn2 = make_float2(mn, mn), sc2 = make_float2(sc, sc), inv2 = make_float2(inv, inv);
  const int64_t out_row = static_cast<int64_t>(h) * tokens + t;
  scale[out_row * NG + gi] = Dtype<T>::from_f(sc);
  minimum[out_row * NG + gi] = Dtype<T>::from_f(mn);
  if constexpr (BITS == 8) {
    uint8_t* out = codes8 + out_row * D + gi * G;
#pragma unroll
    for (int c = 0; c < G; c += 16) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w[q] = 0;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          const uint2 cc = quant_bits2(pair_at((c + 4 * q + j) / 2), mn2, sc2, inv2, kMax);
          w[q] += (cc.x << (8 * j)) + (cc.y << (8 * (j + 1)));
        }
        w[q] -= round_bias<8, 4>();
      }
      *reinterpret_cast<uint4*>(out + c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    constexpr int F = 32 / BITS;
    constexpr int W = G / F;  // words per group: 2-bit 2/4/8, 4-bit 4/8/16
    uint32_t w[W];
#pragma unroll
    for (int k = 0; k < W; ++k) {
      w[k] = 0;
#pragma unroll
      for (int j = 0; j < F; j += 2) {
        const uint2 cc = quant_bits2(pair_at((k * F + j) / 2), mn2, sc2, inv2, kMax);
        w[k] += (cc.x << (j * BITS)) + (cc.y << ((j + 1) * BITS));
      }
      w[k] -= round_bias<BITS, F>();
    }
    uint32_t* out = codes32 + out_row * (D / F) + gi * W;
#pragma unroll
    for (int k = 0; k < W; k += 2) *reinterpret_cast<uint2*>(out + k) = make_uint2(w[k], w[k + 1]);
  }
}

template <typename T, int BITS, int D, int G, bool VEC>
__global__ void __launch_bounds__(256) pack_value_kernel(const T* __restrict__ x, int64_t stride_t,
                                                         int64_t stride_h, int tokens, int heads,
                                                         uint32_t* __restrict__ codes32,
                                                         uint8_t* __restrict__ codes8,
                                                         T* __restrict__ scale, T* __restrict__ minimum) {
  pack_value_item<T, BITS, D, G, VEC>(x, stride_t, stride_h, tokens, heads, codes32, codes8, scale, minimum,
                                      static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
}

// ---------------------------------------------------------------- fused key + value pack
// One launch for both halves of PackedKIVICache.from_dense's pack step: blocks
// [0, key_blocks) quantize keys, two (token group, head) items per 256-thread
// block with a lane pair per channel pair (pack_key_half_item); the remaining
// blocks quantize values, one (token row, channel group) per thread.  The
// codes and statistics equal the separate kernels'; one launch instead of
// two saves one launch and one memory ramp per sequence.  Built for group 32
// only.  Six blocks per SM (40 registers, a 12-byte spill) beat four or five
// without a spill and eight (32 registers, an 84-byte spill): each thread's
// load -> reduce -> store pass is latency-bound, so resident warps count most.
struct PackSide {
  const void* x;
  int64_t stride_t, stride_h;
  void* codes;
  void* scale;
  void* minimum;
};

template <int KB, int VB, int G>
__global__ void __launch_bounds__(256, 6) pack_kv_kernel(PackSide k, PackSide v, int tokens, int heads, int key_blocks) {
  using T = __nv_bfloat16;
  constexpr int D = 128, LANES = D, ITEMS = 256 / LANES;  // a lane pair per channel pair
  static_assert(G == 32, "the fused kernels run group 32");
  if (static_cast<int>(blockIdx.x) < key_blocks) {
    const int groups = tokens / G;
    const int item = blockIdx.x * ITEMS + threadIdx.x / LANES;
    if (item >= groups * heads) return;
    pack_key_half_item<KB>(static_cast<const T*>(k.x), k.stride_t, k.stride_h, tokens, D,
                           static_cast<uint32_t*>(k.codes), static_cast<uint8_t*>(k.codes),
                           static_cast<T*>(k.scale), static_cast<T*>(k.minimum), item % groups, item / groups,
                           (threadIdx.x % LANES) >> 1, threadIdx.x & 1);
  } else {
    const int64_t item = static_cast<int64_t>(blockIdx.x - key_blocks) * 256 + threadIdx.x;
    pack_value_item<T, VB, D, G, true>(static_cast<const T*>(v.x), v.stride_t, v.stride_h, tokens, heads,
                                       static_cast<uint32_t*>(v.codes), static_cast<uint8_t*>(v.codes),
                                       static_cast<T*>(v.scale), static_cast<T*>(v.minimum), item);
  }
}

// Many segments in one launch: blockIdx.y picks a job (one segment's key and
// value sides and its token count), blockIdx.x runs the fused kernel's block
// index inside that job; blocks past a shorter job's end exit.  One launch
// (and one memory ramp) packs a whole batch of sequences.
struct PackJob {
  PackSide k, v;
  int tokens, key_blocks, blocks, pad;
};

template <int KB, int VB, int G>
__global__ void __launch_bounds__(256, 6) pack_kv_batched_kernel(const PackJob* __restrict__ jobs, int heads) {
  using T = __nv_bfloat16;
  constexpr int D = 128, LANES = D, ITEMS = 256 / LANES;  // a lane pair per channel pair
  static_assert(G == 32, "the fused kernels run group 32");
  const PackJob& j = jobs[blockIdx.y];
  const int b = static_cast<int>(blockIdx.x);
  if (b >= j.blocks) return;
  if (b < j.key_blocks) {
    const int groups = j.tokens / G;
    const int item = b * ITEMS + threadIdx.x / LANES;
    if (item >= groups * heads) return;
    pack_key_half_item<KB>(static_cast<const T*>(j.k.x), j.k.stride_t, j.k.stride_h, j.tokens, D,
                           static_cast<uint32_t*>(j.k.codes), static_cast<uint8_t*>(j.k.codes),
                           static_cast<T*>(j.k.scale), static_cast<T*>(j.k.minimum), item % groups, item / groups,
                           (threadIdx.x % LANES) >> 1, threadIdx.x & 1);
  } else {
    const int64_t item = static_cast<int64_t>(b - j.key_blocks) * 256 + threadIdx.x;
    pack_value_item<T, VB, D, G, true>(static_cast<const T*>(j.v.x), j.v.stride_t, j.v.stride_h, j.tokens, heads,
                                       static_cast<uint32_t*>(j.v.codes), static_cast<uint8_t*>(j.v.codes),
                                       static_cast<T*>(j.v.scale), static_cast<T*>(j.v.minimum), item);
  }
}

// ---------------------------------------------------------------- dequantize
__device__ __forceinline__ float dequant(uint32_t code, float s, float m) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), s), m);
}

// Key: one CTA per (token tile of 32, head), one thread per channel.
template <typename ST, typename OT, int BITS>
__global__ void __launch_bounds__(128) dequant_key_kernel(const void* __restrict__ codes,
                                                          const ST* __restrict__ scale,
                                                          const ST* __restrict__ minimum, int tokens,
                                                          int head_dim, int group, int t0, int n,
                                                          OT* __restrict__ out, int64_t ost_t,
                                                          int64_t ost_h) {
  const int h = blockIdx.y, d = threadIdx.x;
  if (d >= head_dim) return;
  const int i0 = blockIdx.x * 32;
  const int i1 = min(n, i0 + 32);
  constexpr uint32_t kMask = (BITS == 8) ? 0xFFu : ((1u << BITS) - 1u);
  const int groups = tokens / group;
  for (int i = i0; i < i1; ++i) {
    const int t = t0 + i;
    uint32_t code;
    if constexpr (BITS == 8) {
      code = static_cast<const uint8_t*>(codes)[(static_cast<int64_t>(h) * tokens + t) * head_dim + d];
    } else {
      constexpr int F = 32 / BITS;
      const uint32_t w =
          static_cast<const uint32_t*>(codes)[(static_cast<int64_t>(h) * (tokens / F) + t / F) * head_dim + d];
      code = (w >> ((t % F) * BITS)) & kMask;
    }
    const int64_t stat = (static_cast<int64_t>(h) * groups + t / group) * head_dim + d;
    const float v = dequant(code, Dtype<ST>::to_f(scale[stat]), Dtype<ST>::to_f(minimum[stat]));
    out[i * ost_t + h * ost_h + d] = Dtype<OT>::from_f(v);
  }
}

// Value: one thread per (token, head, channel).
template <typename ST, typename OT, int BITS>
__global__ void __launch_bounds__(256) dequant_value_kernel(const void* __restrict__ codes,
                                                            const ST* __restrict__ scale,
                                                            const ST* __restrict__ minimum, int tokens,
                                                            int heads, int head_dim, int group, int t0,
                                                            int n, OT* __restrict__ out, int64_t ost_t,
                                                            int64_t ost_h) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(n) * heads * head_dim;
  if (idx >= total) return;
  const int d = static_cast<int>(idx % head_dim);
  const int h = static_cast<int>((idx / head_dim) % heads);
  const int i = static_cast<int>(idx / (static_cast<int64_t>(head_dim) * heads));
  const int t = t0 + i;
  const int64_t row = static_cast<int64_t>(h) * tokens + t;
  uint32_t code;
  if constexpr (BITS == 8) {
    code = static_cast<const uint8_t*>(codes)[row * head_dim + d];
  } else {
    constexpr int F = 32 / BITS;
    const uint32_t w = static_cast<const uint32_t*>(codes)[row * (head_dim / F) + d / F];
    code = (w >> ((d % F) * BITS)) & ((1u << BITS) - 1u);
  }
  const int64_t stat = row * (head_dim / group) + d / group;
  const float v = dequant(code, Dtype<ST>::to_f(scale[stat]), Dtype<ST>::to_f(minimum[stat]));
  out[i * ost_t + h * ost_h + d] = Dtype<OT>::from_f(v);
}

// ---------------------------------------------------------------- fake quantization
template <typename T>
__global__ void fake_quant_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t outer,
                                  int64_t length, int64_t inner, int group, float max_code) {
  const int64_t n_groups = (length + group - 1) / group;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= outer * n_groups * inner) return;
  const int64_t i = idx % inner;
  const int64_t gidx = (idx / inner) % n_groups;
  const int64_t o = idx / (inner * n_groups);
  const int64_t start = gidx * group;
  const int64_t stop = min(length, start + group);
  const int64_t base = o * length * inner + i;
  // The group's elements are read CH at a time (all CH loads in flight
  // before the first is used) and folded in element order, as a plain loop
  // over the group would fold them.
  constexpr int CH = 16;
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t l0 = start; l0 < stop; l0 += CH) {
    float v[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = l0 + j < stop ? ld(x + base + (l0 + j) * inner) : 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (l0 + j < stop) {
        mn = fminf(mn, v[j]);
        mx = fmaxf(mx, v[j]);
      }
  }
  // builtin.py:50 clamps the range before dividing (unlike the packed quantizer).
  const float sc = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), FLT_EPSILON), max_code);
  for (int64_t l0 = start; l0 < stop; l0 += CH) {
    float v[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = l0 + j < stop ? ld(x + base + (l0 + j) * inner) : 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (l0 + j < stop) {
        const float q = static_cast<float>(quant_code(v[j], mn, sc, max_code));
        out[base + (l0 + j) * inner] = Dtype<T>::from_f(__fadd_rn(__fmul_rn(q, sc), mn));
      }
  }
}

// Groups of `group` contiguous elements (the quantized dimension is the
// innermost one and every group is full): one thread per group reads it with
// 16-byte loads, four in flight at a time, folds min and max in element
// order and writes the fake-quantized group with 16-byte stores.  Same
// arithmetic as fake_quant_kernel.  group % (16 / sizeof(T)) == 0 and 16-byte
// aligned tensors.
template <typename T>
__global__ void fake_quant_rows_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t groups, int group,
                                       float max_code) {
  constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte vector
  constexpr int UNROLL = 4;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + g * group);
  uint4* dst = reinterpret_cast<uint4*>(out + g * group);
  const int vecs = group / EPV;
  float mn = INFINITY, mx = -INFINITY;
  for (int c0 = 0; c0 < vecs; c0 += UNROLL) {
    uint4 w[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) w[u] = c0 + u < vecs ? src[c0 + u] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      if (c0 + u < vecs) {
        const T* e = reinterpret_cast<const T*>(&w[u]);
#pragma unroll
        for (int j = 0; j < EPV; ++j) {
          const float v = Dtype<T>::to_f(e[j]);
          mn = fminf(mn, v);
          mx = fmaxf(mx, v);
        }
      }
  }
  const float sc = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), FLT_EPSILON), max_code);
  for (int c0 = 0; c0 < vecs; c0 += UNROLL) {
    uint4 w[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) w[u] = c0 + u < vecs ? src[c0 + u] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      if (c0 + u < vecs) {
        T* e = reinterpret_cast<T*>(&w[u]);
#pragma unroll
        for (int j = 0; j < EPV; ++j) {
          const float q = static_cast<float>(quant_code(Dtype<T>::to_f(e[j]), mn, sc, max_code));
          e[j] = Dtype<T>::from_f(__fadd_rn(__fmul_rn(q, sc), mn));
        }
        dst[c0 + u] = w[u];
      }
  }
}

}  // namespace
}  // namespace ucb

using ucb_host::check_launch;
using ucb_host::set_error;

namespace {

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

int validate_pack(const char* what, const void* x, int dtype, int64_t tokens, int64_t heads, int64_t head_dim,
                  int bits, int group, const void* codes, const void* scale, const void* minimum) {
  if (!x || !codes || !scale || !minimum) return set_error(UCB_ERR_INVALID, "%s: null pointer", what);
  if (dtype != UCB_BF16 && dtype != UCB_F16 && dtype != UCB_F32)
    return set_error(UCB_ERR_INVALID, "%s: dtype %d unsupported", what, dtype);
  if (bits != 2 && bits != 4 && bits != 8)
    return set_error(UCB_ERR_INVALID, "%s: bits must be 2, 4 or 8 (got %d)", what, bits);
  if (head_dim != 64 && head_dim != 128)
    return set_error(UCB_ERR_UNSUPPORTED, "%s: head_dim must be 64 or 128 (got %lld)", what, (long long)head_dim);
  if (group != 32 && group != 64 && group != 128)
    return set_error(UCB_ERR_UNSUPPORTED, "%s: group_size must be 32, 64 or 128 (got %d)", what, group);
  if (tokens <= 0 || heads <= 0 || tokens > (1LL << 30) || heads > 1024)
    return set_error(UCB_ERR_INVALID, "%s: bad tokens/heads (%lld, %lld)", what, (long long)tokens, (long long)heads);
  return UCB_OK;
}

template <typename T>
int launch_pack_key(const void* x, int64_t T_, int64_t H, int64_t D, int64_t st, int64_t sh, int bits,
                    int group, void* codes, void* scale, void* minimum, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>(T_ / group), static_cast<unsigned>(H));
  const T* xp = static_cast<const T*>(x);
  auto* c32 = static_cast<uint32_t*>(codes);
  auto* c8 = static_cast<uint8_t*>(codes);
  T* sp = static_cast<T*>(scale);
  T* mp = static_cast<T*>(minimum);
#define UCB_PACK_KEY(B_, G_) \
  if (bits == B_ && group == G_) { \
    ucb::pack_key_kernel<T, B_, G_><<<grid, (unsigned)(D / 2), 0, s>>>(xp, st, sh, (int)T_, (int)D, c32, c8, sp, mp); \
    return check_launch("pack_key_kernel"); \
  }
  UCB_PACK_KEY(2, 32) UCB_PACK_KEY(2, 64) UCB_PACK_KEY(2, 128)
  UCB_PACK_KEY(4, 32) UCB_PACK_KEY(4, 64) UCB_PACK_KEY(4, 128)
  UCB_PACK_KEY(8, 32) UCB_PACK_KEY(8, 64) UCB_PACK_KEY(8, 128)
#undef UCB_PACK_KEY
  return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_key: unsupported (bits=%d, group=%d)", bits, group);
}

template <typename T, int BITS, int D>
int launch_pack_value_g(const void* x, int64_t T_, int64_t H, int64_t st, int64_t sh, int group, void* codes,
                        void* scale, void* minimum, cudaStream_t s) {
  const int64_t items = T_ * H * (D / group);  // one thread per (row, channel group)
  dim3 grid(static_cast<unsigned>((items + 255) / 256));
  const T* xp = static_cast<const T*>(x);
  auto* c32 = static_cast<uint32_t*>(codes);
  auto* c8 = static_cast<uint8_t*>(codes);
  T* sp = static_cast<T*>(scale);
  T* mp = static_cast<T*>(minimum);
  constexpr int EPV = 16 / (int)sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && st % EPV == 0 && sh % EPV == 0;
#define UCB_PACK_VALUE(G_)                                                                                 \
  if (group == G_) {                                                                                       \
    if constexpr (G_ <= D) {                                                                               \
      if (vec)                                                                                             \
        ucb::pack_value_kernel<T, BITS, D, G_, true><<<grid, 256, 0, s>>>(xp, st, sh, (int)T_, (int)H, c32, c8, sp, mp); \
      else                                                                                                 \
        ucb::pack_value_kernel<T, BITS, D, G_, false><<<grid, 256, 0, s>>>(xp, st, sh, (int)T_, (int)H, c32, c8, sp, mp); \
      return check_launch("pack_value_kernel");                                                            \
    }                                                                                                      \
  }
  UCB_PACK_VALUE(32) UCB_PACK_VALUE(64) UCB_PACK_VALUE(128)
#undef UCB_PACK_VALUE
  return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_value: unsupported (head_dim=%d, group=%d)", D, group);
}

template <typename T, int D>
int launch_pack_value_b(const void* x, int64_t T_, int64_t H, int64_t st, int64_t sh, int bits, int group,
                        void* codes, void* scale, void* minimum, cudaStream_t s) {
  if (bits == 2) return launch_pack_value_g<T, 2, D>(x, T_, H, st, sh, group, codes, scale, minimum, s);
  if (bits == 4) return launch_pack_value_g<T, 4, D>(x, T_, H, st, sh, group, codes, scale, minimum, s);
  return launch_pack_value_g<T, 8, D>(x, T_, H, st, sh, group, codes, scale, minimum, s);
}

template <typename T>
int launch_pack_value(const void* x, int64_t T_, int64_t H, int64_t D, int64_t st, int64_t sh, int bits,
                      int group, void* codes, void* scale, void* minimum, cudaStream_t s) {
  if (D == 128) return launch_pack_value_b<T, 128>(x, T_, H, st, sh, bits, group, codes, scale, minimum, s);
  return launch_pack_value_b<T, 64>(x, T_, H, st, sh, bits, group, codes, scale, minimum, s);
}

template <typename ST, typename OT>
int launch_dequant(bool key, const void* codes, const void* scale, const void* minimum, int64_t T_,
                   int64_t H, int64_t D, int bits, int group, int64_t t0, int64_t t1, void* out,
                   int64_t ost_t, int64_t ost_h, cudaStream_t s) {
  const int n = static_cast<int>(t1 - t0);
  const ST* sp = static_cast<const ST*>(scale);
  const ST* mp = static_cast<const ST*>(minimum);
  OT* op = static_cast<OT*>(out);
  if (key) {
    dim3 grid(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>(H));
    if (bits == 2)
      ucb::dequant_key_kernel<ST, OT, 2><<<grid, 128, 0, s>>>(codes, sp, mp, (int)T_, (int)D, group, (int)t0, n, op, ost_t, ost_h);
    else if (bits == 4)
      ucb::dequant_key_kernel<ST, OT, 4><<<grid, 128, 0, s>>>(codes, sp, mp, (int)T_, (int)D, group, (int)t0, n, op, ost_t, ost_h);
    else
      ucb::dequant_key_kernel<ST, OT, 8><<<grid, 128, 0, s>>>(codes, sp, mp, (int)T_, (int)D, group, (int)t0, n, op, ost_t, ost_h);
    return check_launch("dequant_key_kernel");
  }
  const int64_t total = static_cast<int64_t>(n) * H * D;
  dim3 grid(static_cast<unsigned>((total + 255) / 256));
  if (bits == 2)
    ucb::dequant_value_kernel<ST, OT, 2><<<grid, 256, 0, s>>>(codes, sp, mp, (int)T_, (int)H, (int)D, group, (int)t0, n, op, ost_t, ost_h);
  else if (bits == 4)
    ucb::dequant_value_kernel<ST, OT, 4><<<grid, 256, 0, s>>>(codes, sp, mp, (int)T_, (int)H, (int)D, group, (int)t0, n, op, ost_t, ost_h);
  else
    ucb::dequant_value_kernel<ST, OT, 8><<<grid, 256, 0, s>>>(codes, sp, mp, (int)T_, (int)H, (int)D, group, (int)t0, n, op, ost_t, ost_h);
  return check_launch("dequant_value_kernel");
}

template <typename ST>
int dispatch_dequant_out(bool key, int out_dtype, const void* codes, const void* scale, const void* minimum,
                         int64_t T_, int64_t H, int64_t D, int bits, int group, int64_t t0, int64_t t1,
                         void* out, int64_t ost_t, int64_t ost_h, cudaStream_t s) {
  switch (out_dtype) {
    case UCB_BF16:
      return launch_dequant<ST, __nv_bfloat16>(key, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
    case UCB_F16:
      return launch_dequant<ST, __half>(key, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
    default:
      return launch_dequant<ST, float>(key, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
  }
}

int dequant_entry(bool key, const void* codes, const void* scale, const void* minimum, int stat_dtype,
                  int64_t T_, int64_t H, int64_t D, int bits, int group, int64_t t0, int64_t t1, void* out,
                  int out_dtype, int64_t ost_t, int64_t ost_h, void* stream) {
  const char* what = key ? "ucb_kivi_dequant_key" : "ucb_kivi_dequant_value";
  int rc = validate_pack(what, codes, stat_dtype, T_, H, D, bits, group, codes, scale, minimum);
  if (rc) return rc;
  if (!out) return set_error(UCB_ERR_INVALID, "%s: null output", what);
  if (out_dtype != UCB_BF16 && out_dtype != UCB_F16 && out_dtype != UCB_F32)
    return set_error(UCB_ERR_INVALID, "%s: out dtype %d unsupported", what, out_dtype);
  if (key && T_ % group) return set_error(UCB_ERR_INVALID, "%s: tokens %% group_size != 0", what);
  if (!key && D % group) return set_error(UCB_ERR_INVALID, "%s: head_dim %% group_size != 0", what);
  if (t0 < 0 || t1 > T_ || t1 < t0) return set_error(UCB_ERR_INVALID, "%s: bad token range", what);
  if (t1 == t0) return UCB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (stat_dtype) {
    case UCB_BF16:
      return dispatch_dequant_out<__nv_bfloat16>(key, out_dtype, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
    case UCB_F16:
      return dispatch_dequant_out<__half>(key, out_dtype, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
    default:
      return dispatch_dequant_out<float>(key, out_dtype, codes, scale, minimum, T_, H, D, bits, group, t0, t1, out, ost_t, ost_h, s);
  }
}

}  // namespace

extern "C" int ucb_kivi_pack_key(const void* x, int dtype, int64_t tokens, int64_t heads, int64_t head_dim,
                                  int64_t stride_token, int64_t stride_head, int bits, int group_size,
                                  void* codes, void* scale, void* minimum, void* stream) {
  int rc = validate_pack("ucb_kivi_pack_key", x, dtype, tokens, heads, head_dim, bits, group_size, codes, scale, minimum);
  if (rc) return rc;
  if (tokens % group_size)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_key: tokens (%lld) must be a multiple of group_size (%d)",
                     (long long)tokens, group_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UCB_BF16:
      return launch_pack_key<__nv_bfloat16>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
    case UCB_F16:
      return launch_pack_key<__half>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
    default:
      return launch_pack_key<float>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
  }
}

extern "C" int ucb_kivi_pack_value(const void* x, int dtype, int64_t tokens, int64_t heads, int64_t head_dim,
                                    int64_t stride_token, int64_t stride_head, int bits, int group_size,
                                    void* codes, void* scale, void* minimum, void* stream) {
  int rc = validate_pack("ucb_kivi_pack_value", x, dtype, tokens, heads, head_dim, bits, group_size, codes, scale, minimum);
  if (rc) return rc;
  if (head_dim % group_size)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_value: head_dim must be a multiple of group_size");
  if (head_dim == 64 && group_size == 128)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_value: group_size exceeds head_dim");
  const int elem = dtype == UCB_F32 ? 4 : 2;
  const int vpl_bytes = static_cast<int>(head_dim / 32) * elem;
  if (!aligned(x, vpl_bytes) || (stride_token * elem) % vpl_bytes || (stride_head * elem) % vpl_bytes)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_value: rows must be %d-byte aligned", vpl_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UCB_BF16:
      return launch_pack_value<__nv_bfloat16>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
    case UCB_F16:
      return launch_pack_value<__half>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
    default:
      return launch_pack_value<float>(x, tokens, heads, head_dim, stride_token, stride_head, bits, group_size, codes, scale, minimum, s);
  }
}

extern "C" int ucb_kivi_pack_kv(const void* key, const void* value, int dtype, int64_t tokens, int64_t heads,
                                int64_t head_dim, int64_t key_stride_token, int64_t key_stride_head,
                                int64_t value_stride_token, int64_t value_stride_head, int k_bits, int v_bits,
                                int group_size, void* key_codes, void* key_scale, void* key_minimum,
                                void* value_codes, void* value_scale, void* value_minimum, void* stream) {
  int rc = validate_pack("ucb_kivi_pack_kv", key, dtype, tokens, heads, head_dim, k_bits, group_size, key_codes,
                         key_scale, key_minimum);
  if (rc) return rc;
  rc = validate_pack("ucb_kivi_pack_kv", value, dtype, tokens, heads, head_dim, v_bits, group_size, value_codes,
                     value_scale, value_minimum);
  if (rc) return rc;
  if (tokens % group_size)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_kv: tokens (%lld) must be a multiple of group_size (%d)",
                     (long long)tokens, group_size);
  if (dtype != UCB_BF16 || head_dim != 128 || group_size != 32)
    return set_error(UCB_ERR_UNSUPPORTED,
                     "ucb_kivi_pack_kv: bf16, head_dim 128, group 32 only (use the separate entries)");
  if (!aligned(value, 16) || value_stride_token % 8 || value_stride_head % 8)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_kv: value rows must be 16-byte aligned");
  if ((tokens / group_size) * heads > (1LL << 31) - 1 || tokens * heads * (head_dim / group_size) > (1LL << 40))
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_kv: problem too large");
  const ucb::PackSide k{key, key_stride_token, key_stride_head, key_codes, key_scale, key_minimum};
  const ucb::PackSide v{value, value_stride_token, value_stride_head, value_codes, value_scale, value_minimum};
  const int key_blocks = static_cast<int>(((tokens / group_size) * heads + 1) / 2);
  const int64_t value_items = tokens * heads * (head_dim / group_size);
  const int64_t blocks = key_blocks + (value_items + 255) / 256;
  if (blocks > 0x7fffffffLL) return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_kv: problem too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define UCB_PACK_KV(KB_, VB_, G_)                                                                             \
  if (k_bits == KB_ && v_bits == VB_ && group_size == G_) {                                                   \
    ucb::pack_kv_kernel<KB_, VB_, G_><<<static_cast<unsigned>(blocks), 256, 0, s>>>(k, v, (int)tokens, (int)heads, \
                                                                                     key_blocks);              \
    return check_launch("pack_kv_kernel");                                                                    \
  }
#define UCB_PACK_KV_G(KB_, VB_) UCB_PACK_KV(KB_, VB_, 32)
  UCB_PACK_KV_G(2, 2) UCB_PACK_KV_G(2, 4) UCB_PACK_KV_G(2, 8)
  UCB_PACK_KV_G(4, 2) UCB_PACK_KV_G(4, 4) UCB_PACK_KV_G(4, 8)
  UCB_PACK_KV_G(8, 2) UCB_PACK_KV_G(8, 4) UCB_PACK_KV_G(8, 8)
#undef UCB_PACK_KV_G
#undef UCB_PACK_KV
  return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_kv: unsupported (bits %d/%d, group %d)", k_bits, v_bits,
                   group_size);
}

extern "C" int ucb_kivi_dequant_key(const void* codes, const void* scale, const void* minimum, int stat_dtype,
                                     int64_t quantized_tokens, int64_t heads, int64_t head_dim, int bits,
                                     int group_size, int64_t token_begin, int64_t token_end, void* out,
                                     int out_dtype, int64_t out_stride_token, int64_t out_stride_head,
                                     void* stream) {
  return dequant_entry(true, codes, scale, minimum, stat_dtype, quantized_tokens, heads, head_dim, bits,
                       group_size, token_begin, token_end, out, out_dtype, out_stride_token, out_stride_head,
                       stream);
}

extern "C" int ucb_kivi_dequant_value(const void* codes, const void* scale, const void* minimum,
                                       int stat_dtype, int64_t quantized_tokens, int64_t heads,
                                       int64_t head_dim, int bits, int group_size, int64_t token_begin,
                                       int64_t token_end, void* out, int out_dtype, int64_t out_stride_token,
                                       int64_t out_stride_head, void* stream) {
  return dequant_entry(false, codes, scale, minimum, stat_dtype, quantized_tokens, heads, head_dim, bits,
                       group_size, token_begin, token_end, out, out_dtype, out_stride_token, out_stride_head,
                       stream);
}

extern "C" int ucb_fake_quant(const void* x, void* out, int dtype, int64_t outer, int64_t length, int64_t inner,
                              int bits, int group_size, void* stream) {
  if (!x || !out) return set_error(UCB_ERR_INVALID, "ucb_fake_quant: null pointer");
  if (bits != 2 && bits != 3 && bits != 4 && bits != 8)
    return set_error(UCB_ERR_INVALID, "ucb_fake_quant: unsupported bits %d", bits);
  if (outer < 0 || length < 0 || inner < 0) return set_error(UCB_ERR_INVALID, "ucb_fake_quant: negative size");
  if (outer * length * inner == 0) return UCB_OK;
  // builtin.py:23-26: the group is clamped to [1, length].
  const int group = static_cast<int>(group_size < 1 ? 1 : (group_size > length ? length : group_size));
  const int64_t n_groups = (length + group - 1) / group;
  const int64_t work = outer * n_groups * inner;
  const float max_code = static_cast<float>((1 << bits) - 1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int esize = dtype == UCB_F32 ? 4 : 2;
  if (inner == 1 && length % group == 0 && group % (16 / esize) == 0 && aligned(x, 16) && aligned(out, 16) &&
      (dtype == UCB_BF16 || dtype == UCB_F16 || dtype == UCB_F32)) {
    // contiguous full groups: one thread per group, 16-byte accesses
    const unsigned blocks = static_cast<unsigned>((work + 127) / 128);
    if (dtype == UCB_BF16)
      ucb::fake_quant_rows_kernel<__nv_bfloat16><<<blocks, 128, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), work, group, max_code);
    else if (dtype == UCB_F16)
      ucb::fake_quant_rows_kernel<__half><<<blocks, 128, 0, s>>>(static_cast<const __half*>(x),
                                                                   static_cast<__half*>(out), work, group, max_code);
    else
      ucb::fake_quant_rows_kernel<float><<<blocks, 128, 0, s>>>(static_cast<const float*>(x),
                                                                  static_cast<float*>(out), work, group, max_code);
    return check_launch("fake_quant_rows_kernel");
  }
  dim3 grid(static_cast<unsigned>((work + 255) / 256));
  switch (dtype) {
    case UCB_BF16:
      ucb::fake_quant_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), outer, length, inner, group, max_code);
      break;
    case UCB_F16:
      ucb::fake_quant_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(out), outer, length, inner, group, max_code);
      break;
    case UCB_F32:
      ucb::fake_quant_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), static_cast<float*>(out), outer, length, inner, group, max_code);
      break;
    default:
      return set_error(UCB_ERR_INVALID, "ucb_fake_quant: dtype %d unsupported", dtype);
  }
  return check_launch("fake_quant_kernel");
}

extern "C" int64_t ucb_kivi_pack_job_bytes(void) { return (int64_t)sizeof(ucb::PackJob); }

extern "C" int ucb_kivi_pack_kv_batched(const void* jobs, int num_jobs, int max_blocks, int64_t heads, int k_bits,
                                        int v_bits, int group_size, void* stream) {
  if (!jobs || num_jobs <= 0 || num_jobs > 65535 || max_blocks <= 0)
    return set_error(UCB_ERR_INVALID, "ucb_kivi_pack_kv_batched: bad job table");
  if (group_size != 32 || heads <= 0)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_kv_batched: group 32 only");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(max_blocks), static_cast<unsigned>(num_jobs));
  const auto* j = static_cast<const ucb::PackJob*>(jobs);
#define UCB_PACK_KVB(KB_, VB_)                                                                       \
  if (k_bits == KB_ && v_bits == VB_) {                                                              \
    ucb::pack_kv_batched_kernel<KB_, VB_, 32><<<grid, 256, 0, s>>>(j, (int)heads);                   \
    return check_launch("pack_kv_batched_kernel");                                                   \
  }
  UCB_PACK_KVB(2, 2) UCB_PACK_KVB(2, 4) UCB_PACK_KVB(2, 8)
  UCB_PACK_KVB(4, 2) UCB_PACK_KVB(4, 4) UCB_PACK_KVB(4, 8)
  UCB_PACK_KVB(8, 2) UCB_PACK_KVB(8, 4) UCB_PACK_KVB(8, 8)
#undef UCB_PACK_KVB
  return set_error(UCB_ERR_UNSUPPORTED, "ucb_kivi_pack_kv_batched: unsupported bits %d/%d", k_bits, v_bits);
}
