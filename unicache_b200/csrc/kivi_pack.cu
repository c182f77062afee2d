// KIVI grouped quantization, bit-packing, dequantization and fake quantization.
//
// Arithmetic contract (bit-exact with unicache/storage/physical.py:139-201 and
// unicache/operators/builtin.py:31-53): every step is one IEEE fp32 operation
// with round-to-nearest (explicit __fsub_rn/__fdiv_rn/__fmul_rn/__fadd_rn, so
// the compiler cannot contract them into FMAs), rounding to integers is
// round-half-even (rintf), and stores into bf16/fp16 round to nearest even.
// This translation unit must not be compiled with fast-math.
#include <cfloat>

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

// ---------------------------------------------------------------- key pack
// One CTA per (token group, head); one thread per channel.  Groups run along
// tokens, so a thread reduces a column of `group` values and emits
// group*bits/32 words for its channel.
template <typename T, int BITS>
__global__ void __launch_bounds__(128) pack_key_kernel(const T* __restrict__ x, int64_t stride_t,
                                                       int64_t stride_h, int tokens, int head_dim,
                                                       int group, uint32_t* __restrict__ codes32,
                                                       uint8_t* __restrict__ codes8,
                                                       T* __restrict__ scale, T* __restrict__ minimum) {
  const int g = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  if (d >= head_dim) return;
  const int groups = tokens / group;
  const T* col = x + static_cast<int64_t>(g) * group * stride_t + h * stride_h + d;
  float mn = INFINITY, mx = -INFINITY;
  for (int i = 0; i < group; ++i) {
    const float v = ld(col + i * stride_t);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  const float sc = quant_scale(mn, mx, kMax);
  const int64_t stat = (static_cast<int64_t>(h) * groups + g) * head_dim + d;
  scale[stat] = Dtype<T>::from_f(sc);
  minimum[stat] = Dtype<T>::from_f(mn);
  if constexpr (BITS == 8) {
    uint8_t* out = codes8 + (static_cast<int64_t>(h) * tokens + static_cast<int64_t>(g) * group) * head_dim + d;
    for (int i = 0; i < group; ++i) {
      out[static_cast<int64_t>(i) * head_dim] =
          static_cast<uint8_t>(quant_code(ld(col + i * stride_t), mn, sc, kMax));
    }
  } else {
    constexpr int F = 32 / BITS;
    const int words = group / F;
    uint32_t* out = codes32 + (static_cast<int64_t>(h) * (tokens / F) + static_cast<int64_t>(g) * words) * head_dim + d;
    for (int w = 0; w < words; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < F; ++j) {
        word |= quant_code(ld(col + (w * F + j) * stride_t), mn, sc, kMax) << (j * BITS);
      }
      out[static_cast<int64_t>(w) * head_dim] = word;
    }
  }
}

// ---------------------------------------------------------------- value pack
// One warp per (token, head) row of D channels; lane l holds VPL = D/32
// consecutive channels.  A group of G channels spans G/VPL lanes.
template <typename T, int BITS, int D, int G>
__global__ void __launch_bounds__(256) pack_value_kernel(const T* __restrict__ x, int64_t stride_t,
                                                         int64_t stride_h, int tokens, int heads,
                                                         uint32_t* __restrict__ codes32,
                                                         uint8_t* __restrict__ codes8,
                                                         T* __restrict__ scale, T* __restrict__ minimum) {
  constexpr int VPL = D / 32;
  constexpr int LPG = G / VPL;  // lanes per group
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(tokens) * heads) return;
  const int t = static_cast<int>(row / heads), h = static_cast<int>(row % heads);
  const T* src = x + t * stride_t + h * stride_h + lane * VPL;
  float v[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) v[j] = ld(src + j);
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int j = 1; j < VPL; ++j) {
    mn = fminf(mn, v[j]);
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int off = 1; off < LPG; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  constexpr float kMax = static_cast<float>((1 << BITS) - 1);
  const float sc = quant_scale(mn, mx, kMax);
  const int64_t out_row = static_cast<int64_t>(h) * tokens + t;
  if (lane % LPG == 0) {
    const int gd = lane / LPG;
    scale[out_row * (D / G) + gd] = Dtype<T>::from_f(sc);
    minimum[out_row * (D / G) + gd] = Dtype<T>::from_f(mn);
  }
  uint32_t code[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) code[j] = quant_code(v[j], mn, sc, kMax);
  if constexpr (BITS == 8) {
    uint8_t* out = codes8 + out_row * D + lane * VPL;
#pragma unroll
    for (int j = 0; j < VPL; ++j) out[j] = static_cast<uint8_t>(code[j]);
  } else {
    constexpr int F = 32 / BITS;
    constexpr int LPW = F / VPL;  // lanes per word
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) word |= code[j] << (((lane * VPL + j) % F) * BITS);
#pragma unroll
    for (int off = 1; off < LPW; off <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, off);
    if (lane % LPW == 0) codes32[out_row * (D / F) + lane / LPW] = word;
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
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t l = start; l < stop; ++l) {
    const float v = ld(x + base + l * inner);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  // builtin.py:50 clamps the range before dividing (unlike the packed quantizer).
  const float sc = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), FLT_EPSILON), max_code);
  for (int64_t l = start; l < stop; ++l) {
    const float v = ld(x + base + l * inner);
    const float q = static_cast<float>(quant_code(v, mn, sc, max_code));
    out[base + l * inner] = Dtype<T>::from_f(__fadd_rn(__fmul_rn(q, sc), mn));
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
  if (bits == 2)
    ucb::pack_key_kernel<T, 2><<<grid, 128, 0, s>>>(xp, st, sh, (int)T_, (int)D, group, c32, c8, sp, mp);
  else if (bits == 4)
    ucb::pack_key_kernel<T, 4><<<grid, 128, 0, s>>>(xp, st, sh, (int)T_, (int)D, group, c32, c8, sp, mp);
  else
    ucb::pack_key_kernel<T, 8><<<grid, 128, 0, s>>>(xp, st, sh, (int)T_, (int)D, group, c32, c8, sp, mp);
  return check_launch("pack_key_kernel");
}

template <typename T, int BITS, int D>
int launch_pack_value_g(const void* x, int64_t T_, int64_t H, int64_t st, int64_t sh, int group, void* codes,
                        void* scale, void* minimum, cudaStream_t s) {
  const int64_t rows = T_ * H;
  dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  const T* xp = static_cast<const T*>(x);
  auto* c32 = static_cast<uint32_t*>(codes);
  auto* c8 = static_cast<uint8_t*>(codes);
  T* sp = static_cast<T*>(scale);
  T* mp = static_cast<T*>(minimum);
  if (group == 32)
    ucb::pack_value_kernel<T, BITS, D, 32><<<grid, 256, 0, s>>>(xp, st, sh, (int)T_, (int)H, c32, c8, sp, mp);
  else if (group == 64)
    ucb::pack_value_kernel<T, BITS, D, 64><<<grid, 256, 0, s>>>(xp, st, sh, (int)T_, (int)H, c32, c8, sp, mp);
  else
    ucb::pack_value_kernel<T, BITS, D, 128><<<grid, 256, 0, s>>>(xp, st, sh, (int)T_, (int)H, c32, c8, sp, mp);
  return check_launch("pack_value_kernel");
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
