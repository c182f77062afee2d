// Per-layer element-wise steps of the configuration-5 decoder
// (unicache_b200.workloads.Qwen2PackedDecode), each one launch instead of a
// chain of framework element-wise kernels:
//  * ucb_rms_norm: RMSNorm of bf16 rows (Qwen2RMSNorm: fp32 statistics, the
//    normalised row rounded to bf16, then times the bf16 weight);
//  * ucb_qkv_rope_append: rotary embedding of the new token's query and key
//    heads at its position (half-split rotation, fp32 arithmetic, one bf16
//    rounding), the query written for the decode kernel and the key and value
//    appended to the dense decode suffix at the row that a device-side length
//    names -- the cache's write path for decode tokens, which the reference
//    appends to its dense cache;
//  * ucb_silu_mul: the SwiGLU gate, silu(gate) rounded to bf16 times up.
// The arithmetic follows the framework expressions the decoder used before
// (each intermediate rounded to bf16 where they round), so eager and captured
// steps see the same values.
#include <algorithm>

#include "common.cuh"

namespace ucb {
namespace {

constexpr int NORM_THREADS = 256;

__global__ void __launch_bounds__(NORM_THREADS) rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ w, int hidden,
                                                                float eps, __nv_bfloat16* __restrict__ out) {
  const __nv_bfloat16* row = x + (int64_t)blockIdx.x * hidden;
  __nv_bfloat16* dst = out + (int64_t)blockIdx.x * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += NORM_THREADS) {
    const float v = __bfloat162float(row[i]);
    ss = fmaf(v, v, ss);
  }
  __shared__ float part[NORM_THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int k = 0; k < NORM_THREADS / 32; ++k) total += part[k];
  const float r = rsqrtf(total / (float)hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += NORM_THREADS) {
    const float t = __bfloat162float(__float2bfloat16(__bfloat162float(row[i]) * r));
    dst[i] = __float2bfloat16(t * __bfloat162float(w[i]));
  }
}

// Block (b, head): head < hq rotates query head `head` into q_out[b, head];
// hq <= head < hq + hkv rotates key head head - hq into the key suffix; the
// last hkv heads copy the value head into the value suffix.  Thread i owns
// channels i and i + half.
__global__ void qkv_rope_append_kernel(const __nv_bfloat16* __restrict__ qkv, int hq, int hkv, int d,
                                       const int32_t* __restrict__ length, int prompt,
                                       const float* __restrict__ inv_freq, __nv_bfloat16* __restrict__ q_out,
                                       __nv_bfloat16* __restrict__ suffix_k, __nv_bfloat16* __restrict__ suffix_v,
                                       int capacity, unsigned int* err) {
  const int b = blockIdx.x, head = blockIdx.y, i = threadIdx.x, half = d / 2;
  const int slot = *length - 1;
  const __nv_bfloat16* src = qkv + ((int64_t)b * (hq + 2 * hkv) + head) * d;
  __nv_bfloat16* dst;
  if (head < hq) {
    dst = q_out + ((int64_t)b * hq + head) * d;
  } else {
    if (slot < 0 || slot >= capacity) {  // the suffix is full: nothing is appended
      if (i == 0) atomicOr(err, DEVERR_BAD_DESCRIPTOR);
      return;
    }
    const int kvh = (head - hq) % hkv;
    __nv_bfloat16* base = head < hq + hkv ? suffix_k : suffix_v;
    dst = base + (((int64_t)b * capacity + slot) * hkv + kvh) * d;
  }
  if (head >= hq + hkv) {  // value: copied as it is
    dst[i] = src[i];
    dst[i + half] = src[i + half];
    return;
  }
  const float angle = (float)(prompt + max(slot, 0)) * inv_freq[i];
  float s, c;
  sincosf(angle, &s, &c);
  const float x1 = __bfloat162float(src[i]), x2 = __bfloat162float(src[i + half]);
  dst[i] = __float2bfloat16(x1 * c - x2 * s);
  dst[i + half] = __float2bfloat16(x2 * c + x1 * s);
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, int rows, int ffn,
                                __nv_bfloat16* __restrict__ out) {
  const int64_t n = (int64_t)rows * ffn;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / ffn, c = e % ffn;
    const float g = __bfloat162float(gate_up[r * 2 * ffn + c]);
    const float u = __bfloat162float(gate_up[r * 2 * ffn + ffn + c]);
    const float act = __bfloat162float(__float2bfloat16(g / (1.f + expf(-g))));
    out[e] = __float2bfloat16(act * u);
  }
}

}  // namespace
}  // namespace ucb

using ucb_host::set_error;

extern "C" int ucb_rms_norm(const void* x, const void* weight, int rows, int hidden, float eps, void* out,
                            void* stream) {
  if (!x || !weight || !out) return set_error(UCB_ERR_INVALID, "ucb_rms_norm: null pointer");
  if (rows <= 0 || hidden <= 0) return set_error(UCB_ERR_INVALID, "ucb_rms_norm: empty input");
  ucb::rms_norm_kernel<<<rows, ucb::NORM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight), hidden, eps,
      static_cast<__nv_bfloat16*>(out));
  return ucb_host::check_launch("rms_norm_kernel");
}

extern "C" int ucb_qkv_rope_append(const void* qkv, int batch, int hq, int hkv, int head_dim, const int32_t* length,
                                   int prompt, const float* inv_freq, void* q_out, void* suffix_k, void* suffix_v,
                                   int capacity, void* stream) {
  if (!qkv || !length || !inv_freq || !q_out || !suffix_k || !suffix_v)
    return set_error(UCB_ERR_INVALID, "ucb_qkv_rope_append: null pointer");
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv || capacity <= 0)
    return set_error(UCB_ERR_INVALID, "ucb_qkv_rope_append: bad shape");
  if (head_dim <= 0 || head_dim % 2 || head_dim > 2048)
    return set_error(UCB_ERR_INVALID, "ucb_qkv_rope_append: head_dim must be even and at most 2048");
  unsigned int* err = ucb_host::device_error_word();
  if (!err) return set_error(UCB_ERR_CUDA, "ucb_qkv_rope_append: device error word unavailable");
  const dim3 grid(batch, hq + 2 * hkv);
  ucb::qkv_rope_append_kernel<<<grid, head_dim / 2, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), hq, hkv, head_dim, length, prompt, inv_freq,
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(suffix_k), static_cast<__nv_bfloat16*>(suffix_v),
      capacity, err);
  return ucb_host::check_launch("qkv_rope_append_kernel");
}

extern "C" int ucb_silu_mul(const void* gate_up, int rows, int ffn, void* out, void* stream) {
  if (!gate_up || !out) return set_error(UCB_ERR_INVALID, "ucb_silu_mul: null pointer");
  if (rows <= 0 || ffn <= 0) return set_error(UCB_ERR_INVALID, "ucb_silu_mul: empty input");
  const int64_t n = (int64_t)rows * ffn;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  ucb::silu_mul_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate_up), rows, ffn, static_cast<__nv_bfloat16*>(out));
  return ucb_host::check_launch("silu_mul_kernel");
}
