// The packed cache's generic attention parts (materialised logits and the
// probability x value product), replacing packed_kivi_attention_parts of the
// reference (unicache/storage/kivi_cuda.py:238-329; the CPU layout computes
// the same from dequantize(), unicache/storage/physical.py:452-475):
//
//   logits[h, i, t] = q[i, h, :] . k_hat[t, kv(h), :] / sqrt(D)        (fp32)
//   out[h, i, :]    = sum_t p[h, i, t] v_hat[t, kv(h), :]               (bf16)
//
// over the segment's quantized tokens followed by its residual rows.  Used
// where an operator needs the probabilities themselves (the fused decode and
// long-query kernels never call it).
//
// Design: a CTA takes 64 query rows (4 warps x 16) of one KV head and walks
// the tokens in tiles of 16.  Per tile the CTA restores k_hat (or v_hat) into
// a shared-memory tile exactly as the reference's dequantize() does (code *
// scale + minimum in fp32, one rounding to bf16; residual rows copied), then
// every warp runs mma.sync m16n8k16 bf16 against it (ldmatrix for keys,
// ldmatrix.trans for values), accumulating in fp32.
#include "common.cuh"

namespace ucb {
namespace parts {

constexpr int D = 128;
constexpr int TT = 16;            // tokens per tile
constexpr int ROWB = 272;         // shared-memory row stride (bytes): 256 + 16, conflict-free ldmatrix
constexpr int ROWS_PER_CTA = 64;  // 4 warps x 16 query rows

struct Segment {
  const void* codes;        // this head: K [T/f, D] int32 words (uint8 [T, D] at 8 bits); V [T, D/f] (uint8 [T, D])
  const uint16_t* scale;    // bf16 statistics: K [T/G, D], V [T, D/G]
  const uint16_t* minimum;
  int64_t codes_head, stats_head;  // element strides between KV heads
  const __nv_bfloat16* residual;   // [R, H, D] rows, strides below
  int64_t res_token, res_head;
  int quantized, residual_rows, bits, group;
};

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Restore tokens [t0, t0 + 16) of one KV head into tile[16][128] (bf16, row
// stride ROWB): thread = (token t0 + tid / 8, 16 channels (tid % 8) * 16).
template <bool KEYS>
__device__ void fill_tile(const Segment& s, int kv, int t0, unsigned char* tile) {
  const int tid = threadIdx.x, lt = tid >> 3, c0 = (tid & 7) * 16, t = t0 + lt;
  uint32_t out[8];
  if (t < s.quantized) {
    float v[16];
    if (KEYS) {
      const int g = t / s.group;
      const uint16_t* sc = s.scale + kv * s.stats_head + (int64_t)g * D + c0;
      const uint16_t* mn = s.minimum + kv * s.stats_head + (int64_t)g * D + c0;
      if (s.bits == 8) {
        const uint8_t* cw = static_cast<const uint8_t*>(s.codes) + kv * s.codes_head + (int64_t)t * D + c0;
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = fmaf((float)cw[k], bf16f(sc[k]), bf16f(mn[k]));
      } else {
        const int f = 32 / s.bits, shift = s.bits * (t % f);
        const uint32_t mask = (1u << s.bits) - 1u;
        const uint32_t* cw = static_cast<const uint32_t*>(s.codes) + kv * s.codes_head + (int64_t)(t / f) * D + c0;
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = fmaf((float)((cw[k] >> shift) & mask), bf16f(sc[k]), bf16f(mn[k]));
      }
    } else {
      const int ng = D / s.group;
      const int64_t so = kv * s.stats_head + (int64_t)t * ng + c0 / s.group;  // 16 channels share a group (G >= 32)
      const float sg = bf16f(s.scale[so]), mg = bf16f(s.minimum[so]);
      if (s.bits == 8) {
        const uint8_t* cw = static_cast<const uint8_t*>(s.codes) + kv * s.codes_head + (int64_t)t * D + c0;
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = fmaf((float)cw[k], sg, mg);
      } else {
        const int f = 32 / s.bits;
        const uint32_t mask = (1u << s.bits) - 1u;
        const uint32_t* cw = static_cast<const uint32_t*>(s.codes) + kv * s.codes_head + (int64_t)t * (D / f);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int ch = c0 + k;
          v[k] = fmaf((float)((cw[ch / f] >> (s.bits * (ch % f))) & mask), sg, mg);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = pack_bf16x2(v[2 * k], v[2 * k + 1]);
  } else if (t < s.quantized + s.residual_rows) {
    const uint4* src = reinterpret_cast<const uint4*>(s.residual + (int64_t)(t - s.quantized) * s.res_token +
                                                      kv * s.res_head + c0);
    const uint4 a = src[0], b = src[1];
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = 0u;
  }
  uint4* dst = reinterpret_cast<uint4*>(tile + lt * ROWB + c0 * 2);
  dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
  dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
}

// logits[(kv*grp + g) * Lq + i][t] for row r = g * Lq + i of KV head kv.
__global__ void __launch_bounds__(128) logits_kernel(Segment s, const __nv_bfloat16* __restrict__ query, int lq,
                                                     int hq, int grp, float scale, float* __restrict__ logits) {
  __shared__ __align__(16) unsigned char tile[TT * ROWB];
  const int kv = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, lr = lane >> 2, lc = lane & 3;
  const int rows = grp * lq, n_tok = s.quantized + s.residual_rows;
  const int r0 = blockIdx.x * ROWS_PER_CTA + warp * 16 + lr, r1 = r0 + 8;
  uint32_t a[8][4];
  auto qrow = [&](int r) -> const __nv_bfloat16* {
    return query + ((int64_t)(r % lq) * hq + kv * grp + r / lq) * D;
  };
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int ch = 16 * kk + 2 * lc;
    a[kk][0] = r0 < rows ? *reinterpret_cast<const uint32_t*>(qrow(r0) + ch) : 0u;
    a[kk][1] = r1 < rows ? *reinterpret_cast<const uint32_t*>(qrow(r1) + ch) : 0u;
    a[kk][2] = r0 < rows ? *reinterpret_cast<const uint32_t*>(qrow(r0) + ch + 8) : 0u;
    a[kk][3] = r1 < rows ? *reinterpret_cast<const uint32_t*>(qrow(r1) + ch + 8) : 0u;
  }
  const uint32_t tbase = smem_u32(tile);
  const int mi = lane >> 3;  // ldmatrix matrix this lane addresses: tokens (mi >> 1) * 8 + lane % 8, channel half mi & 1
  const uint32_t laddr = tbase + ((mi >> 1) * 8 + (lane & 7)) * ROWB + (mi & 1) * 16;
  float* out0 = logits + ((int64_t)kv * grp * lq + r0) * n_tok;
  float* out1 = logits + ((int64_t)kv * grp * lq + r1) * n_tok;
  for (int t0 = 0; t0 < n_tok; t0 += TT) {
    __syncthreads();
    fill_tile<true>(s, kv, t0, tile);
    __syncthreads();
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t b[4];
      ldmatrix_x4(b, laddr + kk * 32);
      mma_bf16(acc[0], a[kk], b[0], b[1]);
      mma_bf16(acc[1], a[kk], b[2], b[3]);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = t0 + 8 * j + 2 * lc;
      if (r0 < rows) {
        if (t < n_tok) out0[t] = acc[j][0] * scale;
        if (t + 1 < n_tok) out0[t + 1] = acc[j][1] * scale;
      }
      if (r1 < rows) {
        if (t < n_tok) out1[t] = acc[j][2] * scale;
        if (t + 1 < n_tok) out1[t + 1] = acc[j][3] * scale;
      }
    }
  }
}

template <typename P>
__device__ __forceinline__ float prob(const P* p, int t, int n) {
  return t < n ? Dtype<P>::to_f(p[t]) : 0.f;
}

// out[(kv*grp + g) * Lq + i][:] = sum_t probs[...][t] v_hat[t] (probabilities
// rounded to bf16 first, as the reference casts them to the value dtype).
template <typename P>
__global__ void __launch_bounds__(128) apply_kernel(Segment s, const P* __restrict__ probs, int lq, int grp,
                                                    __nv_bfloat16* __restrict__ out) {
  __shared__ __align__(16) unsigned char tile[TT * ROWB];
  const int kv = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, lr = lane >> 2, lc = lane & 3;
  const int rows = grp * lq, n_tok = s.quantized + s.residual_rows;
  const int r0 = blockIdx.x * ROWS_PER_CTA + warp * 16 + lr, r1 = r0 + 8;
  const P* p0 = probs + ((int64_t)kv * grp * lq + min(r0, rows - 1)) * n_tok;
  const P* p1 = probs + ((int64_t)kv * grp * lq + min(r1, rows - 1)) * n_tok;
  float acc[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const uint32_t tbase = smem_u32(tile);
  const int mi = lane >> 3;  // ldmatrix.trans: tokens (mi & 1) * 8 + lane % 8, channel block mi >> 1
  const uint32_t laddr = tbase + ((mi & 1) * 8 + (lane & 7)) * ROWB + (mi >> 1) * 16;
  for (int t0 = 0; t0 < n_tok; t0 += TT) {
    __syncthreads();
    fill_tile<false>(s, kv, t0, tile);
    __syncthreads();
    const int t = t0 + 2 * lc;
    uint32_t a[4];
    a[0] = r0 < rows ? pack_bf16x2(prob(p0, t, n_tok), prob(p0, t + 1, n_tok)) : 0u;
    a[1] = r1 < rows ? pack_bf16x2(prob(p1, t, n_tok), prob(p1, t + 1, n_tok)) : 0u;
    a[2] = r0 < rows ? pack_bf16x2(prob(p0, t + 8, n_tok), prob(p0, t + 9, n_tok)) : 0u;
    a[3] = r1 < rows ? pack_bf16x2(prob(p1, t + 8, n_tok), prob(p1, t + 9, n_tok)) : 0u;
#pragma unroll
    for (int n = 0; n < 16; n += 2) {
      uint32_t b[4];
      ldmatrix_x4_trans(b, laddr + n * 16);
      mma_bf16(acc[n], a, b[0], b[1]);
      mma_bf16(acc[n + 1], a, b[2], b[3]);
    }
  }
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int ch = 8 * n + 2 * lc;
    if (r0 < rows)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)kv * grp * lq + r0) * D + ch) = pack_bf16x2(acc[n][0], acc[n][1]);
    if (r1 < rows)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)kv * grp * lq + r1) * D + ch) = pack_bf16x2(acc[n][2], acc[n][3]);
  }
}

}  // namespace parts
}  // namespace ucb

using ucb_host::check_launch;
using ucb_host::set_error;

namespace {
int make_segment(ucb::parts::Segment* s, const void* codes, const void* scale, const void* minimum,
                 int64_t codes_head, int64_t stats_head, const void* residual, int64_t res_token, int64_t res_head,
                 int64_t quantized, int64_t residual_rows, int bits, int group, const char* what) {
  if (quantized < 0 || residual_rows < 0 || quantized + residual_rows <= 0 || quantized + residual_rows > (1 << 30))
    return set_error(UCB_ERR_INVALID, "%s: bad token counts", what);
  if (quantized && (!codes || !scale || !minimum)) return set_error(UCB_ERR_INVALID, "%s: null packed tensor", what);
  if (residual_rows && !residual) return set_error(UCB_ERR_INVALID, "%s: null residual", what);
  if (bits != 2 && bits != 4 && bits != 8) return set_error(UCB_ERR_UNSUPPORTED, "%s: bits must be 2, 4 or 8", what);
  if (group != 32 && group != 64 && group != 128)
    return set_error(UCB_ERR_UNSUPPORTED, "%s: group_size must be 32, 64 or 128", what);
  if (residual_rows && ((reinterpret_cast<uintptr_t>(residual) & 15) || (res_token & 7) || (res_head & 7)))
    return set_error(UCB_ERR_INVALID, "%s: residual rows must be 16-byte aligned", what);
  s->codes = codes;
  s->scale = static_cast<const uint16_t*>(scale);
  s->minimum = static_cast<const uint16_t*>(minimum);
  s->codes_head = codes_head;
  s->stats_head = stats_head;
  s->residual = static_cast<const __nv_bfloat16*>(residual);
  s->res_token = res_token;
  s->res_head = res_head;
  s->quantized = (int)quantized;
  s->residual_rows = (int)residual_rows;
  s->bits = bits;
  s->group = group;
  return UCB_OK;
}
}  // namespace

extern "C" int ucb_kivi_attention_logits(const void* query, int64_t queries, int q_heads, int kv_heads,
                                         const void* key_code, const void* key_scale, const void* key_minimum,
                                         int64_t codes_head_stride, int64_t stats_head_stride,
                                         const void* residual_key, int64_t res_token_stride, int64_t res_head_stride,
                                         int64_t quantized_tokens, int64_t residual_tokens, int bits, int group_size,
                                         float softmax_scale, float* logits, void* stream) {
  const char* what = "ucb_kivi_attention_logits";
  if (!query || !logits) return set_error(UCB_ERR_INVALID, "%s: null pointer", what);
  if (queries <= 0 || kv_heads <= 0 || q_heads % kv_heads) return set_error(UCB_ERR_INVALID, "%s: bad shape", what);
  if ((int64_t)queries * (q_heads / kv_heads) > (1 << 30)) return set_error(UCB_ERR_INVALID, "%s: too many rows", what);
  ucb::parts::Segment s;
  int rc = make_segment(&s, key_code, key_scale, key_minimum, codes_head_stride, stats_head_stride, residual_key,
                        res_token_stride, res_head_stride, quantized_tokens, residual_tokens, bits, group_size, what);
  if (rc) return rc;
  const int grp = q_heads / kv_heads, rows = (int)queries * grp;
  dim3 grid((rows + ucb::parts::ROWS_PER_CTA - 1) / ucb::parts::ROWS_PER_CTA, kv_heads);
  ucb::parts::logits_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      s, static_cast<const __nv_bfloat16*>(query), (int)queries, q_heads, grp, softmax_scale, logits);
  return check_launch("logits_kernel");
}

extern "C" int ucb_kivi_attention_apply(const void* probs, int probs_dtype, int64_t queries, int q_heads,
                                        int kv_heads, const void* value_code, const void* value_scale,
                                        const void* value_minimum, int64_t codes_head_stride,
                                        int64_t stats_head_stride, const void* residual_value,
                                        int64_t res_token_stride, int64_t res_head_stride, int64_t quantized_tokens,
                                        int64_t residual_tokens, int bits, int group_size, void* out, void* stream) {
  const char* what = "ucb_kivi_attention_apply";
  if (!probs || !out) return set_error(UCB_ERR_INVALID, "%s: null pointer", what);
  if (queries <= 0 || kv_heads <= 0 || q_heads % kv_heads) return set_error(UCB_ERR_INVALID, "%s: bad shape", what);
  if ((int64_t)queries * (q_heads / kv_heads) > (1 << 30)) return set_error(UCB_ERR_INVALID, "%s: too many rows", what);
  ucb::parts::Segment s;
  int rc = make_segment(&s, value_code, value_scale, value_minimum, codes_head_stride, stats_head_stride,
                        residual_value, res_token_stride, res_head_stride, quantized_tokens, residual_tokens, bits,
                        group_size, what);
  if (rc) return rc;
  const int grp = q_heads / kv_heads, rows = (int)queries * grp;
  dim3 grid((rows + ucb::parts::ROWS_PER_CTA - 1) / ucb::parts::ROWS_PER_CTA, kv_heads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* o = static_cast<__nv_bfloat16*>(out);
  switch (probs_dtype) {
    case UCB_BF16:
      ucb::parts::apply_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(s, static_cast<const __nv_bfloat16*>(probs),
                                                                    (int)queries, grp, o);
      break;
    case UCB_F16:
      ucb::parts::apply_kernel<__half><<<grid, 128, 0, st>>>(s, static_cast<const __half*>(probs), (int)queries, grp,
                                                             o);
      break;
    case UCB_F32:
      ucb::parts::apply_kernel<float><<<grid, 128, 0, st>>>(s, static_cast<const float*>(probs), (int)queries, grp,
                                                            o);
      break;
    default:
      return set_error(UCB_ERR_UNSUPPORTED, "%s: probabilities must be bf16, f16 or f32", what);
  }
  return check_launch("apply_kernel");
}
