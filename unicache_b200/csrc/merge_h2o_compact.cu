// LSE merge of attention summaries, H2O scoring / selection / gathering and
// dense-cache row compaction.
#include <cfloat>

#include "common.cuh"

using ucb_host::check_launch;
using ucb_host::set_error;

namespace ucb {
namespace {

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return Dtype<T>::to_f(*p);
}

// ---------------------------------------------------------------- LSE merge
// unicache/adapters/bagel.py:57-72: total = logsumexp_i(lse_i);
// out = sum_i o_i * exp(lse_i - total).  One CTA per (head, row).
constexpr int kMaxMerge = 64;
struct MergeArgs {
  const void* o[kMaxMerge];
  const float* lse[kMaxMerge];
};

template <typename T>
__global__ void lse_merge_kernel(MergeArgs args, int n, int64_t rows, int64_t heads, int64_t head_dim, T* out,
                                 float* lse_out) {
  const int64_t row = blockIdx.x % rows;
  const int64_t h = blockIdx.x / rows;
  __shared__ float w[kMaxMerge];
  __shared__ float total_s;
  if (threadIdx.x == 0) {
    float peak = -INFINITY;
    for (int i = 0; i < n; ++i) peak = fmaxf(peak, args.lse[i][h * rows + row]);
    float sum = 0.f;
    if (peak != -INFINITY) {
      for (int i = 0; i < n; ++i) sum += expf(args.lse[i][h * rows + row] - peak);
    }
    const float total = (peak == -INFINITY) ? -INFINITY : peak + logf(sum);
    for (int i = 0; i < n; ++i) w[i] = expf(args.lse[i][h * rows + row] - total);
    total_s = total;
    if (lse_out) lse_out[h * rows + row] = total;
  }
  __syncthreads();
  for (int64_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < n; ++i) {
      const T* o = static_cast<const T*>(args.o[i]);
      acc += ldf(o + (row * heads + h) * head_dim + d) * w[i];
    }
    out[(row * heads + h) * head_dim + d] = Dtype<T>::from_f(acc);
  }
}

// ---------------------------------------------------------------- block scan helper
template <int THREADS>
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) smem_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = (lane < THREADS / 32) ? smem_warp[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += y;
    }
    if (lane < THREADS / 32) smem_warp[lane] = s;
  }
  __syncthreads();
  const int warp_prefix = warp ? smem_warp[warp - 1] : 0;
  total = smem_warp[THREADS / 32 - 1];
  __syncthreads();
  return warp_prefix + x - v;
}

// ---------------------------------------------------------------- H2O select
// Order-preserving key: larger score -> larger unsigned key.
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kSelThreads = 1024;

// One CTA per KV head: radix-select the heavy_k-th largest key of the history
// (4 passes of 8 bits), then emit, in ascending index order, every index whose
// key is larger plus the lowest-index entries equal to it.
__global__ void __launch_bounds__(kSelThreads) h2o_select_kernel(const float* __restrict__ scores,
                                                                 int64_t stride, int64_t tokens,
                                                                 int64_t history_end, int64_t heavy_k,
                                                                 int64_t recent, int64_t* __restrict__ out) {
  const int h = blockIdx.x, tid = threadIdx.x;
  const float* row = scores + h * stride;
  int64_t* orow = out + h * (heavy_k + recent);
  __shared__ unsigned int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int64_t s_krem;
  __shared__ int scan_smem[32];
  if (heavy_k > 0) {
    uint32_t prefix = 0, mask = 0;
    int64_t krem = heavy_k;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
      __syncthreads();
      for (int64_t i = tid; i < history_end; i += kSelThreads) {
        const uint32_t key = score_key(row[i]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int64_t cum = 0;
        int sel = 0;
        for (int b = 255; b >= 0; --b) {
          if (cum + hist[b] >= krem) {
            sel = b;
            break;
          }
          cum += hist[b];
        }
        s_prefix = prefix | (static_cast<uint32_t>(sel) << shift);
        s_krem = krem - cum;
      }
      __syncthreads();
      prefix = s_prefix;
      krem = s_krem;
      mask |= 255u << shift;
      __syncthreads();
    }
    const uint32_t thr = prefix;
    const int64_t need_eq = krem;  // entries equal to thr to keep (lowest indices)
    int64_t eq_carry = 0, out_carry = 0;
    for (int64_t base = 0; base < history_end; base += kSelThreads) {
      const int64_t i = base + tid;
      uint32_t key = 0;
      const bool in = i < history_end;
      if (in) key = score_key(row[i]);
      const int is_eq = (in && key == thr) ? 1 : 0;
      int eq_total;
      const int eq_rank = block_exclusive_scan<kSelThreads>(is_eq, scan_smem, eq_total);
      const int take = (in && (key > thr || (is_eq && eq_carry + eq_rank < need_eq))) ? 1 : 0;
      int take_total;
      const int pos = block_exclusive_scan<kSelThreads>(take, scan_smem, take_total);
      if (take) orow[out_carry + pos] = i;
      eq_carry += eq_total;
      out_carry += take_total;
    }
  }
  for (int64_t i = tid; i < recent; i += kSelThreads) orow[heavy_k + i] = tokens - recent + i;
}

// ---------------------------------------------------------------- gather
template <typename V>
__global__ void gather_rows_kernel(const unsigned char* __restrict__ src, int64_t stride_h_bytes,
                                   int64_t stride_t_bytes, int64_t row_vecs, const int64_t* __restrict__ index,
                                   int64_t keep, unsigned char* __restrict__ dst) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
  const int h = blockIdx.y;
  if (r >= keep) return;
  const int64_t idx = index[h * keep + r];
  const V* s = reinterpret_cast<const V*>(src + h * stride_h_bytes + idx * stride_t_bytes);
  V* d = reinterpret_cast<V*>(dst + ((int64_t)h * keep + r) * row_vecs * (int64_t)sizeof(V));
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) d[v] = s[v];
}

// ---------------------------------------------------------------- score accumulation
template <typename T>
__global__ void accumulate_probs_kernel(const T* __restrict__ probs, int grp, int64_t queries, int64_t tokens,
                                        int kv_heads, float* __restrict__ scores, int accumulate) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int kv = blockIdx.y;
  if (t >= tokens) return;
  float total = 0.f;
  for (int g = 0; g < grp; ++g) {
    const T* p = probs + ((int64_t)(kv * grp + g) * queries) * tokens + t;
    float s = 0.f;
    for (int64_t q = 0; q < queries; ++q) s += ldf(p + q * tokens);
    total += s;
  }
  float* o = scores + (int64_t)kv * tokens + t;
  *o = accumulate ? *o + total : total;
}

// ---------------------------------------------------------------- H2O scoring
// Received attention per KV head without materialised probabilities
// (operators/physical.py:63-65 sums softmax probabilities over queries and
// the heads of a GQA group): scores[kv, t] (+)= sum over the kv head's rows
// (query head h = kv*grp + g, query i) of exp(scale * q_{i,h} . k_t - lse_{h,i}),
// with lse the natural-log normaliser of each row over ALL keys of the
// attention (the attention kernels return it), so the terms are exactly the
// probabilities the reference reduces.

// bf16 keys and queries on the tensor cores (mma.sync m16n8k16, fp32
// accumulate: bf16 products are exact).  A CTA of 4 warps takes 128 tokens of
// one KV head (each warp 2 tiles of 16 tokens, A fragments held in registers
// for the whole launch) and streams the head's query rows through shared
// memory in chunks of 64; every 8 rows are one MMA column block.
constexpr int kScoreRows = 64;    // query rows per shared-memory chunk
constexpr int kScoreRowB = 272;   // row stride (bytes): 256 + 16, conflict-free ldmatrix
__global__ void __launch_bounds__(128) scores_mma_kernel(const __nv_bfloat16* __restrict__ query, int64_t queries,
                                                         int q_heads, const __nv_bfloat16* __restrict__ key,
                                                         int64_t ks_t, int64_t ks_h, int64_t tokens, int grp,
                                                         const float* __restrict__ lse, float scale_log2,
                                                         float* __restrict__ scores, int accumulate) {
  constexpr int D = 128;
  constexpr float LOG2E_F = 1.4426950408889634f;
  __shared__ __align__(16) unsigned char qs[kScoreRows * kScoreRowB];
  __shared__ float ls[kScoreRows];
  const int kv = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int64_t tok_base = (int64_t)blockIdx.x * 128 + warp * 32;
  // A fragments: lane holds tokens (r, r+8) of each 16-token tile, channels
  // 16kk + {2c, 2c+1, 2c+8, 2c+9}.
  uint32_t a[2][8][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const int64_t t0 = tok_base + 16 * mt + r, t1 = t0 + 8;
    const __nv_bfloat16* k0 = key + t0 * ks_t + (int64_t)kv * ks_h;
    const __nv_bfloat16* k1 = key + t1 * ks_t + (int64_t)kv * ks_h;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int ch = 16 * kk + 2 * c;
      a[mt][kk][0] = t0 < tokens ? *reinterpret_cast<const uint32_t*>(k0 + ch) : 0u;
      a[mt][kk][1] = t1 < tokens ? *reinterpret_cast<const uint32_t*>(k1 + ch) : 0u;
      a[mt][kk][2] = t0 < tokens ? *reinterpret_cast<const uint32_t*>(k0 + ch + 8) : 0u;
      a[mt][kk][3] = t1 < tokens ? *reinterpret_cast<const uint32_t*>(k1 + ch + 8) : 0u;
    }
  }
  float sum[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [tile][token r / r+8], this lane's columns
  const int64_t rows = (int64_t)grp * queries;
  const uint32_t qbase = smem_u32(qs);
  // ldmatrix x4 row addresses: matrix m = lane / 8 covers channels 8m..8m+7 of
  // a 32-channel block (two k-chunks), row = query row (lane % 8).
  const uint32_t lm_off = (lane & 7) * kScoreRowB + (lane >> 3) * 16;
  for (int64_t base = 0; base < rows; base += kScoreRows) {
    __syncthreads();
    for (int i = threadIdx.x; i < kScoreRows * (D / 8); i += blockDim.x) {
      const int rr = i / (D / 8), chunk = i % (D / 8);
      const int64_t row = base + rr;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < rows) {
        const int g = (int)(row / queries);
        const int64_t qi = row % queries;
        v = reinterpret_cast<const uint4*>(query + (qi * q_heads + kv * grp + g) * D)[chunk];
      }
      *reinterpret_cast<uint4*>(qs + rr * kScoreRowB + chunk * 16) = v;
    }
    for (int i = threadIdx.x; i < kScoreRows; i += blockDim.x) {
      const int64_t row = base + i;
      ls[i] = row < rows ? lse[(int64_t)(kv * grp + row / queries) * queries + row % queries] * LOG2E_F : INFINITY;
    }
    __syncthreads();
#pragma unroll 1
    for (int nb = 0; nb < kScoreRows / 8; ++nb) {
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {  // pairs of k-chunks
        uint32_t b[4];
        ldmatrix_x4(b, qbase + nb * 8 * kScoreRowB + kp * 64 + lm_off);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          mma_bf16(acc[mt], a[mt][2 * kp], b[0], b[1]);
          mma_bf16(acc[mt], a[mt][2 * kp + 1], b[2], b[3]);
        }
      }
      const float l0 = ls[nb * 8 + 2 * c], l1 = ls[nb * 8 + 2 * c + 1];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        sum[mt][0] += fast_exp2(fmaf(acc[mt][0], scale_log2, -l0)) + fast_exp2(fmaf(acc[mt][1], scale_log2, -l1));
        sum[mt][1] += fast_exp2(fmaf(acc[mt][2], scale_log2, -l0)) + fast_exp2(fmaf(acc[mt][3], scale_log2, -l1));
      }
    }
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v = sum[mt][h];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      const int64_t t = tok_base + 16 * mt + r + 8 * h;
      if (c == 0 && t < tokens) {
        float* o = scores + (int64_t)kv * tokens + t;
        *o = accumulate ? *o + v : v;
      }
    }
  }
}

// fp32 (or any dtype) on the CUDA cores, for fp32 caches.  Block (x, kv):
// 64 tokens of KV head kv x 4 row groups (256 threads); a thread holds its
// token's key row and takes every fourth query row of each 32-row chunk
// staged in shared memory, four rows per pass (four independent FMA chains);
// the four groups' sums of a token are added in group order, so the result
// does not depend on scheduling.  Row offsets of a chunk are formed once per
// row (one division), not per staged element.
constexpr int kScoreQ = 32;  // query rows staged per round (a multiple of 16)
constexpr int kScoreTok = 64, kScoreGroups = 4;
static_assert(kScoreQ % (4 * kScoreGroups) == 0, "each group takes four rows per pass");

template <typename T>
__device__ __forceinline__ void stage_rows(const T* __restrict__ query, int64_t queries, int q_heads, int kv,
                                           int grp, int64_t rows, int64_t base, int nthreads, float (*qs)[128],
                                           int64_t* qoff) {
  constexpr int D = 128;
  if (threadIdx.x < kScoreQ) {
    const int64_t rr = base + threadIdx.x;
    qoff[threadIdx.x] = rr < rows ? ((rr % queries) * q_heads + kv * grp + rr / queries) * D : -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kScoreQ * D; i += nthreads) {
    const int64_t off = qoff[i >> 7];
    qs[i >> 7][i & (D - 1)] = off >= 0 ? Dtype<T>::to_f(query[off + (i & (D - 1))]) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kScoreTok * kScoreGroups) scores_cuda_core_kernel(
    const T* __restrict__ query, int64_t queries, int q_heads, const T* __restrict__ key, int64_t ks_t, int64_t ks_h,
    int64_t tokens, int grp, const float* __restrict__ lse, float scale, float* __restrict__ scores,
    int accumulate) {
  constexpr int D = 128, THREADS = kScoreTok * kScoreGroups;
  const int kv = blockIdx.y, tl = threadIdx.x % kScoreTok, rg = threadIdx.x / kScoreTok;
  const int64_t t = blockIdx.x * (int64_t)kScoreTok + tl;
  __shared__ float qs[kScoreQ][D];
  __shared__ float ls[kScoreQ];
  __shared__ int64_t qoff[kScoreQ];
  __shared__ float part[kScoreGroups][kScoreTok];
  float k[D];
  if (t < tokens) {
    const T* kr = key + t * ks_t + kv * ks_h;
#pragma unroll
    for (int d = 0; d < D; ++d) k[d] = Dtype<T>::to_f(kr[d]);
  }
  float total = 0.f;
  const int64_t rows = (int64_t)grp * queries;
  for (int64_t base = 0; base < rows; base += kScoreQ) {
    __syncthreads();
    stage_rows(query, queries, q_heads, kv, grp, rows, base, THREADS, qs, qoff);
    if (threadIdx.x < kScoreQ) {
      const int64_t rr = base + threadIdx.x;
      ls[threadIdx.x] = rr < rows ? lse[(int64_t)(kv * grp + rr / queries) * queries + rr % queries] : INFINITY;
    }
    __syncthreads();
    if (t < tokens) {
      for (int j = 4 * rg; j < kScoreQ; j += 4 * kScoreGroups) {
        float dot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int d = 0; d < D; ++d) {
#pragma unroll
          for (int r = 0; r < 4; ++r) dot[r] = fmaf(qs[j + r][d], k[d], dot[r]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) total += expf(dot[r] * scale - ls[j + r]);
      }
    }
  }
  part[rg][tl] = total;
  __syncthreads();
  if (rg == 0 && t < tokens) {
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < kScoreGroups; ++g) sum += part[g][tl];
    float* o = scores + (int64_t)kv * tokens + t;
    *o = accumulate ? *o + sum : sum;
  }
}

// Natural-log normaliser of every (query head, query) row over the given keys
// (for callers whose attention covers exactly these keys), in two launches.
// lse_partial_kernel: block (x, kv, z) takes 64 tokens of KV head kv and the
// z-th 32-row chunk of the head's query group (rows are independent, so the
// chunks spread over the grid), one thread per token holding its key row;
// each thread forms its logits (four rows per pass, as the scoring kernel
// does) and each row's (max, sum of exp) over the block's tokens is reduced
// by shuffles and across the warps, then stored as the block's partial.  lse_combine_kernel folds the partials
// of every row over the token blocks: M = max m, L = sum l * exp(m - M),
// lse = M + log(L).
constexpr int kLseTok = 64;
template <typename T>
__global__ void __launch_bounds__(kLseTok) lse_partial_kernel(const T* __restrict__ query, int64_t queries,
                                                              int q_heads, const T* __restrict__ key, int64_t ks_t,
                                                              int64_t ks_h, int64_t tokens, int grp, float scale,
                                                              float2* __restrict__ partial, int token_blocks) {
  constexpr int D = 128, WARPS = kLseTok / 32;
  const int kv = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)kLseTok + threadIdx.x;
  const int64_t base = (int64_t)blockIdx.z * kScoreQ;  // this block's 32-row chunk
  const bool live = t < tokens;
  __shared__ float qs[kScoreQ][D];
  __shared__ int64_t qoff[kScoreQ];
  __shared__ float2 red[kScoreQ][WARPS];
  float k[D];
  if (live) {
    const T* kr = key + t * ks_t + kv * ks_h;
#pragma unroll
    for (int d = 0; d < D; ++d) k[d] = Dtype<T>::to_f(kr[d]);
  }
  const int64_t rows = (int64_t)grp * queries;  // rr = g * queries + q of this KV head's group
  stage_rows(query, queries, q_heads, kv, grp, rows, base, kLseTok, qs, qoff);
  __syncthreads();
  for (int j = 0; j < kScoreQ; j += 4) {
    float dot[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
#pragma unroll
        for (int r = 0; r < 4; ++r) dot[r] = fmaf(qs[j + r][d], k[d], dot[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float sv = live ? dot[r] * scale : -INFINITY;
      float m = sv;
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      float l = (m == -INFINITY) ? 0.f : expf(sv - m);
#pragma unroll
      for (int off = 16; off; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) red[j + r][warp] = make_float2(m, l);
    }
  }
  __syncthreads();
  if (threadIdx.x < kScoreQ && base + threadIdx.x < rows) {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) m = fmaxf(m, red[threadIdx.x][w].x);
    float l = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float2 p = red[threadIdx.x][w];
        if (p.x != -INFINITY) l += p.y * expf(p.x - m);
      }
    }
    const int64_t row = (int64_t)kv * rows + base + threadIdx.x;  // = h * queries + q
    partial[row * token_blocks + blockIdx.x] = make_float2(m, l);
  }
}

__global__ void lse_combine_kernel(const float2* __restrict__ partial, int64_t rows, int token_blocks,
                                   float* __restrict__ lse) {
  const int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float2* p = partial + row * token_blocks;
  float m = -INFINITY;
  for (int b = 0; b < token_blocks; ++b) m = fmaxf(m, p[b].x);
  float l = 0.f;
  for (int b = 0; b < token_blocks; ++b)
    if (p[b].x != -INFINITY) l += p[b].y * expf(p[b].x - m);
  lse[row] = m + logf(l);
}

// ---------------------------------------------------------------- compaction
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) mask_prefix_kernel(const uint8_t* __restrict__ mask, int64_t rows,
                                                                   int64_t* __restrict__ prefix) {
  __shared__ int scan_smem[32];
  int64_t carry = 0;
  for (int64_t base = 0; base < rows; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const int f = (i < rows && mask[i]) ? 1 : 0;
    int total;
    const int ex = block_exclusive_scan<kScanThreads>(f, scan_smem, total);
    if (i < rows) prefix[i] = carry + ex;
    carry += total;
  }
  if (threadIdx.x == 0) prefix[rows] = carry;
}

template <typename V>
__global__ void compact_rows_kernel(const unsigned char* __restrict__ src, int64_t row_vecs,
                                    const uint8_t* __restrict__ mask, const int64_t* __restrict__ prefix,
                                    int64_t rows, const int64_t* __restrict__ types, unsigned char* __restrict__ dst,
                                    int64_t* __restrict__ types_out) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows || !mask[r]) return;
  const int64_t o = prefix[r];
  const V* s = reinterpret_cast<const V*>(src + r * row_vecs * (int64_t)sizeof(V));
  V* d = reinterpret_cast<V*>(dst + o * row_vecs * (int64_t)sizeof(V));
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) d[v] = s[v];
  if (types && (threadIdx.x & 31) == 0) types_out[o] = types[r];
}

}  // namespace
}  // namespace ucb

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

extern "C" int ucb_lse_merge(int n, const void* const* out_ptrs, const float* const* lse_ptrs, int dtype, int64_t rows,
                             int64_t heads, int64_t head_dim, void* out, float* lse_out, void* stream) {
  if (n <= 0 || n > ucb::kMaxMerge) return set_error(UCB_ERR_INVALID, "ucb_lse_merge: n must be in [1, 64]");
  if (!out_ptrs || !lse_ptrs || !out) return set_error(UCB_ERR_INVALID, "ucb_lse_merge: null pointer");
  if (rows <= 0 || heads <= 0 || head_dim <= 0) return set_error(UCB_ERR_INVALID, "ucb_lse_merge: empty shape");
  ucb::MergeArgs args;
  for (int i = 0; i < n; ++i) {
    if (!out_ptrs[i] || !lse_ptrs[i]) return set_error(UCB_ERR_INVALID, "ucb_lse_merge: null summary %d", i);
    args.o[i] = out_ptrs[i];
    args.lse[i] = lse_ptrs[i];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(rows * heads);
  const int threads = head_dim >= 128 ? 128 : 64;
  switch (dtype) {
    case UCB_BF16:
      ucb::lse_merge_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(args, n, rows, heads, head_dim, static_cast<__nv_bfloat16*>(out), lse_out);
      break;
    case UCB_F16:
      ucb::lse_merge_kernel<__half><<<grid, threads, 0, s>>>(args, n, rows, heads, head_dim, static_cast<__half*>(out), lse_out);
      break;
    case UCB_F32:
      ucb::lse_merge_kernel<float><<<grid, threads, 0, s>>>(args, n, rows, heads, head_dim, static_cast<float*>(out), lse_out);
      break;
    default:
      return set_error(UCB_ERR_INVALID, "ucb_lse_merge: dtype %d unsupported", dtype);
  }
  return check_launch("lse_merge_kernel");
}

extern "C" int ucb_h2o_select(const float* scores, int64_t score_stride, int heads, int64_t tokens,
                              int64_t history_end, int64_t heavy_k, int64_t recent, int64_t* index_out,
                              void* stream) {
  if (!scores || !index_out) return set_error(UCB_ERR_INVALID, "ucb_h2o_select: null pointer");
  if (heads <= 0 || tokens <= 0 || tokens > (1LL << 24))
    return set_error(UCB_ERR_INVALID, "ucb_h2o_select: tokens must be in [1, 2^24]");
  if (history_end < 0 || history_end > tokens || heavy_k < 0 || heavy_k > history_end || recent < 0 ||
      recent > tokens || history_end + recent > tokens)
    return set_error(UCB_ERR_INVALID, "ucb_h2o_select: inconsistent budget (history_end=%lld heavy=%lld recent=%lld)",
                     (long long)history_end, (long long)heavy_k, (long long)recent);
  if (heavy_k + recent == 0) return UCB_OK;
  ucb::h2o_select_kernel<<<heads, ucb::kSelThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      scores, score_stride, tokens, history_end, heavy_k, recent, index_out);
  return check_launch("h2o_select_kernel");
}

extern "C" int ucb_gather_rows(const void* src, int64_t src_stride_head, int64_t src_stride_token, int64_t row_elems,
                               int elem_bytes, const int64_t* index, int heads, int64_t keep, void* dst,
                               void* stream) {
  if (!src || !index || !dst) return set_error(UCB_ERR_INVALID, "ucb_gather_rows: null pointer");
  if (heads <= 0 || keep < 0 || row_elems <= 0 || (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8))
    return set_error(UCB_ERR_INVALID, "ucb_gather_rows: bad shape");
  if (keep == 0) return UCB_OK;
  const int64_t row_bytes = row_elems * elem_bytes;
  const int64_t sh = src_stride_head * elem_bytes, st = src_stride_token * elem_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(static_cast<unsigned>((keep + 7) / 8), static_cast<unsigned>(heads));
  const auto* sp = static_cast<const unsigned char*>(src);
  auto* dp = static_cast<unsigned char*>(dst);
  if (row_bytes % 16 == 0 && sh % 16 == 0 && st % 16 == 0 && aligned16(src) && aligned16(dst))
    ucb::gather_rows_kernel<uint4><<<grid, 256, 0, s>>>(sp, sh, st, row_bytes / 16, index, keep, dp);
  else if (row_bytes % 8 == 0 && sh % 8 == 0 && st % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 7) == 0 &&
           (reinterpret_cast<uintptr_t>(dst) & 7) == 0)
    ucb::gather_rows_kernel<uint2><<<grid, 256, 0, s>>>(sp, sh, st, row_bytes / 8, index, keep, dp);
  else if (row_bytes % 4 == 0 && sh % 4 == 0 && st % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 3) == 0 &&
           (reinterpret_cast<uintptr_t>(dst) & 3) == 0)
    ucb::gather_rows_kernel<uint32_t><<<grid, 256, 0, s>>>(sp, sh, st, row_bytes / 4, index, keep, dp);
  else
    ucb::gather_rows_kernel<uint8_t><<<grid, 256, 0, s>>>(sp, sh, st, row_bytes, index, keep, dp);
  return check_launch("gather_rows_kernel");
}

extern "C" int ucb_h2o_accumulate_probs(const void* probs, int dtype, int q_heads, int64_t queries, int64_t tokens,
                                        int kv_heads, float* scores, int accumulate, void* stream) {
  if (!probs || !scores) return set_error(UCB_ERR_INVALID, "ucb_h2o_accumulate_probs: null pointer");
  if (kv_heads <= 0 || q_heads % kv_heads)
    return set_error(UCB_ERR_INVALID, "Query heads must be divisible by KV heads for GQA H2O");
  if (tokens <= 0 || queries <= 0) return UCB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(static_cast<unsigned>((tokens + 255) / 256), static_cast<unsigned>(kv_heads));
  const int grp = q_heads / kv_heads;
  switch (dtype) {
    case UCB_F32:
      ucb::accumulate_probs_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(probs), grp, queries, tokens, kv_heads, scores, accumulate);
      break;
    case UCB_BF16:
      ucb::accumulate_probs_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(probs), grp, queries, tokens, kv_heads, scores, accumulate);
      break;
    case UCB_F16:
      ucb::accumulate_probs_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(probs), grp, queries, tokens, kv_heads, scores, accumulate);
      break;
    default:
      return set_error(UCB_ERR_INVALID, "ucb_h2o_accumulate_probs: dtype %d unsupported", dtype);
  }
  return check_launch("accumulate_probs_kernel");
}

extern "C" int ucb_h2o_scores(const void* query, int dtype, int64_t queries, int q_heads, const void* key,
                              int64_t key_stride_token, int64_t key_stride_head, int64_t tokens, int kv_heads,
                              int head_dim, const float* lse, float* lse_workspace, float softmax_scale,
                              float* scores, int accumulate, void* stream) {
  if (!query || !key || !scores || (!lse && !lse_workspace))
    return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: null pointer");
  if (head_dim != 128) return set_error(UCB_ERR_UNSUPPORTED, "ucb_h2o_scores: head_dim must be 128");
  if (kv_heads <= 0 || q_heads % kv_heads)
    return set_error(UCB_ERR_INVALID, "Query heads must be divisible by KV heads for GQA H2O");
  if (dtype != UCB_BF16 && dtype != UCB_F32)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_h2o_scores: bfloat16 or float32 query and keys");
  if (tokens <= 0 || queries <= 0) return UCB_OK;
  const int grp = q_heads / kv_heads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (lse == nullptr) {
    // workspace: lse [q_heads * queries] floats, then the partials (8-byte aligned)
    const int64_t rows = (int64_t)q_heads * queries;
    const int token_blocks = static_cast<int>((tokens + ucb::kLseTok - 1) / ucb::kLseTok);
    float2* partial = reinterpret_cast<float2*>(lse_workspace + ((rows + 1) & ~int64_t(1)));
    if (reinterpret_cast<uintptr_t>(lse_workspace) & 7)
      return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: lse_workspace must be 8-byte aligned");
    const int64_t chunks = ((int64_t)grp * queries + ucb::kScoreQ - 1) / ucb::kScoreQ;
    if (chunks > 65535) return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: too many query rows per KV head");
    const dim3 pgrid(static_cast<unsigned>(token_blocks), static_cast<unsigned>(kv_heads),
                     static_cast<unsigned>(chunks));
    if (dtype == UCB_BF16)
      ucb::lse_partial_kernel<__nv_bfloat16><<<pgrid, ucb::kLseTok, 0, s>>>(
          static_cast<const __nv_bfloat16*>(query), queries, q_heads, static_cast<const __nv_bfloat16*>(key),
          key_stride_token, key_stride_head, tokens, grp, softmax_scale, partial, token_blocks);
    else
      ucb::lse_partial_kernel<float><<<pgrid, ucb::kLseTok, 0, s>>>(
          static_cast<const float*>(query), queries, q_heads, static_cast<const float*>(key), key_stride_token,
          key_stride_head, tokens, grp, softmax_scale, partial, token_blocks);
    int rc = check_launch("lse_partial_kernel");
    if (rc) return rc;
    ucb::lse_combine_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, s>>>(partial, rows, token_blocks,
                                                                                      lse_workspace);
    rc = check_launch("lse_combine_kernel");
    if (rc) return rc;
    lse = lse_workspace;
  }
  dim3 grid(static_cast<unsigned>((tokens + 127) / 128), static_cast<unsigned>(kv_heads));
  if (dtype == UCB_BF16) {
    if ((reinterpret_cast<uintptr_t>(query) & 15) || (reinterpret_cast<uintptr_t>(key) & 3) ||
        (key_stride_token & 1) || (key_stride_head & 1))
      return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: bf16 query must be 16-byte and key rows 4-byte aligned");
    ucb::scores_mma_kernel<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(query), queries, q_heads,
                                                static_cast<const __nv_bfloat16*>(key), key_stride_token,
                                                key_stride_head, tokens, grp, lse,
                                                softmax_scale * 1.4426950408889634f, scores, accumulate);
    return check_launch("scores_mma_kernel");
  }
  const dim3 grid64(static_cast<unsigned>((tokens + ucb::kScoreTok - 1) / ucb::kScoreTok),
                    static_cast<unsigned>(kv_heads));
  ucb::scores_cuda_core_kernel<float><<<grid64, ucb::kScoreTok * ucb::kScoreGroups, 0, s>>>(
      static_cast<const float*>(query), queries, q_heads,
                                                           static_cast<const float*>(key), key_stride_token,
                                                           key_stride_head, tokens, grp, lse, softmax_scale, scores,
                                                           accumulate);
  return check_launch("scores_cuda_core_kernel");
}

extern "C" int ucb_h2o_scores_from_lse(const void* query, int64_t queries, int q_heads, const void* key,
                                       int64_t key_stride_token, int64_t key_stride_head, int64_t tokens,
                                       int kv_heads, int head_dim, const float* lse, float softmax_scale,
                                       float* scores, int accumulate, void* stream) {
  if (!lse) return set_error(UCB_ERR_INVALID, "ucb_h2o_scores_from_lse: null pointer");
  return ucb_h2o_scores(query, UCB_BF16, queries, q_heads, key, key_stride_token, key_stride_head, tokens, kv_heads,
                        head_dim, lse, nullptr, softmax_scale, scores, accumulate, stream);
}

extern "C" int ucb_compact_rows(const void* src, int64_t row_bytes, const uint8_t* mask, int64_t rows,
                                const int64_t* types, void* dst, int64_t* types_out, int64_t* prefix,
                                int64_t* kept_host, void* stream) {
  if (!src || !mask || !dst || !prefix) return set_error(UCB_ERR_INVALID, "ucb_compact_rows: null pointer");
  if (types && !types_out) return set_error(UCB_ERR_INVALID, "ucb_compact_rows: types_out required");
  if (rows < 0 || row_bytes <= 0) return set_error(UCB_ERR_INVALID, "ucb_compact_rows: bad shape");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (kept_host) *kept_host = 0;
    return UCB_OK;
  }
  ucb::mask_prefix_kernel<<<1, ucb::kScanThreads, 0, s>>>(mask, rows, prefix);
  int rc = check_launch("mask_prefix_kernel");
  if (rc) return rc;
  dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  const auto* sp = static_cast<const unsigned char*>(src);
  auto* dp = static_cast<unsigned char*>(dst);
  if (row_bytes % 16 == 0 && aligned16(src) && aligned16(dst))
    ucb::compact_rows_kernel<uint4><<<grid, 256, 0, s>>>(sp, row_bytes / 16, mask, prefix, rows, types, dp, types_out);
  else
    ucb::compact_rows_kernel<uint8_t><<<grid, 256, 0, s>>>(sp, row_bytes, mask, prefix, rows, types, dp, types_out);
  rc = check_launch("compact_rows_kernel");
  if (rc) return rc;
  if (kept_host) {
    if (cudaMemcpyAsync(kept_host, prefix + rows, sizeof(int64_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return set_error(UCB_ERR_CUDA, "ucb_compact_rows: reading the kept count failed");
  }
  return UCB_OK;
}

extern "C" int64_t ucb_h2o_scores_workspace_floats(int64_t queries, int q_heads, int64_t tokens) {
  const int64_t rows = (int64_t)q_heads * queries;
  const int64_t token_blocks = (tokens + ucb::kLseTok - 1) / ucb::kLseTok;
  return ((rows + 1) & ~int64_t(1)) + 2 * rows * token_blocks;
}
