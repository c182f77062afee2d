// LSE merge of attention summaries, H2O scoring / selection / gathering and
// dense-cache row compaction.
#include <cfloat>

#include <cooperative_groups.h>

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
// STAGED: the history's keys are read from global memory once into shared
// memory (history_end * 4 bytes of dynamic shared memory, at most
// kSelStagedMax keys) and every pass reads them there; otherwise each pass
// reads the scores again.
constexpr int64_t kSelStagedMax = 51200;
template <bool STAGED>
__global__ void __launch_bounds__(kSelThreads) h2o_select_kernel(const float* __restrict__ scores,
                                                                 int64_t stride, int64_t tokens,
                                                                 int64_t history_end, int64_t heavy_k,
                                                                 int64_t recent, int64_t* __restrict__ out) {
  const int h = blockIdx.x, tid = threadIdx.x;
  const float* row = scores + h * stride;
  int64_t* orow = out + h * (heavy_k + recent);
  extern __shared__ uint32_t staged_keys[];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int64_t s_krem;
  __shared__ int scan_smem[32];
  auto key_at = [&](int64_t i) { return STAGED ? staged_keys[i] : score_key(row[i]); };
  if (heavy_k > 0) {
    if constexpr (STAGED) {
      for (int64_t i = tid; i < history_end; i += kSelThreads) staged_keys[i] = score_key(row[i]);
      __syncthreads();
    }
    uint32_t prefix = 0, mask = 0;
    int64_t krem = heavy_k;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
      __syncthreads();
      // histogram of the candidates' next byte; the lanes of a warp that share
      // a bin add once (scores of one row share their high bytes, so plain
      // per-element atomics would queue on a few bins)
      for (int64_t base = 0; base < history_end; base += kSelThreads) {
        const int64_t i = base + tid;
        const uint32_t key = i < history_end ? key_at(i) : 0u;
        const bool cand = i < history_end && (key & mask) == prefix;
        const unsigned active = __ballot_sync(0xffffffffu, cand);
        if (cand) {
          const unsigned bin = (key >> shift) & 255u;
          const unsigned peers = __match_any_sync(active, bin);
          if ((tid & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], static_cast<unsigned>(__popc(peers)));
        }
      }
      __syncthreads();
      if (tid < 32) {
        // the bin holding the krem-th largest candidate: lane l sums bins
        // 255 - 8l down to 248 - 8l, a scan over the lanes finds the lane,
        // then that lane walks its eight bins (as a scan from bin 255 would)
        const int lane = tid;
        int64_t own = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) own += hist[255 - 8 * lane - q];
        int64_t incl = own;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int64_t v = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += v;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= krem);
        const int first = hit ? __ffs(hit) - 1 : -1;
        if (first < 0 && lane == 31) {  // not reached for a consistent budget
          s_prefix = prefix;
          s_krem = krem - incl;
        } else if (lane == first) {
          int64_t cum = incl - own;
          int sel = 0;
          for (int q = 0; q < 8; ++q) {
            const int b = 255 - 8 * lane - q;
            if (cum + hist[b] >= krem) {
              sel = b;
              break;
            }
            cum += hist[b];
          }
          s_prefix = prefix | (static_cast<uint32_t>(sel) << shift);
          s_krem = krem - cum;
        }
      }
      __syncthreads();
      prefix = s_prefix;
      krem = s_krem;
      mask |= 255u << shift;
      __syncthreads();
    }
    const uint32_t thr = prefix;
    const int64_t need_eq = krem;  // entries equal to thr to keep (lowest indices)
    // Thread t owns the contiguous slice [t * chunk, (t + 1) * chunk) of the
    // history: it counts the keys above thr and equal to it, one scan over
    // the equal counts tells it how many of its equal keys are among the
    // need_eq lowest-index ones, a second scan over the kept counts gives its
    // output offset, and it writes its kept indices in ascending order.
    const int64_t chunk = (history_end + kSelThreads - 1) / kSelThreads;
    const int64_t lo = min(history_end, tid * chunk), hi = min(history_end, lo + chunk);
    int n_gt = 0, n_eq = 0;
    for (int64_t i = lo; i < hi; ++i) {
      const uint32_t key = key_at(i);
      n_gt += key > thr;
      n_eq += key == thr;
    }
    int eq_total;
    const int eq_before = block_exclusive_scan<kSelThreads>(n_eq, scan_smem, eq_total);
    const int64_t eq_room = need_eq - eq_before;  // equal keys still wanted before this slice
    const int eq_take = eq_room <= 0 ? 0 : (eq_room < n_eq ? static_cast<int>(eq_room) : n_eq);
    int take_total;
    int64_t pos = block_exclusive_scan<kSelThreads>(n_gt + eq_take, scan_smem, take_total);
    int eq_left = eq_take;
    for (int64_t i = lo; i < hi; ++i) {
      const uint32_t key = key_at(i);
      if (key > thr || (key == thr && eq_left > 0)) {
        eq_left -= key == thr;
        orow[pos++] = i;
      }
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
// Logits of one KV head's query rows against its keys, as register-blocked
// tiles on the CUDA cores (fp32 arithmetic, for fp32 callers whose scores
// must keep fp32 accuracy; bf16 inputs are widened exactly).  A 256-thread
// block holds a 64-row query tile and a 64-token key tile, all 128 channels,
// in shared memory ([row][channel], 132-float pitch: the 16-byte loads of 8
// consecutive rows fall in distinct banks).  Thread (ty, tx) = (tid / 16,
// tid % 16) owns rows ty + 16i and tokens tx + 16j (i, j < 4): 16
// accumulators, 64 independent FMAs per four channels.  Every logit is one
// fmaf chain over channels 0..127 in order, the arithmetic of a plain dot
// product loop.  Query row rr of the head's group (rr = g * queries + q) is
// query[q, kv * grp + g, :].  Tiles are staged with 16-byte (fp32) or 8-byte
// (bf16) loads, a warp per row, when every row start is aligned (VEC), else
// element by element.
constexpr int kTile = 64, kTileThreads = 256, kTilePitch = 132;
constexpr int kLseTok = kTile;  // token block of the LSE partials
constexpr int kTileSmemBytes = 2 * kTile * kTilePitch * 4;

// The four channels [4c, 4c + 4) of one row, widened to fp32 (zeros for a
// missing row: src == nullptr).
template <typename T, bool VEC>
__device__ __forceinline__ float4 load_quad(const T* src, int c) {
  if (src == nullptr) return make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (VEC && sizeof(T) == 4) {
    return *reinterpret_cast<const float4*>(src + 4 * c);
  } else if constexpr (VEC) {
    const uint2 w = *reinterpret_cast<const uint2*>(src + 4 * c);
    return make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
  } else {
    return make_float4(Dtype<T>::to_f(src[4 * c]), Dtype<T>::to_f(src[4 * c + 1]), Dtype<T>::to_f(src[4 * c + 2]),
                       Dtype<T>::to_f(src[4 * c + 3]));
  }
}

template <typename T>
__device__ __forceinline__ const T* query_row(const T* query, int64_t queries, int q_heads, int kv, int grp,
                                              int64_t rows, int64_t rr) {
  if (rr >= rows) return nullptr;
  return query + ((rr % queries) * q_heads + kv * grp + rr / queries) * 128;
}

// One thread's eight quads of a 64 x 128 tile (thread tid takes rows tid / 32
// + 8n, channel quad tid % 32: a warp reads one row), to registers and then
// to shared memory.
template <typename T, bool VEC, typename RowFn>
__device__ __forceinline__ void load_tile_regs(RowFn row_ptr, float4 (&v)[8]) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int n = 0; n < 8; ++n) v[n] = load_quad<T, VEC>(row_ptr(tid / 32 + 8 * n), tid % 32);
}
__device__ __forceinline__ void store_tile_regs(float* tile, const float4 (&v)[8]) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int n = 0; n < 8; ++n)
    *reinterpret_cast<float4*>(tile + (tid / 32 + 8 * n) * kTilePitch + 4 * (tid % 32)) = v[n];
}

// acc[i][j] = logit of tile row ty + 16i and tile token tx + 16j.
__device__ __forceinline__ void tile_logits(const float* qs, const float* ks, float (&acc)[4][4]) {
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
  for (int c = 0; c < 32; ++c) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(qs + (ty + 16 * i) * kTilePitch + 4 * c);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(ks + (tx + 16 * j) * kTilePitch + 4 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
        acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
        acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
        acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
      }
  }
}

// H2O scores from the LSE: a cluster of kScoreCluster blocks owns tokens
// [64y, 64y + 64) of KV head z; block x of the cluster keeps that key tile in
// shared memory and walks row tiles x, x + 8, x + 16, ... of the head's query
// rows (the next tile's rows loading into registers while the current
// tile's logits run), adding exp(logit * scale - lse[row]) per token.  The 16
// row groups of a block are added in group order, then rank 0 adds the
// cluster's eight block sums in rank order through distributed shared
// memory, so the result does not depend on scheduling.
constexpr int kScoreCluster = 8;
template <typename T, bool VEC>
__global__ void __cluster_dims__(kScoreCluster, 1, 1) __launch_bounds__(kTileThreads) scores_tile_kernel(
    const T* __restrict__ query, int64_t queries, int q_heads, const T* __restrict__ key, int64_t ks_t, int64_t ks_h,
    int64_t tokens, int grp, const float* __restrict__ lse, float scale, float* __restrict__ scores,
    int accumulate) {
  extern __shared__ __align__(16) float tile_smem[];
  float* qs = tile_smem;
  float* ks = tile_smem + kTile * kTilePitch;
  __shared__ float part[16][kTile];
  __shared__ float block_sum[kTile];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int kv = blockIdx.z, tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t t0 = blockIdx.y * (int64_t)kTile;
  const int64_t rows = (int64_t)grp * queries;
  constexpr int64_t kStride = (int64_t)kScoreCluster * kTile;
  auto lse_of = [&](int64_t rr) {
    return rr < rows ? lse[(int64_t)(kv * grp + rr / queries) * queries + rr % queries] : INFINITY;
  };
  float tot[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t r0 = (int64_t)rank * kTile;
  if (r0 < rows) {
    float4 v[8];
    load_tile_regs<T, VEC>(
        [&](int r) -> const T* { return t0 + r < tokens ? key + (t0 + r) * ks_t + kv * ks_h : nullptr; }, v);
    store_tile_regs(ks, v);
    load_tile_regs<T, VEC>([&](int r) { return query_row(query, queries, q_heads, kv, grp, rows, r0 + r); }, v);
    store_tile_regs(qs, v);
    for (; r0 < rows; r0 += kStride) {
      float l[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) l[i] = lse_of(r0 + ty + 16 * i);
      const int64_t r1 = r0 + kStride;
      if (r1 < rows)
        load_tile_regs<T, VEC>([&](int r) { return query_row(query, queries, q_heads, kv, grp, rows, r1 + r); }, v);
      __syncthreads();  // this tile's rows are in shared memory
      float acc[4][4];
      tile_logits(qs, ks, acc);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) tot[j] += expf(acc[i][j] * scale - l[i]);
      __syncthreads();  // every thread is done with this tile's rows
      if (r1 < rows) store_tile_regs(qs, v);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) part[ty][tx + 16 * j] = tot[j];
  __syncthreads();
  if (tid < kTile) {
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < 16; ++g) sum += part[g][tid];
    block_sum[tid] = sum;
  }
  cluster.sync();  // every block's sums are visible to the cluster
  if (rank == 0 && tid < kTile && t0 + tid < tokens) {
    float sum = 0.f;
#pragma unroll
    for (int b = 0; b < kScoreCluster; ++b) sum += *cluster.map_shared_rank(&block_sum[tid], b);
    float* o = scores + (int64_t)kv * tokens + t0 + tid;
    *o = accumulate ? *o + sum : sum;
  }
  cluster.sync();  // the peers' shared memory stays alive until rank 0 has read it
}

// Natural-log normaliser of every (query head, query) row over the given keys
// (for callers whose attention covers exactly these keys), in two launches.
// lse_tile_kernel: block (x, y, kv) computes the 64-row x 64-token logit tile
// (rows 64y.., tokens 64x..) and stores each row's (max, sum of exp) over
// its tokens as the block's partial (four values per thread, then shuffles
// across the 16 threads of a row).  lse_combine_kernel folds the partials of
// every row over the token blocks: M = max m, L = sum l * exp(m - M),
// lse = M + log(L).
template <typename T, bool VEC>
__global__ void __launch_bounds__(kTileThreads) lse_tile_kernel(const T* __restrict__ query, int64_t queries,
                                                                int q_heads, const T* __restrict__ key, int64_t ks_t,
                                                                int64_t ks_h, int64_t tokens, int grp, float scale,
                                                                float2* __restrict__ partial, int token_blocks) {
  extern __shared__ __align__(16) float tile_smem[];
  float* qs = tile_smem;
  float* ks = tile_smem + kTile * kTilePitch;
  const int kv = blockIdx.z, tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t t0 = blockIdx.x * (int64_t)kTile, r0 = blockIdx.y * (int64_t)kTile;
  const int64_t rows = (int64_t)grp * queries;
  float4 v[8];
  load_tile_regs<T, VEC>(
      [&](int r) -> const T* { return t0 + r < tokens ? key + (t0 + r) * ks_t + kv * ks_h : nullptr; }, v);
  store_tile_regs(ks, v);
  load_tile_regs<T, VEC>([&](int r) { return query_row(query, queries, q_heads, kv, grp, rows, r0 + r); }, v);
  store_tile_regs(qs, v);
  __syncthreads();
  float acc[4][4];
  tile_logits(qs, ks, acc);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float sv[4], m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sv[j] = t0 + tx + 16 * j < tokens ? acc[i][j] * scale : -INFINITY;
      m = fmaxf(m, sv[j]);
    }
#pragma unroll
    for (int off = 8; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float l = 0.f;
    if (m != -INFINITY) {
#pragma unroll
      for (int j = 0; j < 4; ++j) l += expf(sv[j] - m);
    }
#pragma unroll
    for (int off = 8; off; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    const int64_t rr = r0 + ty + 16 * i;
    if (tx == 0 && rr < rows) partial[((int64_t)kv * rows + rr) * token_blocks + blockIdx.x] = make_float2(m, l);
  }
}

// Shared-memory reservation of the tile kernels, once per device.
template <typename KernelT>
int reserve_tile_smem(KernelT kernel, int slot) {
  static bool done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[slot][dev]) return UCB_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTileSmemBytes) != cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "ucb_h2o_scores: cannot reserve %d bytes of shared memory",
                               kTileSmemBytes);
  if (dev >= 0 && dev < 64) done[slot][dev] = true;
  return UCB_OK;
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (history_end <= ucb::kSelStagedMax) {
    const int bytes = static_cast<int>(history_end * 4);
    static bool reserved[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !reserved[dev]) {
      if (cudaFuncSetAttribute(ucb::h2o_select_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ucb::kSelStagedMax * 4)) != cudaSuccess)
        return set_error(UCB_ERR_CUDA, "ucb_h2o_select: cannot reserve shared memory");
      if (dev >= 0 && dev < 64) reserved[dev] = true;
    }
    ucb::h2o_select_kernel<true><<<heads, ucb::kSelThreads, bytes, s>>>(scores, score_stride, tokens, history_end,
                                                                       heavy_k, recent, index_out);
  } else {
    ucb::h2o_select_kernel<false><<<heads, ucb::kSelThreads, 0, s>>>(scores, score_stride, tokens, history_end,
                                                                     heavy_k, recent, index_out);
  }
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
    const int64_t row_blocks = ((int64_t)grp * queries + ucb::kTile - 1) / ucb::kTile;
    if (row_blocks > 65535 || kv_heads > 65535)
      return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: too many query rows per KV head");
    const dim3 pgrid(static_cast<unsigned>(token_blocks), static_cast<unsigned>(row_blocks),
                     static_cast<unsigned>(kv_heads));
    // quads of four elements load as one 8-byte (bf16) or 16-byte (fp32)
    // access when every row start is aligned to that size
    const uintptr_t align_mask = dtype == UCB_BF16 ? 7 : 15;
    const bool vec = ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key)) & align_mask) == 0 &&
                     key_stride_token % 4 == 0 && key_stride_head % 4 == 0;
    int rc = UCB_OK;
    if (dtype == UCB_BF16) {
      const auto* qb = static_cast<const __nv_bfloat16*>(query);
      const auto* kb = static_cast<const __nv_bfloat16*>(key);
      if (vec) {
        rc = ucb::reserve_tile_smem(ucb::lse_tile_kernel<__nv_bfloat16, true>, 0);
        if (!rc)
          ucb::lse_tile_kernel<__nv_bfloat16, true><<<pgrid, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
              qb, queries, q_heads, kb, key_stride_token, key_stride_head, tokens, grp, softmax_scale, partial,
              token_blocks);
      } else {
        rc = ucb::reserve_tile_smem(ucb::lse_tile_kernel<__nv_bfloat16, false>, 1);
        if (!rc)
          ucb::lse_tile_kernel<__nv_bfloat16, false><<<pgrid, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
              qb, queries, q_heads, kb, key_stride_token, key_stride_head, tokens, grp, softmax_scale, partial,
              token_blocks);
      }
    } else {
      const auto* qf = static_cast<const float*>(query);
      const auto* kf = static_cast<const float*>(key);
      if (vec) {
        rc = ucb::reserve_tile_smem(ucb::lse_tile_kernel<float, true>, 2);
        if (!rc)
          ucb::lse_tile_kernel<float, true><<<pgrid, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
              qf, queries, q_heads, kf, key_stride_token, key_stride_head, tokens, grp, softmax_scale, partial,
              token_blocks);
      } else {
        rc = ucb::reserve_tile_smem(ucb::lse_tile_kernel<float, false>, 3);
        if (!rc)
          ucb::lse_tile_kernel<float, false><<<pgrid, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
              qf, queries, q_heads, kf, key_stride_token, key_stride_head, tokens, grp, softmax_scale, partial,
              token_blocks);
      }
    }
    if (rc) return rc;
    rc = check_launch("lse_tile_kernel");
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
  const int64_t score_blocks = (tokens + ucb::kTile - 1) / ucb::kTile;
  if (score_blocks > 65535 || kv_heads > 65535)
    return set_error(UCB_ERR_INVALID, "ucb_h2o_scores: too many keys for the fp32 scoring grid");
  const dim3 grid64(ucb::kScoreCluster, static_cast<unsigned>(score_blocks), static_cast<unsigned>(kv_heads));
  const bool vec = (((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key)) & 15) == 0) &&
                   key_stride_token % 4 == 0 && key_stride_head % 4 == 0;
  const auto* qf = static_cast<const float*>(query);
  const auto* kf = static_cast<const float*>(key);
  int rc2 = vec ? ucb::reserve_tile_smem(ucb::scores_tile_kernel<float, true>, 0)
                : ucb::reserve_tile_smem(ucb::scores_tile_kernel<float, false>, 1);
  if (rc2) return rc2;
  if (vec)
    ucb::scores_tile_kernel<float, true><<<grid64, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
        qf, queries, q_heads, kf, key_stride_token, key_stride_head, tokens, grp, lse, softmax_scale, scores,
        accumulate);
  else
    ucb::scores_tile_kernel<float, false><<<grid64, ucb::kTileThreads, ucb::kTileSmemBytes, s>>>(
        qf, queries, q_heads, kf, key_stride_token, key_stride_head, tokens, grp, lse, softmax_scale, scores,
        accumulate);
  return check_launch("scores_tile_kernel");
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
