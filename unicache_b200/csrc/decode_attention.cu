// Single-token (decode) attention over packed KIVI and dense bf16 spans.
//
// Replaces, for q_len == 1: packed_kivi_attention_parts + softmax + apply_value
// (unicache/storage/kivi_cuda.py:238-329), the quantized-prefix summary
// (kivi_cuda.py:96-120) and the frozen-H2O concat path
// (unicache/adapters/bagel.py:1860-1901).
//
// Design (B200, HBM-bound, one persistent CTA per SM):
//  * The batch is a set of (sequence, KV head) pairs; each pair owns spans
//    (packed KIVI segments or dense bf16 rows).  Spans are cut into stages
//    (64 packed tokens or 8 dense tokens) and all stages of all pairs form
//    one flattened sequence of units.  The host gives every CTA a contiguous
//    range of units of equal bytes and every warp a contiguous sub-range that
//    crosses at most one segment boundary (segment = a pair's packed or dense
//    units), so the result does not depend on scheduling.
//  * Each warp streams its units with the TMA bulk-copy engine (cp.async.bulk,
//    no tensor map, no multicast) into a private two-slot ring guarded by
//    mbarriers; every wait is bounded.
//  * The query heads of a GQA group are the N=8 columns of mma.sync m16n8k16.
//    Keys: each code is dequantized to bf16 in registers exactly as the
//    reference restores its cache (one rounding of code*scale + minimum),
//    then QK runs on the tensor cores.  Values: the code is placed in an fp16
//    *subnormal* (code * 2^(p-24), multiplied exactly by the tensor core) and
//    the per-token group scale is folded into the probabilities:
//       sum_t p_t v_td = sum_t (p_t s_tg) c_td + sum_t p_t m_tg.
//  * Online softmax in the log2 domain per warp.  A warp writes the state
//    (max, sum, unnormalised rows) of each segment it processed to a
//    planner-assigned slot in global memory and exits (no CTA barrier, no
//    atomics); a second, stream-ordered kernel (state_merge_kernel or
//    state_merge_wide_kernel) folds each pair's slots into out and LSE.
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace ucb {
namespace decode {

constexpr int D = 128;
constexpr int KCH = D / 16;       // k-chunks of 16 channels
constexpr int NT = 64;            // tokens per packed stage
constexpr int DT = 8;             // tokens per dense stage
constexpr int DROW = 272;         // dense shared-memory row stride (bytes), conflict-free ldmatrix
constexpr int DENSE_STAGE = 2 * DT * DROW;
constexpr int MAXC = 4;           // pairs one CTA may touch
constexpr int MAX_SPANS = 16;     // spans one CTA may touch
constexpr uint32_t WAIT_LIMIT = 1u << 22;
constexpr int PARTIAL_FLOATS = 16 + 8 * D;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__host__ __device__ constexpr int round_up(int x, int a) { return (x + a - 1) / a * a; }

template <int KB, int VB, int G, typename ST>
struct Cfg {
  static constexpr int WARPS = (KB == 2 && VB == 2) ? 12 : 8;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int NG = D / G;                    // value groups per token
  static constexpr int GPS = (G >= NT) ? 1 : NT / G;  // key groups per stage
  static constexpr int KC = NT * D * KB / 8;
  static constexpr int VC = NT * D * VB / 8;
  static constexpr int KS = GPS * D * (int)sizeof(ST);
  static constexpr int VS = NT * NG * (int)sizeof(ST);
  static constexpr int OFF_KC = 0;
  static constexpr int OFF_VC = OFF_KC + KC;
  static constexpr int OFF_KS = OFF_VC + VC;
  static constexpr int OFF_KM = OFF_KS + KS;
  static constexpr int OFF_VS = OFF_KM + KS;
  static constexpr int OFF_VM = OFF_VS + VS;
  static constexpr int PACKED_STAGE = OFF_VM + VS;
  static constexpr int SLOT = round_up(PACKED_STAGE > DENSE_STAGE ? PACKED_STAGE : DENSE_STAGE, 128);
  static constexpr int OFF_Q = WARPS * 2 * SLOT;                  // MAXC x 8 query rows (bf16)
  static constexpr int OFF_ZERO = OFF_Q + MAXC * 8 * D * 2;           // one zero row
  static constexpr int OFF_BAR = OFF_ZERO + D * 2;                    // WARPS x 2 mbarriers
  static constexpr int OFF_SPANS = round_up(OFF_BAR + WARPS * 2 * 8, 16);  // the CTA's spans
  static constexpr int SMEM = OFF_SPANS + MAX_SPANS * (int)sizeof(ucb_span);
  static_assert(KC >= NT * NG * 4 + 16 * NG * 8, "value tables must fit the key-code area");
};

// Token <-> MMA-row map inside a 16-token tile.  Row r and row r+8 of lane
// group r share one byte of a 2-bit key word, and the four tokens a lane needs
// as AV k-columns fall in four different shared-memory bank groups.
__device__ __forceinline__ int tile_pos(int r) { return (r & 1) ? (((r >> 1) + 2) & 3) : (r >> 1); }
__device__ __forceinline__ int tile_tok(int m) {
  const int r = m & 7;
  const int p = (m < 8) ? tile_pos(r) : ((tile_pos(r) + 1) & 3);
  return 4 * (r & 3) + p;
}

struct WarpState {
  float mrun[2];  // running max (log2 domain) for heads 2c, 2c+1
  float lrun[2];  // lane-partial running sums
};

__device__ __forceinline__ float warp_max_r(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}
__device__ __forceinline__ float warp_sum_r(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// Online-softmax update for NTILE C fragments.  `lg` holds raw q.k (or -inf
// for masked slots) and becomes exp2(q.k * scale_log2 - running max); the max
// is kept in the log2 domain.  Returns whether any lane's running max moved
// (then the accumulators need the alpha factors).
template <int NTILE>
__device__ __forceinline__ bool softmax_update(float (&lg)[NTILE][4], float scale_log2, WarpState& st, float& alpha0,
                                               float& alpha1) {
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NTILE; ++j) {
    mx0 = fmaxf(mx0, fmaxf(lg[j][0], lg[j][2]));
    mx1 = fmaxf(mx1, fmaxf(lg[j][1], lg[j][3]));
  }
  mx0 = warp_max_r(mx0) * scale_log2;
  mx1 = warp_max_r(mx1) * scale_log2;
  const float n0 = fmaxf(st.mrun[0], mx0), n1 = fmaxf(st.mrun[1], mx1);
  const bool moved = __any_sync(0xffffffffu, n0 != st.mrun[0] || n1 != st.mrun[1]);
  alpha0 = fast_exp2(st.mrun[0] - n0);
  alpha1 = fast_exp2(st.mrun[1] - n1);
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int j = 0; j < NTILE; ++j) {
    lg[j][0] = fast_exp2(fmaf(lg[j][0], scale_log2, -n0));
    lg[j][1] = fast_exp2(fmaf(lg[j][1], scale_log2, -n1));
    lg[j][2] = fast_exp2(fmaf(lg[j][2], scale_log2, -n0));
    lg[j][3] = fast_exp2(fmaf(lg[j][3], scale_log2, -n1));
    s0 += lg[j][0] + lg[j][2];
    s1 += lg[j][1] + lg[j][3];
  }
  st.lrun[0] = st.lrun[0] * alpha0 + s0;
  st.lrun[1] = st.lrun[1] * alpha1 + s1;
  st.mrun[0] = n0;
  st.mrun[1] = n1;
  return moved;
}

__device__ __forceinline__ uint2 lds64(const unsigned char* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }

// Tokens of a span this launch reads: a dense span whose key_scale field
// points at a device int32 (a growing decode suffix) holds min(tokens, that
// value) live tokens; every other span holds `tokens`.  The planner sizes a
// growing span for its capacity, so one plan (and one captured graph) serves
// every step while the suffix grows.  The CTA reads each growing span's
// length once, after copying its span records into shared memory, and stores
// the live count in the shared copy's `tokens` (the length does not change
// during a launch).
__device__ __forceinline__ int live_tokens(const ucb_span& sp) { return sp.tokens; }

struct Params {
  const __nv_bfloat16* query;
  int64_t query_stride;
  int grp;  // query heads per KV head
  int hq;   // query heads per sequence (row length of lse)
  const ucb_span* spans;
  int num_spans;
  const ucb_decode_cta* ctas;
  const int32_t* warp_bounds;  // per CTA: WARPS+1 unit boundaries
  const ucb_decode_pair* pairs;
  int num_pairs;
  float scale_log2;  // softmax_scale * log2(e)
  float* partials;             // warp states, one slot each
  int max_partials;            // slots the partials buffer holds; larger slot indices are rejected
  const int32_t* warp_slots;   // per CTA and warp: {first-segment slot, last-segment slot}, -1 = none
  __nv_bfloat16* out;
  int64_t out_stride;
  float* lse;
  unsigned int* err;
  uint64_t* trace;  // optional: per CTA 32 words, see ucb_decode_set_trace
};

template <int KB, int VB, int G, typename ST>
struct Kernel {
  using C = Cfg<KB, VB, G, ST>;

  // -------------------------------------------------------------- stage issue
  __device__ static void issue_packed(const ucb_span& sp, int t0, int t1, unsigned char* slot, uint64_t* bar,
                                      int lane) {
    if (lane != 0) return;
    const int n = t1 - t0;
    const uint32_t kc = n * D * KB / 8, vc = n * D * VB / 8;
    const int g0 = t0 / G;
    const int gcount = (G >= NT) ? 1 : (n + G - 1) / G;
    const uint32_t ks = gcount * D * sizeof(ST);
    const uint32_t vs = n * C::NG * sizeof(ST);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, kc + vc + 2 * ks + 2 * vs);
    const unsigned char* kcode = static_cast<const unsigned char*>(sp.key_code) + (size_t)t0 * D * KB / 8;
    const unsigned char* vcode = static_cast<const unsigned char*>(sp.value_code) + (size_t)t0 * D * VB / 8;
    const unsigned char* kscale = static_cast<const unsigned char*>(sp.key_scale) + (size_t)g0 * D * sizeof(ST);
    const unsigned char* kmin = static_cast<const unsigned char*>(sp.key_minimum) + (size_t)g0 * D * sizeof(ST);
    const unsigned char* vscale = static_cast<const unsigned char*>(sp.value_scale) + (size_t)t0 * C::NG * sizeof(ST);
    const unsigned char* vmin = static_cast<const unsigned char*>(sp.value_minimum) + (size_t)t0 * C::NG * sizeof(ST);
    const uint64_t pol = l2_evict_first_policy();
    bulk_g2s_hint(slot + C::OFF_KC, kcode, kc, bar, pol);
    bulk_g2s_hint(slot + C::OFF_VC, vcode, vc, bar, pol);
    bulk_g2s_hint(slot + C::OFF_KS, kscale, ks, bar, pol);
    bulk_g2s_hint(slot + C::OFF_KM, kmin, ks, bar, pol);
    bulk_g2s_hint(slot + C::OFF_VS, vscale, vs, bar, pol);
    bulk_g2s_hint(slot + C::OFF_VM, vmin, vs, bar, pol);
  }

  __device__ static void issue_dense(const ucb_span& sp, int t0, int t1, unsigned char* slot, uint64_t* bar,
                                     int lane) {
    const int n = max(0, t1 - t0);  // a growing span's unit past its live length copies nothing
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, 2u * n * D * 2u);
    }
    __syncwarp();
    const int row = lane & 7;
    if (lane < 16 && row < n) {
      const bool is_v = lane >= 8;
      const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(is_v ? sp.value_code : sp.key_code);
      const int64_t stride = is_v ? sp.value_stride : sp.key_stride;
      bulk_g2s_hint(slot + (is_v ? DT * DROW : 0) + row * DROW, base + (t0 + row) * stride, D * 2, bar,
                    l2_evict_first_policy());
    }
  }

  // -------------------------------------------------------------- packed stage
  template <bool FULL>
  __device__ static void packed_stage(const unsigned char* slot, int n_valid, int lane, const uint32_t (&qbp)[KCH][2],
                                      float scale_log2, WarpState& st, float (&o)[8][4], float (&accm)[4]) {
    const int r = lane >> 2, c = lane & 3;
    const int pr = tile_pos(r), pr2 = (pr + 1) & 3;
    const int tok_lo = 4 * (r & 3) + pr, tok_hi = 4 * (r & 3) + pr2;

    // Keys: every code is dequantized to bf16 exactly as the reference stores
    // its restored cache (physical.py:178-201: one rounding of code*scale+min),
    // then QK runs on the tensor cores against the raw bf16 query.  The four
    // 16-token tiles are interleaved so four MMA chains are in flight.
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // 2-bit: one PRMT copies byte (r%4) of two key words into both bytes of
    // each half, one shift by 2*pr brings the codes of rows r and r+8 to bits
    // 0-1 and 2-3 of each half; a single AND/OR then forms 128 + code or
    // 32 + code exactly in bf16.  4-bit: one PRMT per row.
    uint32_t sel_lo, sel_hi, sh_lo, sh_hi;
    if constexpr (KB == 2) {
      const uint32_t b = r & 3;
      sel_lo = sel_hi = b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12);
      sh_lo = sh_hi = 2 * pr;
    } else {
      const int blo = (r & 1) * 2 + (pr >> 1), bhi = (r & 1) * 2 + (pr2 >> 1);
      sel_lo = blo | ((4 + blo) << 8);
      sel_hi = bhi | ((4 + bhi) << 8);
      sh_lo = 4 * (pr & 1);
      sh_hi = 4 * (pr2 & 1);
    }
    // Channel map of the QK contraction: in k-chunk kk, lane c owns channels
    // 32*(kk/2) + 8c + 4*(kk%2) + {0..3} (k = 2c, 2c+1, 2c+8, 2c+9), so one
    // 128-bit load brings a lane's statistics for two chunks.
    uint4 ks4[C::GPS], km4[C::GPS];
#pragma unroll
    for (int kk = 0; kk < KCH; ++kk) {
      const int ch = 32 * (kk >> 1) + 8 * c + 4 * (kk & 1);
      if ((kk & 1) == 0) {
#pragma unroll
        for (int gi = 0; gi < C::GPS; ++gi) {
          ks4[gi] = lds128(slot + C::OFF_KS + (gi * D + ch) * (int)sizeof(ST));
          km4[gi] = lds128(slot + C::OFF_KM + (gi * D + ch) * (int)sizeof(ST));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int gi = (G >= NT) ? 0 : (16 * j) / G;
        const uint32_t s0 = (kk & 1) ? ks4[gi].z : ks4[gi].x, s1 = (kk & 1) ? ks4[gi].w : ks4[gi].y;
        const uint32_t m0 = (kk & 1) ? km4[gi].z : km4[gi].x, m1 = (kk & 1) ? km4[gi].w : km4[gi].y;
        const int wr = (KB == 2) ? j : 2 * j + ((r & 3) >> 1);
        const uint4 w = lds128(slot + C::OFF_KC + (wr * D + ch) * 4);
        uint32_t a[4];
        if constexpr (KB == 2) {
          const uint32_t z0 = prmt(w.x, w.y, sel_lo) >> sh_lo, z1 = prmt(w.z, w.w, sel_lo) >> sh_lo;
          a[0] = bf16x2_dequant((z0 & 0x00030003u) | 0x43004300u, 0xC300C300u, s0, m0);
          a[1] = bf16x2_dequant((z0 & 0x000C000Cu) | 0x42004200u, 0xC200C200u, s0, m0);
          a[2] = bf16x2_dequant((z1 & 0x00030003u) | 0x43004300u, 0xC300C300u, s1, m1);
          a[3] = bf16x2_dequant((z1 & 0x000C000Cu) | 0x42004200u, 0xC200C200u, s1, m1);
        } else {
          const uint32_t y0l = prmt(w.x, w.y, sel_lo), y1l = prmt(w.z, w.w, sel_lo);
          const uint32_t y0h = prmt(w.x, w.y, sel_hi), y1h = prmt(w.z, w.w, sel_hi);
          a[0] = bf16x2_dequant(((y0l >> sh_lo) & 0x000F000Fu) | 0x43004300u, 0xC300C300u, s0, m0);
          a[1] = bf16x2_dequant(((y0h >> sh_hi) & 0x000F000Fu) | 0x43004300u, 0xC300C300u, s0, m0);
          a[2] = bf16x2_dequant(((y1l >> sh_lo) & 0x000F000Fu) | 0x43004300u, 0xC300C300u, s1, m1);
          a[3] = bf16x2_dequant(((y1h >> sh_hi) & 0x000F000Fu) | 0x43004300u, 0xC300C300u, s1, m1);
        }
        mma_bf16(acc[j], a, qbp[kk][0], qbp[kk][1]);
      }
    }
    float lg[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool vlo = FULL || 16 * j + tok_lo < n_valid, vhi = FULL || 16 * j + tok_hi < n_valid;
      lg[j][0] = vlo ? acc[j][0] : -INFINITY;
      lg[j][1] = vlo ? acc[j][1] : -INFINITY;
      lg[j][2] = vhi ? acc[j][2] : -INFINITY;
      lg[j][3] = vhi ? acc[j][3] : -INFINITY;
    }

    float alpha0, alpha1;
    if (softmax_update<4>(lg, scale_log2, st, alpha0, alpha1)) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= alpha0;
        o[i][1] *= alpha1;
        o[i][2] *= alpha0;
        o[i][3] *= alpha1;
      }
      accm[0] *= alpha0;
      accm[1] *= alpha1;
    }

    // Values.  Per stage the warp turns the value statistics into two small
    // fp16 tables in the (now free) key-code area: SD[t][g] = (s, s) for the
    // probability scaling, and MT[j][g][c] = the A fragment (minima of the
    // lane's four k-tokens) of the minimum term, which then runs as one MMA
    // per 16-token tile: sum_t p_th m_tg.  Tokens past the end get zeros.
    __syncwarp();
    unsigned char* sd_tab = const_cast<unsigned char*>(slot) + C::OFF_KC;
    unsigned char* mt_tab = sd_tab + NT * C::NG * 4;
    {
      uint32_t sw[C::NG];
      const unsigned char* src = slot + C::OFF_VS + 2 * lane * C::NG * (int)sizeof(ST);
      if constexpr (C::NG == 4) {
        const uint4 v = lds128(src);
        sw[0] = v.x; sw[1] = v.y; sw[2] = v.z; sw[3] = v.w;
      } else if constexpr (C::NG == 2) {
        const uint2 v = lds64(src);
        sw[0] = v.x; sw[1] = v.y;
      } else {
        sw[0] = *reinterpret_cast<const uint32_t*>(src);
      }
      uint32_t dup[2 * C::NG];
#pragma unroll
      for (int k = 0; k < 2 * C::NG; ++k) {
        const float f = (k & 1) ? bf16hi(sw[k >> 1]) : bf16lo(sw[k >> 1]);
        const bool valid = FULL || 2 * lane + k / C::NG < n_valid;
        dup[k] = valid ? pack_f16x2(f, f) : 0u;
      }
      uint32_t* dst = reinterpret_cast<uint32_t*>(sd_tab) + 2 * lane * C::NG;
#pragma unroll
      for (int k = 0; k < 2 * C::NG; k += 4 < 2 * C::NG ? 4 : 2 * C::NG) {
        if constexpr (2 * C::NG >= 4)
          *reinterpret_cast<uint4*>(dst + k) = make_uint4(dup[k], dup[k + 1], dup[k + 2], dup[k + 3]);
        else
          *reinterpret_cast<uint2*>(dst + k) = make_uint2(dup[k], dup[k + 1]);
      }
    }
#pragma unroll
    for (int e0 = 0; e0 < 16 * C::NG; e0 += 32) {
      const int e = e0 + lane;
      if (16 * C::NG >= 32 || e < 16 * C::NG) {
        const int jj = e / (4 * C::NG), g = (e >> 2) & (C::NG - 1), cc = e & 3;
        const int tk[4] = {16 * jj + tile_tok(2 * cc), 16 * jj + tile_tok(2 * cc + 1), 16 * jj + tile_tok(2 * cc + 8),
                           16 * jj + tile_tok(2 * cc + 9)};
        float mv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint16_t raw = *reinterpret_cast<const uint16_t*>(slot + C::OFF_VM + (tk[q] * C::NG + g) * 2);
          mv[q] = (FULL || tk[q] < n_valid) ? bf16lo(raw) : 0.f;
        }
        *reinterpret_cast<uint2*>(mt_tab + e * 8) = make_uint2(pack_f16x2(mv[0], mv[1]), pack_f16x2(mv[2], mv[3]));
      }
    }
    fence_proxy_async_smem();  // the slot's next bulk copy overwrites these tables
    __syncwarp();
    const int u0 = tile_tok(2 * c), u1 = tile_tok(2 * c + 1), u2 = tile_tok(2 * c + 8), u3 = tile_tok(2 * c + 9);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t p_lo = pack_f16x2(lg[j][0], lg[j][1]), p_hi = pack_f16x2(lg[j][2], lg[j][3]);
      {
        const uint2 am = lds64(mt_tab + ((j * C::NG + (r & (C::NG - 1))) * 4 + c) * 8);
        const uint32_t aa[4] = {am.x, am.x, am.y, am.y};  // rows >= NG are don't-care
        mma_f16(accm, aa, movmatrix_trans(p_lo), movmatrix_trans(p_hi));
      }
      uint32_t sl[C::NG], sh[C::NG];
      {
        const unsigned char* rl = sd_tab + (16 * j + tok_lo) * C::NG * 4;
        const unsigned char* rh = sd_tab + (16 * j + tok_hi) * C::NG * 4;
        if constexpr (C::NG == 4) {
          const uint4 x = lds128(rl), y = lds128(rh);
          sl[0] = x.x; sl[1] = x.y; sl[2] = x.z; sl[3] = x.w;
          sh[0] = y.x; sh[1] = y.y; sh[2] = y.z; sh[3] = y.w;
        } else if constexpr (C::NG == 2) {
          const uint2 x = lds64(rl), y = lds64(rh);
          sl[0] = x.x; sl[1] = x.y;
          sh[0] = y.x; sh[1] = y.y;
        } else {
          sl[0] = *reinterpret_cast<const uint32_t*>(rl);
          sh[0] = *reinterpret_cast<const uint32_t*>(rh);
        }
      }
      uint32_t bp[C::NG][2];
#pragma unroll
      for (int g = 0; g < C::NG; ++g) {
        bp[g][0] = movmatrix_trans(hmul2_f16(p_lo, sl[g]));
        bp[g][1] = movmatrix_trans(hmul2_f16(p_hi, sh[g]));
      }
      if constexpr (VB == 2) {
        constexpr int ROW = D * 2 / 8;  // bytes per token
        const unsigned char* vc = slot + C::OFF_VC + 16 * j * ROW;
        const uint4 w0a = lds128(vc + u0 * ROW), w0b = lds128(vc + u0 * ROW + 16);
        const uint4 w1a = lds128(vc + u1 * ROW), w1b = lds128(vc + u1 * ROW + 16);
        const uint4 w2a = lds128(vc + u2 * ROW), w2b = lds128(vc + u2 * ROW + 16);
        const uint4 w3a = lds128(vc + u3 * ROW), w3b = lds128(vc + u3 * ROW + 16);
        const uint32_t W0[8] = {w0a.x, w0a.y, w0a.z, w0a.w, w0b.x, w0b.y, w0b.z, w0b.w};
        const uint32_t W1[8] = {w1a.x, w1a.y, w1a.z, w1a.w, w1b.x, w1b.y, w1b.z, w1b.w};
        const uint32_t W2[8] = {w2a.x, w2a.y, w2a.z, w2a.w, w2b.x, w2b.y, w2b.z, w2b.w};
        const uint32_t W3[8] = {w3a.x, w3a.y, w3a.z, w3a.w, w3b.x, w3b.y, w3b.z, w3b.w};
        const uint32_t sel = (r >> 1) | ((4 + (r >> 1)) << 8);
        const uint32_t mvlo = 0x00030003u << (4 * (r & 1)), mvhi = 0x000C000Cu << (4 * (r & 1));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t y01 = prmt(W0[i], W1[i], sel), y23 = prmt(W2[i], W3[i], sel);
          const uint32_t a[4] = {y01 & mvlo, y01 & mvhi, y23 & mvlo, y23 & mvhi};
          const int g = (16 * i) / G;
          mma_f16(o[i], a, bp[g][0], bp[g][1]);
        }
      } else {
        constexpr int ROW = D * 4 / 8;
        const unsigned char* vc = slot + C::OFF_VC + 16 * j * ROW;
        const uint32_t sel = (r >> 1) | ((4 + (r >> 1)) << 8);
        const uint32_t m4 = 0x000F000Fu << (4 * (r & 1));
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t W[4][8];
          const int us[4] = {u0, u1, u2, u3};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 a0 = lds128(vc + us[u] * ROW + half * 32);
            const uint4 a1 = lds128(vc + us[u] * ROW + half * 32 + 16);
            W[u][0] = a0.x; W[u][1] = a0.y; W[u][2] = a0.z; W[u][3] = a0.w;
            W[u][4] = a1.x; W[u][5] = a1.y; W[u][6] = a1.z; W[u][7] = a1.w;
          }
#pragma unroll
          for (int ii = 0; ii < 4; ++ii) {
            const int i = half * 4 + ii;
            const uint32_t a[4] = {prmt(W[0][2 * ii], W[1][2 * ii], sel) & m4,
                                   prmt(W[0][2 * ii + 1], W[1][2 * ii + 1], sel) & m4,
                                   prmt(W[2][2 * ii], W[3][2 * ii], sel) & m4,
                                   prmt(W[2][2 * ii + 1], W[3][2 * ii + 1], sel) & m4};
            const int g = (16 * i) / G;
            mma_f16(o[i], a, bp[g][0], bp[g][1]);
          }
        }
      }
    }
  }

  // -------------------------------------------------------------- dense stage
  // 8 tokens of bf16 rows; MMA rows beyond them read a shared zero row.
  __device__ static void dense_stage(const unsigned char* slot, int n_valid, int lane, const unsigned char* qrow_smem,
                                     uint32_t zero_row, float scale_log2, WarpState& st, float (&o)[8][4]) {
    const int r = lane >> 2, c = lane & 3;
    const int pr = tile_pos(r), pr2 = (pr + 1) & 3;
    const int tok_lo = 4 * (r & 3) + pr, tok_hi = 4 * (r & 3) + pr2;
    const uint32_t kbase = smem_u32(slot), vbase = smem_u32(slot + DT * DROW);
    const int q = lane >> 3, krow = lane & 7;
    const int tk = tile_tok((q & 1) * 8 + krow), tv = tile_tok((q >> 1) * 8 + krow);
    const uint32_t kaddr = (tk < n_valid ? kbase + tk * DROW : zero_row) + (q >> 1) * 16;
    const uint32_t vaddr = (tv < n_valid ? vbase + tv * DROW : zero_row) + (q & 1) * 16;
    const unsigned char* qh = qrow_smem + r * D * 2;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < KCH; ++kk) {
      uint32_t a[4];
      ldmatrix_x4(a, kaddr + kk * 32);
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(qh + (16 * kk + 2 * c) * 2);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(qh + (16 * kk + 2 * c + 8) * 2);
      mma_bf16(acc, a, b0, b1);
    }
    float lg[1][4];
    lg[0][0] = tok_lo < n_valid ? acc[0] : -INFINITY;
    lg[0][1] = tok_lo < n_valid ? acc[1] : -INFINITY;
    lg[0][2] = tok_hi < n_valid ? acc[2] : -INFINITY;
    lg[0][3] = tok_hi < n_valid ? acc[3] : -INFINITY;
    float alpha0, alpha1;
    if (softmax_update<1>(lg, scale_log2, st, alpha0, alpha1)) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= alpha0;
        o[i][1] *= alpha1;
        o[i][2] *= alpha0;
        o[i][3] *= alpha1;
      }
    }
    const uint32_t b0 = movmatrix_trans(pack_bf16x2(lg[0][0], lg[0][1]));
    const uint32_t b1 = movmatrix_trans(pack_bf16x2(lg[0][2], lg[0][3]));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t a[4];
      ldmatrix_x4_trans(a, vaddr + i * 32);
      mma_bf16(o[i], a, b0, b1);
    }
  }

  // -------------------------------------------------------------- write a warp state
  // Stores (max, sum, out) of the warp's current segment, in natural channel
  // order, into a private shared-memory block [m 8][l 8][O 8 x D].
  __device__ static void store_state(float* dst, bool packed, const WarpState& st, float (&o)[8][4],
                                     const float (&accm)[4], int lane) {
    const int r = lane >> 2, c = lane & 3;
    const float l0 = warp_sum_r(st.lrun[0]), l1 = warp_sum_r(st.lrun[1]);
    // Minimum-term sums: group g, heads 2c and 2c+1 live in lane 4g + c.
    float mg0[C::NG], mg1[C::NG];
#pragma unroll
    for (int g = 0; g < C::NG; ++g) {
      mg0[g] = __shfl_sync(0xffffffffu, accm[0], 4 * g + c);
      mg1[g] = __shfl_sync(0xffffffffu, accm[1], 4 * g + c);
    }
    if (r == 0) {
      dst[2 * c] = st.mrun[0];
      dst[2 * c + 1] = st.mrun[1];
      dst[8 + 2 * c] = l0;
      dst[8 + 2 * c + 1] = l1;
    }
    float* ao = dst + 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int d_lo, d_hi;
      float v[4];
      if (packed) {
        float f_lo, f_hi;
        if constexpr (VB == 2) {
          d_lo = 16 * i + 2 * r;
          d_hi = d_lo + 1;
          f_lo = __int_as_float((127 + 24 - 4 * (r & 1)) << 23);
          f_hi = __int_as_float((127 + 22 - 4 * (r & 1)) << 23);
        } else {
          d_lo = 16 * i + r;
          d_hi = d_lo + 8;
          f_lo = f_hi = __int_as_float((127 + 24 - 4 * (r & 1)) << 23);
        }
        const int g = (16 * i) / G;
        v[0] = fmaf(o[i][0], f_lo, mg0[g]);
        v[1] = fmaf(o[i][1], f_lo, mg1[g]);
        v[2] = fmaf(o[i][2], f_hi, mg0[g]);
        v[3] = fmaf(o[i][3], f_hi, mg1[g]);
      } else {
        d_lo = 16 * i + r;
        d_hi = d_lo + 8;
        v[0] = o[i][0];
        v[1] = o[i][1];
        v[2] = o[i][2];
        v[3] = o[i][3];
      }
      ao[(2 * c) * D + d_lo] = v[0];
      ao[(2 * c + 1) * D + d_lo] = v[1];
      ao[(2 * c) * D + d_hi] = v[2];
      ao[(2 * c + 1) * D + d_hi] = v[3];
    }
  }

  // -------------------------------------------------------------- kernel body
  __device__ static void run(const Params& P, unsigned char* smem) {
    const uint64_t t_start = P.trace ? global_timer_ns() : 0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = lane >> 2, c = lane & 3;
    const ucb_decode_cta cta = P.ctas[blockIdx.x];
    const int32_t* bounds = P.warp_bounds + (int64_t)blockIdx.x * (C::WARPS + 1);
    const int u_begin = bounds[warp], u_end = bounds[warp + 1];

    const int2 wslot = reinterpret_cast<const int2*>(P.warp_slots)[blockIdx.x * C::WARPS + warp];
    unsigned char* qs = smem + C::OFF_Q;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR) + warp * 2;
    const uint32_t zero_row = smem_u32(smem + C::OFF_ZERO);
    unsigned char* ring = smem + warp * 2 * C::SLOT;

    // ---- CTA set-up: query rows of its pairs, zero row, barriers.
    for (int i = tid; i < MAXC * 8 * D / 8; i += C::THREADS) {  // 16-byte chunks
      const int pl = i / (8 * D / 8), rem = i % (8 * D / 8);
      const int h = rem / (D / 8), chunk = rem % (D / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (pl < cta.num_pairs && h < P.grp) {
        const ucb_decode_pair pr = P.pairs[cta.pair_begin + pl];
        const __nv_bfloat16* src = P.query + pr.seq * P.query_stride + (int64_t)(pr.kv_head * P.grp + h) * D;
        v = reinterpret_cast<const uint4*>(src)[chunk];
      }
      reinterpret_cast<uint4*>(qs)[i] = v;
    }
    for (int i = tid; i < D * 2 / 16; i += C::THREADS)
      reinterpret_cast<uint4*>(smem + C::OFF_ZERO)[i] = make_uint4(0, 0, 0, 0);
    ucb_span* spans = reinterpret_cast<ucb_span*>(smem + C::OFF_SPANS);
    const int n_spans = cta.reserved[0] - cta.span_begin;  // spans [span_begin, span_end)
    for (int i = tid; i < n_spans * (int)(sizeof(ucb_span) / 8); i += C::THREADS)
      reinterpret_cast<uint64_t*>(spans)[i] = reinterpret_cast<const uint64_t*>(P.spans + cta.span_begin)[i];
    if (lane == 0) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
      fence_mbarrier_init();
    }
    __syncthreads();
    // growing suffixes: the live length, read once per launch
    if (tid < n_spans) {
      const ucb_span& g = P.spans[cta.span_begin + tid];
      if (g.kind == 1 && g.key_scale != nullptr)
        spans[tid].tokens = max(0, min(g.tokens, *static_cast<const volatile int32_t*>(g.key_scale)));
    }
    __syncthreads();

    // ---- the warp's units, in order; an issue cursor runs two units ahead.
    int issue_u = u_begin, issue_span = 0;
    auto issue_next = [&](int slot_idx) {
      while (issue_span + 1 < n_spans && spans[issue_span + 1].unit_begin <= issue_u) ++issue_span;
      const ucb_span& sp = spans[issue_span];
      const int stage = sp.kind == 0 ? NT : DT;
      const int t0 = (issue_u - sp.unit_begin) * stage;
      const int t1 = min(live_tokens(sp), t0 + stage);
      unsigned char* slot = ring + slot_idx * C::SLOT;
      if (sp.kind == 0)
        issue_packed(sp, t0, t1, slot, &bars[slot_idx], lane);
      else
        issue_dense(sp, t0, t1, slot, &bars[slot_idx], lane);
      ++issue_u;
    };
    if (issue_u < u_end) issue_next(0);
    if (issue_u < u_end) issue_next(1);

    WarpState st;
    st.mrun[0] = st.mrun[1] = -INFINITY;
    st.lrun[0] = st.lrun[1] = 0.f;
    float o[8][4];
    float accm[4];
    uint32_t qbp[KCH][2];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) accm[g] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KCH; ++kk) qbp[kk][0] = qbp[kk][1] = 0u;
    int cur_pl = -1, cur_kind = -1, span = 0;
    bool ok = true, stashed = false;
    int s = 0;
    uint64_t waited = 0;  // diagnostics: time blocked on this warp's copies
    for (int u = u_begin; u < u_end; ++u, ++s) {
      const int slot_idx = s & 1;
      const uint64_t w0 = P.trace ? global_timer_ns() : 0;
      if (!mbar_wait_bounded(&bars[slot_idx], (s >> 1) & 1, WAIT_LIMIT)) {
        ok = false;
        break;
      }
      if (P.trace) waited += global_timer_ns() - w0;
      while (span + 1 < n_spans && spans[span + 1].unit_begin <= u) ++span;
      const ucb_span& sp = spans[span];
      const int pl = sp.pair - cta.pair_begin;
      const int kind = sp.kind;
      if (pl != cur_pl || kind != cur_kind) {
        if (cur_pl >= 0) {
          // At most one segment boundary per warp (the planner guarantees it).
          if (stashed || wslot.x < 0 || wslot.x >= P.max_partials) {
            atomicOr(P.err, DEVERR_BAD_DESCRIPTOR);
          } else {
            store_state(P.partials + (int64_t)wslot.x * PARTIAL_FLOATS, cur_kind == 0, st, o, accm, lane);
          }
          stashed = true;
        }
        st.mrun[0] = st.mrun[1] = -INFINITY;
        st.lrun[0] = st.lrun[1] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
        for (int g = 0; g < 4; ++g) accm[g] = 0.f;
        if (kind == 0) {
#pragma unroll
          for (int kk = 0; kk < KCH; ++kk) {
            const uint2 q2 = lds64(qs + ((pl * 8 + r) * D + 32 * (kk >> 1) + 8 * c + 4 * (kk & 1)) * 2);
            qbp[kk][0] = q2.x;
            qbp[kk][1] = q2.y;
          }
        }
        cur_pl = pl;
        cur_kind = kind;
      }
      unsigned char* slot = ring + slot_idx * C::SLOT;
      const int stage = kind == 0 ? NT : DT;
      const int t0 = (u - sp.unit_begin) * stage;
      const int n = min(live_tokens(sp), t0 + stage) - t0;
      if (kind == 0) {
        if (n == NT)
          packed_stage<true>(slot, n, lane, qbp, P.scale_log2, st, o, accm);
        else
          packed_stage<false>(slot, n, lane, qbp, P.scale_log2, st, o, accm);
      } else if (n > 0) {
        dense_stage(slot, n, lane, qs + pl * 8 * D * 2, zero_row, P.scale_log2, st, o);
      }
      __syncwarp();
      if (issue_u < u_end) issue_next(slot_idx);
    }
    if (!ok) {
      // Let copies still in flight land before the shared memory is released.
      for (int k = s; k < s + 2; ++k) {
        if (u_begin + k < u_end) mbar_wait_bounded(&bars[k & 1], (k >> 1) & 1, WAIT_LIMIT);
      }
      if (lane == 0) atomicOr(P.err, DEVERR_MBAR_TIMEOUT);
    } else if (cur_pl >= 0) {
      if (wslot.y < 0 || wslot.y >= P.max_partials)
        atomicOr(P.err, DEVERR_BAD_DESCRIPTOR);
      else
        store_state(P.partials + (int64_t)wslot.y * PARTIAL_FLOATS, cur_kind == 0, st, o, accm, lane);
    }
    if (P.trace && lane == 0) {
      uint64_t* tr = P.trace + 32 * blockIdx.x;
      static_assert(C::WARPS <= 12, "the trace record holds 12 warps");
      tr[6 + warp] = global_timer_ns();
      tr[18 + warp] = waited;
      if (warp == 0) {
        tr[0] = t_start;
        tr[4] = sm_id();
      }
    }
  }
};

template <int KB, int VB, int G, typename ST>
__global__ void __launch_bounds__(Cfg<KB, VB, G, ST>::THREADS, 1) decode_kernel(Params P) {
  extern __shared__ __align__(128) unsigned char smem[];
  Kernel<KB, VB, G, ST>::run(P, smem);
}

// ---------------------------------------------------------------- state merge
// One CTA per (pair, 32-channel chunk), warp h = query head h of the pair.  In
// rounds of 32 states, lane k loads state k's (max, sum) for head h and every
// lane loads its channel of all 32 rows, all in one batch; the round's weights
// exp2(m_k - M) reach the lanes by shuffles.  Output out[seq, kv*grp + h, d]
// in bf16 and, for d == 0, the natural-log LSE.  No shared memory, no CTA
// barrier: each warp is independent.
constexpr int MERGE_DCH = 32;

// One round of the merge: up to 32 states starting at `st` folded into the
// running (M, L, acc) of query head h, channel d (this lane).  Lane k loads
// state k's (max, sum); every lane loads its channel of all rows in one batch.
__device__ __forceinline__ void merge_round(const float* st, int nk, int h, int d, int lane, float& M, float& L,
                                            float& acc) {
  const float mk = lane < nk ? __ldcg(st + (int64_t)lane * PARTIAL_FLOATS + h) : -INFINITY;
  const float lk = lane < nk ? __ldcg(st + (int64_t)lane * PARTIAL_FLOATS + 8 + h) : 0.f;
  float v[32];
#pragma unroll
  for (int q = 0; q < 32; ++q) v[q] = q < nk ? __ldcg(st + (int64_t)q * PARTIAL_FLOATS + 16 + h * D + d) : 0.f;
  float mx = mk;
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float m_new = fmaxf(M, mx);
  if (m_new == -INFINITY) return;  // nothing seen yet (empty states)
  const float wk = (mk == -INFINITY) ? 0.f : fast_exp2(mk - m_new);
  float l = wk * lk;
#pragma unroll
  for (int off = 16; off; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  const float f = (M == -INFINITY) ? 0.f : fast_exp2(M - m_new);
  float a0 = acc * f, a1 = 0.f;
#pragma unroll
  for (int q = 0; q < 32; q += 2) {
    a0 = fmaf(__shfl_sync(0xffffffffu, wk, q), v[q], a0);
    a1 = fmaf(__shfl_sync(0xffffffffu, wk, q + 1), v[q + 1], a1);
  }
  acc = a0 + a1;
  L = fmaf(L, f, l);
  M = m_new;
}

__device__ __forceinline__ void merge_store(const ucb_decode_pair& pr, int grp, int hq, int h, int d, float M, float L,
                                            float acc, __nv_bfloat16* out, int64_t out_stride, float* lse) {
  const int qh = pr.kv_head * grp + h;
  out[pr.seq * out_stride + (int64_t)qh * D + d] = __float2bfloat16_rn(acc / L);
  if (d == 0 && lse != nullptr) lse[(int64_t)pr.seq * hq + qh] = (M + __log2f(L)) * LN2;
}

// Few states per pair (many pairs): CTA per (pair, 32-channel chunk), warp h =
// query head h walks all the pair's states.
// A pair whose slot range does not lie inside [0, max_partials) is a bad
// descriptor: it sets the error word and writes nothing.
__device__ __forceinline__ bool slots_in_range(const ucb_decode_pair& pr, int max_partials, unsigned int* err) {
  if (pr.partial_begin >= 0 && pr.partial_count >= 0 && pr.partial_count <= max_partials - pr.partial_begin)
    return true;
  if (threadIdx.x == 0) atomicOr(err, DEVERR_BAD_DESCRIPTOR);
  return false;
}

__global__ void __launch_bounds__(256) state_merge_kernel(const float* __restrict__ states,
                                                          const ucb_decode_pair* __restrict__ pairs, int grp,
                                                          int hq, __nv_bfloat16* __restrict__ out, int64_t out_stride,
                                                          float* __restrict__ lse, int max_partials,
                                                          unsigned int* err) {
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31, d = blockIdx.y * MERGE_DCH + lane;
  const ucb_decode_pair pr = pairs[blockIdx.x];
  if (!slots_in_range(pr, max_partials, err) || h >= grp) return;
  const float* base = states + (int64_t)pr.partial_begin * PARTIAL_FLOATS;
  float M = -INFINITY, L = 0.f, acc = 0.f;
  for (int k0 = 0; k0 < pr.partial_count; k0 += 32)
    merge_round(base + (int64_t)k0 * PARTIAL_FLOATS, min(32, pr.partial_count - k0), h, d, lane, M, L, acc);
  merge_store(pr, grp, hq, h, d, M, L, acc, out, out_stride, lse);
}

// Many states per pair (few long sequences): CTA per (pair, query head,
// 32-channel chunk); its 8 warps take every 8th block of 32 states and fold
// their partial results through shared memory.
constexpr int WIDE_MERGE_WARPS = 8;
__global__ void __launch_bounds__(WIDE_MERGE_WARPS * 32)
    state_merge_wide_kernel(const float* __restrict__ states, const ucb_decode_pair* __restrict__ pairs, int grp,
                            int hq, __nv_bfloat16* __restrict__ out, int64_t out_stride, float* __restrict__ lse,
                            int max_partials, unsigned int* err) {
  __shared__ float sm_m[WIDE_MERGE_WARPS], sm_l[WIDE_MERGE_WARPS], sm_acc[WIDE_MERGE_WARPS][32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, d = blockIdx.y * MERGE_DCH + lane;
  const int pi = blockIdx.x / grp, h = blockIdx.x % grp;
  const ucb_decode_pair pr = pairs[pi];
  if (!slots_in_range(pr, max_partials, err)) return;  // uniform over the CTA: no barrier is skipped by part of it
  const float* base = states + (int64_t)pr.partial_begin * PARTIAL_FLOATS;
  float M = -INFINITY, L = 0.f, acc = 0.f;
  for (int k0 = 32 * w; k0 < pr.partial_count; k0 += 32 * WIDE_MERGE_WARPS)
    merge_round(base + (int64_t)k0 * PARTIAL_FLOATS, min(32, pr.partial_count - k0), h, d, lane, M, L, acc);
  if (lane == 0) {
    sm_m[w] = M;
    sm_l[w] = L;
  }
  sm_acc[w][lane] = acc;
  __syncthreads();
  if (w != 0) return;
  float Mt = -INFINITY;
#pragma unroll
  for (int k = 0; k < WIDE_MERGE_WARPS; ++k) Mt = fmaxf(Mt, sm_m[k]);
  float Lt = 0.f, At = 0.f;
#pragma unroll
  for (int k = 0; k < WIDE_MERGE_WARPS; ++k) {
    const float f = (sm_m[k] == -INFINITY) ? 0.f : fast_exp2(sm_m[k] - Mt);
    Lt = fmaf(sm_l[k], f, Lt);
    At = fmaf(sm_acc[k][lane], f, At);
  }
  merge_store(pr, grp, hq, h, d, Mt, Lt, At, out, out_stride, lse);
}

template <int KB, int VB, int G, typename ST>
int configure() {
  using C = Cfg<KB, VB, G, ST>;
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return UCB_OK;
  if (cudaFuncSetAttribute(decode_kernel<KB, VB, G, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
      cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel: cannot reserve %d bytes of shared memory", C::SMEM);
  if (dev >= 0 && dev < 64) done[dev] = true;
  return UCB_OK;
}

template <int KB, int VB, int G, typename ST>
int launch(const Params& P, int num_ctas, cudaStream_t s) {
  using C = Cfg<KB, VB, G, ST>;
  int rc = configure<KB, VB, G, ST>();
  if (rc) return rc;
  decode_kernel<KB, VB, G, ST><<<num_ctas, C::THREADS, C::SMEM, s>>>(P);
  rc = ucb_host::check_launch("decode_kernel");
  if (rc) return rc;
  // Stream order makes the merge wait for every warp state.  (Launching it as
  // a programmatic dependent measured slower: 31.7 vs 29.0 us per config-2 step.)
  // Pairs hold about num_ctas * WARPS / num_pairs warp states each: above 64
  // the per-head walk over them gets long, so 8 warps share each head.
  if ((int64_t)num_ctas * C::WARPS > 64LL * P.num_pairs) {
    state_merge_wide_kernel<<<dim3(P.num_pairs * P.grp, D / MERGE_DCH), WIDE_MERGE_WARPS * 32, 0, s>>>(
        static_cast<const float*>(P.partials), P.pairs, P.grp, P.hq, P.out, P.out_stride, P.lse, P.max_partials,
        P.err);
    return ucb_host::check_launch("state_merge_wide_kernel");
  }
  state_merge_kernel<<<dim3(P.num_pairs, D / MERGE_DCH), 256, 0, s>>>(
      static_cast<const float*>(P.partials), P.pairs, P.grp, P.hq, P.out, P.out_stride, P.lse, P.max_partials,
      P.err);
  return ucb_host::check_launch("state_merge_kernel");
}

template <int KB, int VB, int G, typename ST>
int slots(int* out, int* warps) {
  using C = Cfg<KB, VB, G, ST>;
  int rc = configure<KB, VB, G, ST>();
  if (rc) return rc;
  *warps = C::WARPS;
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel<KB, VB, G, ST>, C::THREADS, C::SMEM) !=
          cudaSuccess ||
      cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel: occupancy query failed");
  if (per_sm < 1) return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel does not fit on an SM");
  *out = per_sm * sms;
  return UCB_OK;
}

template <template <int, int, int, typename> class Fn, typename... Args>
int dispatch(int kb, int vb, int g, Args... args) {
#define UCB_CASE(KB_, VB_, G_) \
  if (kb == KB_ && vb == VB_ && g == G_) return Fn<KB_, VB_, G_, __nv_bfloat16>::call(args...);
  UCB_CASE(2, 2, 32) UCB_CASE(2, 2, 64) UCB_CASE(2, 2, 128)
  UCB_CASE(4, 4, 32) UCB_CASE(4, 4, 64) UCB_CASE(4, 4, 128)
  UCB_CASE(2, 4, 32) UCB_CASE(2, 4, 64) UCB_CASE(2, 4, 128)
  UCB_CASE(4, 2, 32) UCB_CASE(4, 2, 64) UCB_CASE(4, 2, 128)
#undef UCB_CASE
  return ucb_host::set_error(UCB_ERR_UNSUPPORTED, "decode: unsupported (k_bits=%d, v_bits=%d, group=%d)", kb, vb, g);
}

template <int KB, int VB, int G, typename ST>
struct LaunchFn {
  static int call(const Params& P, int n, cudaStream_t s) { return launch<KB, VB, G, ST>(P, n, s); }
};
template <int KB, int VB, int G, typename ST>
struct SlotsFn {
  static int call(int* out, int* warps) { return slots<KB, VB, G, ST>(out, warps); }
};


}  // namespace decode
}  // namespace ucb

using ucb_host::set_error;

namespace {
uint64_t* g_decode_trace = nullptr;  // diagnostics only; see ucb_decode_set_trace
}

extern "C" int ucb_decode_set_trace(void* trace_dev) {
  g_decode_trace = static_cast<uint64_t*>(trace_dev);
  return UCB_OK;
}

extern "C" int64_t ucb_decode_partial_bytes(int head_dim) { return (int64_t)(16 + 8 * head_dim) * 4; }

extern "C" int ucb_decode_config(int k_bits, int v_bits, int group_size, int stat_dtype, int* ctas,
                                 int* warps_per_cta) {
  if (!ctas || !warps_per_cta) return set_error(UCB_ERR_INVALID, "ucb_decode_config: null output");
  if (stat_dtype != UCB_BF16) return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_config: bf16 statistics only");
  return ucb::decode::dispatch<ucb::decode::SlotsFn>(k_bits, v_bits, group_size, ctas, warps_per_cta);
}

namespace {
// Shared body of the two decode entry points.  max_partials bounds every slot
// index the kernels may touch (the allocating entry trusts the plan and passes
// INT32_MAX; the allocation-free one passes the static array's slot count).
int decode_attention_impl(const void* query, int64_t query_stride, int num_q_heads, int num_kv_heads, int head_dim,
                          const ucb_span* spans, int num_spans, const ucb_decode_cta* ctas, int num_ctas,
                          const int32_t* warp_bounds, const ucb_decode_pair* pairs, int num_pairs, int k_bits,
                          int v_bits, int group_size, int stat_dtype, float softmax_scale, void* partials,
                          int max_partials, const int32_t* warp_slots, void* out, int64_t out_stride, float* lse,
                          void* stream) {
  if (!query || !spans || !ctas || !warp_bounds || !pairs || !partials || !warp_slots || !out)
    return set_error(UCB_ERR_INVALID, "ucb_decode_attention: null pointer");
  if (head_dim != 128) return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: head_dim must be 128");
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > 8)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: need q_heads/kv_heads in [1, 8]");
  if (stat_dtype != UCB_BF16)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: packed statistics must be bf16");
  if (num_ctas <= 0 || num_pairs <= 0 || num_spans <= 0)
    return set_error(UCB_ERR_INVALID, "ucb_decode_attention: empty batch");
  if (query_stride % 8 || out_stride % 8 || (reinterpret_cast<uintptr_t>(query) & 15))
    return set_error(UCB_ERR_INVALID, "ucb_decode_attention: query/out rows must be 16-byte aligned");
  unsigned int* err = ucb_host::device_error_word();
  if (!err) return set_error(UCB_ERR_CUDA, "ucb_decode_attention: device error word unavailable");
  ucb::decode::Params P;
  P.query = static_cast<const __nv_bfloat16*>(query);
  P.query_stride = query_stride;
  P.grp = num_q_heads / num_kv_heads;
  P.hq = num_q_heads;
  P.spans = spans;
  P.num_spans = num_spans;
  P.ctas = ctas;
  P.warp_bounds = warp_bounds;
  P.pairs = pairs;
  P.num_pairs = num_pairs;
  P.scale_log2 = softmax_scale * ucb::decode::LOG2E;
  P.partials = static_cast<float*>(partials);
  P.max_partials = max_partials;
  P.warp_slots = warp_slots;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.out_stride = out_stride;
  P.lse = lse;
  P.err = err;
  P.trace = g_decode_trace;
  return ucb::decode::dispatch<ucb::decode::LaunchFn>(k_bits, v_bits, group_size, P, num_ctas,
                                                      static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" int ucb_decode_attention(const void* query, int64_t query_stride, int num_q_heads, int num_kv_heads,
                                    int head_dim, const ucb_span* spans, int num_spans, const ucb_decode_cta* ctas,
                                    int num_ctas, const int32_t* warp_bounds, const ucb_decode_pair* pairs,
                                    int num_pairs, int k_bits, int v_bits,
                                    int group_size, int stat_dtype, float softmax_scale, void* partials,
                                    const int32_t* warp_slots, void* out, int64_t out_stride, float* lse,
                                    void* stream) {
  return decode_attention_impl(query, query_stride, num_q_heads, num_kv_heads, head_dim, spans, num_spans, ctas,
                               num_ctas, warp_bounds, pairs, num_pairs, k_bits, v_bits, group_size, stat_dtype,
                               softmax_scale, partials, INT32_MAX, warp_slots, out, out_stride, lse, stream);
}

// ----------------------------------------------------- allocation-free decode
// Some callers cannot allocate device memory at the time they decode: an
// engine that hands the whole HBM pool to its own allocator up front, code
// running while a CUDA graph is being captured by someone else, or a plugin
// host that forbids the library from calling cudaMalloc.  For them the
// warp-state slots live in one statically sized device array that
// the library module carries on every GPU it is loaded on, until exit.
namespace {
constexpr int NOALLOC_MAX_PARTIALS = 512;  // warp-state slots (sum of partial_count)
constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)NOALLOC_MAX_PARTIALS * ucb::decode::PARTIAL_FLOATS * sizeof(float);

// Host code must not use this name as a pointer: it is only a handle from which
// cudaGetSymbolAddress returns the array's address on the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device, looked up once
// per device (the first call on a device does this set-up).
int noalloc_scratch(unsigned char** ptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(UCB_ERR_CUDA, "ucb_decode_attention_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(UCB_ERR_CUDA, "ucb_decode_attention_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *ptr = static_cast<unsigned char*>(g_noalloc_ptr[dev]);
  return UCB_OK;
}
}  // namespace

extern "C" int ucb_decode_attention_noalloc(const void* query, int64_t query_stride, int num_q_heads,
                                            int num_kv_heads, int head_dim, const ucb_span* spans, int num_spans,
                                            const ucb_decode_cta* ctas, int num_ctas, const int32_t* warp_bounds,
                                            const ucb_decode_pair* pairs, int num_pairs,
                                            const int32_t* warp_slots, int num_partials, int k_bits, int v_bits,
                                            int group_size, int stat_dtype, float softmax_scale, void* out,
                                            int64_t out_stride, float* lse, void* stream) {
  if (num_partials <= 0 || num_partials > NOALLOC_MAX_PARTIALS)
    return set_error(UCB_ERR_INVALID,
                     "ucb_decode_attention_noalloc: the plan needs %d partial slots; the static scratch holds 1..%d",
                     num_partials, NOALLOC_MAX_PARTIALS);
  unsigned char* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != UCB_OK) return rc;
  // Slot indices come from device tables the library cannot read on the host,
  // so the kernels check each one against the array's size (a bad index sets
  // DEVERR_BAD_DESCRIPTOR and writes nothing).
  return decode_attention_impl(query, query_stride, num_q_heads, num_kv_heads, head_dim, spans, num_spans, ctas,
                               num_ctas, warp_bounds, pairs, num_pairs, k_bits, v_bits, group_size, stat_dtype,
                               softmax_scale, scratch, num_partials, warp_slots, out, out_stride, lse, stream);
}

