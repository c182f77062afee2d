// Single-token (decode) attention over packed KIVI and dense bf16 spans.
//
// Replaces, for q_len == 1: packed_kivi_attention_parts + softmax + apply_value
// (unicache/storage/kivi_cuda.py:238-329), the quantized-prefix summary
// (kivi_cuda.py:96-120) and the frozen-H2O concat path
// (unicache/adapters/bagel.py:1860-1901).
//
// Design (B200, HBM-bound):
//  * One CTA = one work item = a token range of one span of one (sequence,
//    KV head) pair; 4 warps split the range into contiguous runs of stages.
//  * Each warp streams its stages with the TMA bulk-copy engine
//    (cp.async.bulk, no tensor map, no multicast) into a private two-slot
//    shared-memory ring guarded by mbarriers; every wait is bounded.
//  * The 7 query heads of a GQA group are the N=8 columns of mma.sync
//    m16n8k16; 16 tokens (QK) or 16 channels (AV) are the M rows.  Packed
//    codes never become bf16 values: a PRMT + AND puts each 2/4-bit code into
//    an fp16 *subnormal* (code * 2^(p-24)) that the tensor core multiplies
//    exactly, and the group scales are folded into the other operand:
//       q.k_t  = sum_d (q_d s_gd) c_td + sum_d q_d m_gd          (keys, per channel)
//       sum_t p_t v_td = sum_t (p_t s_tg) c_td + sum_t p_t m_tg  (values, per token)
//    The per-row power of two (p) is undone on the fp32 accumulator.
//  * Online softmax in the log2 domain per warp; warps merge in shared
//    memory; CTAs write (max, sum, out) partials and the last CTA of a pair
//    (atomic ticket, no waiting) merges them into the output and the LSE.
#include <cfloat>

#include "common.cuh"

namespace ucb {
namespace decode {

constexpr int D = 128;
constexpr int KCH = D / 16;       // k-chunks of 16 channels
constexpr int WARPS = 4;
constexpr int NT = 64;            // tokens per packed stage
constexpr int DT = 16;            // tokens per dense stage
constexpr int DROW = 272;         // dense shared-memory row stride (bytes)
constexpr int DENSE_STAGE = 2 * DT * DROW;
constexpr uint32_t WAIT_LIMIT = 1u << 24;
constexpr int PARTIAL_FLOATS = 16 + 8 * D;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__host__ __device__ constexpr int round_up(int x, int a) { return (x + a - 1) / a * a; }

template <int KB, int VB, int G, typename ST>
struct Cfg {
  static constexpr int NG = D / G;                   // value groups per token
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
  static constexpr int WARP_SMEM = 2 * SLOT;
  static constexpr int SMEM = WARPS * WARP_SMEM + 128;  // + mbarriers and flags
  static_assert(WARP_SMEM >= PARTIAL_FLOATS * 4, "warp ring must hold a warp state");
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

// Online-softmax update for `NTILE` C fragments; returns the rescale factors.
template <int NTILE>
__device__ __forceinline__ void softmax_update(float (&lg)[NTILE][4], WarpState& st, float& alpha0,
                                               float& alpha1) {
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NTILE; ++j) {
    mx0 = fmaxf(mx0, fmaxf(lg[j][0], lg[j][2]));
    mx1 = fmaxf(mx1, fmaxf(lg[j][1], lg[j][3]));
  }
  mx0 = warp_max_r(mx0);
  mx1 = warp_max_r(mx1);
  const float n0 = fmaxf(st.mrun[0], mx0), n1 = fmaxf(st.mrun[1], mx1);
  alpha0 = fast_exp2(st.mrun[0] - n0);
  alpha1 = fast_exp2(st.mrun[1] - n1);
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int j = 0; j < NTILE; ++j) {
    lg[j][0] = fast_exp2(lg[j][0] - n0);
    lg[j][1] = fast_exp2(lg[j][1] - n1);
    lg[j][2] = fast_exp2(lg[j][2] - n0);
    lg[j][3] = fast_exp2(lg[j][3] - n1);
    s0 += lg[j][0] + lg[j][2];
    s1 += lg[j][1] + lg[j][3];
  }
  st.lrun[0] = st.lrun[0] * alpha0 + s0;
  st.lrun[1] = st.lrun[1] * alpha1 + s1;
  st.mrun[0] = n0;
  st.mrun[1] = n1;
}

__device__ __forceinline__ uint2 lds64(const unsigned char* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }

struct Params {
  const __nv_bfloat16* query;
  int64_t query_stride;
  int grp;  // query heads per KV head
  int hq;   // query heads per sequence (row length of lse)
  const ucb_span* spans;
  const ucb_decode_item* items;
  const ucb_decode_pair* pairs;
  float scale_log2;  // softmax_scale * log2(e)
  float* partials;
  int* counters;
  __nv_bfloat16* out;
  int64_t out_stride;
  float* lse;
  unsigned int* err;
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
    bulk_g2s(slot + C::OFF_KC, kcode, kc, bar);
    bulk_g2s(slot + C::OFF_VC, vcode, vc, bar);
    bulk_g2s(slot + C::OFF_KS, kscale, ks, bar);
    bulk_g2s(slot + C::OFF_KM, kmin, ks, bar);
    bulk_g2s(slot + C::OFF_VS, vscale, vs, bar);
    bulk_g2s(slot + C::OFF_VM, vmin, vs, bar);
  }

  __device__ static void issue_dense(const ucb_span& sp, int t0, int t1, unsigned char* slot, uint64_t* bar,
                                     int lane) {
    const int n = t1 - t0;
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, 2u * n * D * 2u);
    }
    __syncwarp();
    const int row = lane & 15;
    if (row < n) {
      const bool is_v = lane >= 16;
      const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(is_v ? sp.value_code : sp.key_code);
      const int64_t stride = is_v ? sp.value_stride : sp.key_stride;
      bulk_g2s(slot + (is_v ? DT * DROW : 0) + row * DROW, base + (t0 + row) * stride, D * 2, bar);
    }
  }

  // -------------------------------------------------------------- packed stage
  __device__ static void packed_stage(const unsigned char* slot, int n_valid, int lane, const float (&qf)[KCH][4],
                                      const uint32_t (&qbp)[KCH][2], float scale_log2, WarpState& st,
                                      float (&o)[8][4], float (&accm)[C::NG][2]) {
    const int r = lane >> 2, c = lane & 3;
    const int pr = tile_pos(r), pr2 = (pr + 1) & 3;
    const int tok_lo = 4 * (r & 3) + pr, tok_hi = 4 * (r & 3) + pr2;

    // Per-group key bias  sum_d q_d m_gd  for the groups of this stage (rows = groups).
    const int gps_valid = (G >= NT) ? 1 : (n_valid + G - 1) / G;
    float cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < KCH; ++kk) {
      uint32_t a[4] = {0u, 0u, 0u, 0u};
      if (r < gps_valid) {
        const uint2 m = lds64(slot + C::OFF_KM + (r * D + 16 * kk + 4 * c) * (int)sizeof(ST));
        a[0] = m.x;
        a[2] = m.y;
      }
      mma_bf16(cb, a, qbp[kk][0], qbp[kk][1]);
    }

    float lg[4][4];
#pragma unroll
    for (int gi = 0; gi < C::GPS; ++gi) {
      // q~ = q * key scale of this group, fp16, B-fragment order.
      uint32_t bq[KCH][2];
#pragma unroll
      for (int kk = 0; kk < KCH; ++kk) {
        const uint2 s = lds64(slot + C::OFF_KS + (gi * D + 16 * kk + 4 * c) * (int)sizeof(ST));
        bq[kk][0] = pack_f16x2(qf[kk][0] * bf16lo(s.x), qf[kk][1] * bf16hi(s.x));
        bq[kk][1] = pack_f16x2(qf[kk][2] * bf16lo(s.y), qf[kk][3] * bf16hi(s.y));
      }
      const float b0 = __shfl_sync(0xffffffffu, cb[0], gi * 4 + c) * scale_log2;
      const float b1 = __shfl_sync(0xffffffffu, cb[1], gi * 4 + c) * scale_log2;
      constexpr int TPG = 4 / C::GPS;  // 16-token tiles per group in this stage
#pragma unroll
      for (int jj = 0; jj < TPG; ++jj) {
        const int j = gi * TPG + jj;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        float fac_lo, fac_hi;
        if constexpr (KB == 2) {
          const unsigned char* kc = slot + C::OFF_KC + j * D * 4;
          const uint32_t sel = (r & 3) | ((4 + (r & 3)) << 8);
          const uint32_t mlo = 0x00030003u << (2 * pr), mhi = 0x00030003u << (2 * pr2);
#pragma unroll
          for (int kk = 0; kk < KCH; ++kk) {
            const uint4 w = lds128(kc + (16 * kk + 4 * c) * 4);
            const uint32_t y01 = prmt(w.x, w.y, sel), y23 = prmt(w.z, w.w, sel);
            const uint32_t a[4] = {y01 & mlo, y01 & mhi, y23 & mlo, y23 & mhi};
            mma_f16(acc, a, bq[kk][0], bq[kk][1]);
          }
          fac_lo = __int_as_float((127 + 24 - 2 * pr) << 23);
          fac_hi = __int_as_float((127 + 24 - 2 * pr2) << 23);
        } else {
          const int wr = 2 * j + ((r & 3) >> 1);
          const int blo = (r & 1) * 2 + (pr >> 1), bhi = (r & 1) * 2 + (pr2 >> 1);
          const int plo = 4 * (pr & 1), phi = 4 * (pr2 & 1);
          const uint32_t slo = blo | ((4 + blo) << 8), shi = bhi | ((4 + bhi) << 8);
          const uint32_t mlo = 0x000F000Fu << plo, mhi = 0x000F000Fu << phi;
          const unsigned char* kc = slot + C::OFF_KC + wr * D * 4;
#pragma unroll
          for (int kk = 0; kk < KCH; ++kk) {
            const uint4 w = lds128(kc + (16 * kk + 4 * c) * 4);
            const uint32_t a[4] = {prmt(w.x, w.y, slo) & mlo, prmt(w.x, w.y, shi) & mhi,
                                   prmt(w.z, w.w, slo) & mlo, prmt(w.z, w.w, shi) & mhi};
            mma_f16(acc, a, bq[kk][0], bq[kk][1]);
          }
          fac_lo = __int_as_float((127 + 24 - plo) << 23);
          fac_hi = __int_as_float((127 + 24 - phi) << 23);
        }
        const bool vlo = 16 * j + tok_lo < n_valid, vhi = 16 * j + tok_hi < n_valid;
        lg[j][0] = vlo ? fmaf(acc[0], fac_lo, b0) : -INFINITY;
        lg[j][1] = vlo ? fmaf(acc[1], fac_lo, b1) : -INFINITY;
        lg[j][2] = vhi ? fmaf(acc[2], fac_hi, b0) : -INFINITY;
        lg[j][3] = vhi ? fmaf(acc[3], fac_hi, b1) : -INFINITY;
      }
    }

    float alpha0, alpha1;
    softmax_update<4>(lg, st, alpha0, alpha1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= alpha0;
      o[i][1] *= alpha1;
      o[i][2] *= alpha0;
      o[i][3] *= alpha1;
    }
#pragma unroll
    for (int g = 0; g < C::NG; ++g) {
      accm[g][0] *= alpha0;
      accm[g][1] *= alpha1;
    }

    // AV: one 16-token k-chunk per tile.
    const int u0 = tile_tok(2 * c), u1 = tile_tok(2 * c + 1), u2 = tile_tok(2 * c + 8), u3 = tile_tok(2 * c + 9);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool vlo = 16 * j + tok_lo < n_valid, vhi = 16 * j + tok_hi < n_valid;
      const unsigned char* vs_lo = slot + C::OFF_VS + (16 * j + tok_lo) * C::NG * (int)sizeof(ST);
      const unsigned char* vs_hi = slot + C::OFF_VS + (16 * j + tok_hi) * C::NG * (int)sizeof(ST);
      const int moff = C::OFF_VM - C::OFF_VS;
      float slo[C::NG], shi[C::NG], mlo[C::NG], mhi[C::NG];
#pragma unroll
      for (int g = 0; g < C::NG; g += 2) {
        if constexpr (C::NG == 1) {
          const uint32_t s_l = *reinterpret_cast<const uint16_t*>(vs_lo);
          const uint32_t s_h = *reinterpret_cast<const uint16_t*>(vs_hi);
          const uint32_t m_l = *reinterpret_cast<const uint16_t*>(vs_lo + moff);
          const uint32_t m_h = *reinterpret_cast<const uint16_t*>(vs_hi + moff);
          slo[0] = bf16lo(s_l);
          shi[0] = bf16lo(s_h);
          mlo[0] = bf16lo(m_l);
          mhi[0] = bf16lo(m_h);
        } else {
          const uint32_t s_l = *reinterpret_cast<const uint32_t*>(vs_lo + 2 * g);
          const uint32_t s_h = *reinterpret_cast<const uint32_t*>(vs_hi + 2 * g);
          const uint32_t m_l = *reinterpret_cast<const uint32_t*>(vs_lo + moff + 2 * g);
          const uint32_t m_h = *reinterpret_cast<const uint32_t*>(vs_hi + moff + 2 * g);
          slo[g] = bf16lo(s_l);
          slo[g + 1] = bf16hi(s_l);
          shi[g] = bf16lo(s_h);
          shi[g + 1] = bf16hi(s_h);
          mlo[g] = bf16lo(m_l);
          mlo[g + 1] = bf16hi(m_l);
          mhi[g] = bf16lo(m_h);
          mhi[g + 1] = bf16hi(m_h);
        }
      }
      uint32_t bp[C::NG][2];
#pragma unroll
      for (int g = 0; g < C::NG; ++g) {
        const float sl = vlo ? slo[g] : 0.f, sh = vhi ? shi[g] : 0.f;
        const float ml = vlo ? mlo[g] : 0.f, mh = vhi ? mhi[g] : 0.f;
        bp[g][0] = movmatrix_trans(pack_f16x2(lg[j][0] * sl, lg[j][1] * sl));
        bp[g][1] = movmatrix_trans(pack_f16x2(lg[j][2] * sh, lg[j][3] * sh));
        accm[g][0] = fmaf(lg[j][0], ml, fmaf(lg[j][2], mh, accm[g][0]));
        accm[g][1] = fmaf(lg[j][1], ml, fmaf(lg[j][3], mh, accm[g][1]));
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
  __device__ static void dense_stage(const unsigned char* slot, int n_valid, int lane, const uint32_t (&qb)[KCH][2],
                                     float scale_log2, WarpState& st, float (&o)[8][4]) {
    const int r = lane >> 2, c = lane & 3;
    const int pr = tile_pos(r), pr2 = (pr + 1) & 3;
    const int tok_lo = 4 * (r & 3) + pr, tok_hi = 4 * (r & 3) + pr2;
    // Zero value rows past the end so that 0 * stale never poisons the MMA.
    if (n_valid < DT) {
      unsigned char* vbase = const_cast<unsigned char*>(slot) + DT * DROW;
      for (int idx = lane; idx < (DT - n_valid) * (D * 2 / 16); idx += 32) {
        const int row = n_valid + idx / (D * 2 / 16), chunk = idx % (D * 2 / 16);
        *reinterpret_cast<uint4*>(vbase + row * DROW + chunk * 16) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    const uint32_t kbase = smem_u32(slot), vbase = smem_u32(slot + DT * DROW);
    const int q = lane >> 3, krow = lane & 7;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kaddr = kbase + tile_tok((q & 1) * 8 + krow) * DROW + (q >> 1) * 16;
#pragma unroll
    for (int kk = 0; kk < KCH; ++kk) {
      uint32_t a[4];
      ldmatrix_x4(a, kaddr + kk * 32);
      mma_bf16(acc, a, qb[kk][0], qb[kk][1]);
    }
    float lg[1][4];
    lg[0][0] = tok_lo < n_valid ? acc[0] * scale_log2 : -INFINITY;
    lg[0][1] = tok_lo < n_valid ? acc[1] * scale_log2 : -INFINITY;
    lg[0][2] = tok_hi < n_valid ? acc[2] * scale_log2 : -INFINITY;
    lg[0][3] = tok_hi < n_valid ? acc[3] * scale_log2 : -INFINITY;
    float alpha0, alpha1;
    softmax_update<1>(lg, st, alpha0, alpha1);
    const uint32_t b0 = movmatrix_trans(pack_bf16x2(lg[0][0], lg[0][1]));
    const uint32_t b1 = movmatrix_trans(pack_bf16x2(lg[0][2], lg[0][3]));
    const uint32_t vaddr = vbase + tile_tok((q >> 1) * 8 + krow) * DROW + (q & 1) * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= alpha0;
      o[i][1] *= alpha1;
      o[i][2] *= alpha0;
      o[i][3] *= alpha1;
      uint32_t a[4];
      ldmatrix_x4_trans(a, vaddr + i * 32);
      mma_bf16(o[i], a, b0, b1);
    }
  }

  // -------------------------------------------------------------- kernel body
  __device__ static void run(const Params& P, unsigned char* smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const ucb_decode_item item = P.items[blockIdx.x];
    const ucb_span sp = P.spans[item.span];
    const ucb_decode_pair pair = P.pairs[item.pair];
    const bool packed = sp.kind == 0;
    const int stage_tokens = packed ? NT : DT;

    unsigned char* ring = smem + warp * C::WARP_SMEM;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * C::WARP_SMEM) + warp * 2;
    int* shared_flag = reinterpret_cast<int*>(smem + WARPS * C::WARP_SMEM + 64);
    if (lane == 0) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
      fence_mbarrier_init();
    }
    __syncwarp();

    const int total_stages = (item.token_end - item.token_begin + stage_tokens - 1) / stage_tokens;
    const int s_begin = warp * total_stages / WARPS, s_end = (warp + 1) * total_stages / WARPS;
    const int n_stages = s_end - s_begin;
    auto stage_range = [&](int s, int& t0, int& t1) {
      t0 = item.token_begin + (s_begin + s) * stage_tokens;
      t1 = min(item.token_end, t0 + stage_tokens);
    };
    auto issue = [&](int s) {
      int t0, t1;
      stage_range(s, t0, t1);
      unsigned char* slot = ring + (s & 1) * C::SLOT;
      if (packed)
        issue_packed(sp, t0, t1, slot, &bars[s & 1], lane);
      else
        issue_dense(sp, t0, t1, slot, &bars[s & 1], lane);
    };
    if (n_stages > 0) issue(0);
    if (n_stages > 1) issue(1);

    // Query fragments for this KV head's query heads (row r of B = head r).
    const int head = pair.kv_head * P.grp + r;
    const bool head_ok = r < P.grp;
    const __nv_bfloat16* qrow = P.query + pair.seq * P.query_stride + (int64_t)head * D;

    WarpState st;
    st.mrun[0] = st.mrun[1] = -INFINITY;
    st.lrun[0] = st.lrun[1] = 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float accm[C::NG][2];
#pragma unroll
    for (int g = 0; g < C::NG; ++g) accm[g][0] = accm[g][1] = 0.f;

    int failed_at = -1;
    if (packed) {
      float qf[KCH][4];
      uint32_t qbp[KCH][2];
#pragma unroll
      for (int kk = 0; kk < KCH; ++kk) {
        uint2 u = make_uint2(0u, 0u);
        if (head_ok) u = *reinterpret_cast<const uint2*>(qrow + 16 * kk + 4 * c);
        qbp[kk][0] = u.x;
        qbp[kk][1] = u.y;
        qf[kk][0] = bf16lo(u.x) * P.scale_log2;
        qf[kk][1] = bf16hi(u.x) * P.scale_log2;
        qf[kk][2] = bf16lo(u.y) * P.scale_log2;
        qf[kk][3] = bf16hi(u.y) * P.scale_log2;
      }
      for (int s = 0; s < n_stages; ++s) {
        if (!mbar_wait_bounded(&bars[s & 1], (s >> 1) & 1, WAIT_LIMIT)) {
          failed_at = s;
          break;
        }
        int t0, t1;
        stage_range(s, t0, t1);
        packed_stage(ring + (s & 1) * C::SLOT, t1 - t0, lane, qf, qbp, P.scale_log2, st, o, accm);
        __syncwarp();
        if (s + 2 < n_stages) issue(s + 2);
      }
    } else {
      uint32_t qb[KCH][2];
#pragma unroll
      for (int kk = 0; kk < KCH; ++kk) {
        qb[kk][0] = head_ok ? *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * c) : 0u;
        qb[kk][1] = head_ok ? *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * c + 8) : 0u;
      }
      for (int s = 0; s < n_stages; ++s) {
        if (!mbar_wait_bounded(&bars[s & 1], (s >> 1) & 1, WAIT_LIMIT)) {
          failed_at = s;
          break;
        }
        int t0, t1;
        stage_range(s, t0, t1);
        dense_stage(ring + (s & 1) * C::SLOT, t1 - t0, lane, qb, P.scale_log2, st, o);
        __syncwarp();
        if (s + 2 < n_stages) issue(s + 2);
      }
    }
    if (failed_at >= 0) {
      // Let copies still in flight land before this CTA's shared memory is released.
      for (int s = failed_at; s < failed_at + 2 && s < n_stages; ++s)
        mbar_wait_bounded(&bars[s & 1], (s >> 1) & 1, WAIT_LIMIT);
      if (lane == 0) atomicOr(P.err, DEVERR_MBAR_TIMEOUT);
      st.mrun[0] = st.mrun[1] = -INFINITY;
    }

    // ---------------------------------------------------------- warp epilogue
    float l0 = warp_sum_r(st.lrun[0]), l1 = warp_sum_r(st.lrun[1]);
    float* ws = reinterpret_cast<float*>(ring);  // [m2 8][l 8][O 8 x D]
    if (r == 0) {
      ws[2 * c] = st.mrun[0];
      ws[2 * c + 1] = st.mrun[1];
      ws[8 + 2 * c] = l0;
      ws[8 + 2 * c + 1] = l1;
    }
    float* wo = ws + 16;
    if (packed) {
#pragma unroll
      for (int g = 0; g < C::NG; ++g) {
        accm[g][0] = warp_sum_r(accm[g][0]);
        accm[g][1] = warp_sum_r(accm[g][1]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int d_lo, d_hi;
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
        wo[(2 * c) * D + d_lo] = fmaf(o[i][0], f_lo, accm[g][0]);
        wo[(2 * c + 1) * D + d_lo] = fmaf(o[i][1], f_lo, accm[g][1]);
        wo[(2 * c) * D + d_hi] = fmaf(o[i][2], f_hi, accm[g][0]);
        wo[(2 * c + 1) * D + d_hi] = fmaf(o[i][3], f_hi, accm[g][1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d_lo = 16 * i + r, d_hi = d_lo + 8;
        wo[(2 * c) * D + d_lo] = o[i][0];
        wo[(2 * c + 1) * D + d_lo] = o[i][1];
        wo[(2 * c) * D + d_hi] = o[i][2];
        wo[(2 * c + 1) * D + d_hi] = o[i][3];
      }
    }
    __syncthreads();

    // ---------------------------------------------------------- CTA merge -> partial
    const int tid = threadIdx.x;  // one thread per channel (D == 128 == blockDim)
    float* part = P.partials + (int64_t)item.partial * PARTIAL_FLOATS;
    for (int h = 0; h < P.grp; ++h) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, reinterpret_cast<float*>(smem + w * C::WARP_SMEM)[h]);
      float acc = 0.f, lsum = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < WARPS; ++w) {
          const float* wsw = reinterpret_cast<float*>(smem + w * C::WARP_SMEM);
          const float f = fast_exp2(wsw[h] - M);
          acc = fmaf(f, wsw[16 + h * D + tid], acc);
          lsum = fmaf(f, wsw[8 + h], lsum);
        }
      }
      part[16 + h * D + tid] = acc;
      if (tid == 0) {
        part[h] = M;
        part[8 + h] = lsum;
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(&P.counters[item.pair], 1);
      *shared_flag = (prev == pair.partial_count - 1) ? 1 : 0;
    }
    __syncthreads();
    if (*shared_flag == 0) return;
    __threadfence();

    // ---------------------------------------------------------- last CTA: pair merge
    const float* base = P.partials + (int64_t)pair.partial_begin * PARTIAL_FLOATS;
    for (int h = 0; h < P.grp; ++h) {
      float M = -INFINITY;
      for (int p = 0; p < pair.partial_count; ++p) M = fmaxf(M, __ldcg(base + (int64_t)p * PARTIAL_FLOATS + h));
      float acc = 0.f, lsum = 0.f;
      for (int p = 0; p < pair.partial_count; ++p) {
        const float* pp = base + (int64_t)p * PARTIAL_FLOATS;
        const float mp = __ldcg(pp + h);
        if (mp == -INFINITY) continue;
        const float f = fast_exp2(mp - M);
        acc = fmaf(f, __ldcg(pp + 16 + h * D + tid), acc);
        lsum = fmaf(f, __ldcg(pp + 8 + h), lsum);
      }
      const float val = acc / lsum;
      const int qh = pair.kv_head * P.grp + h;
      P.out[pair.seq * P.out_stride + (int64_t)qh * D + tid] = __float2bfloat16_rn(val);
      if (!isfinite(val)) atomicOr(P.err, DEVERR_BAD_DESCRIPTOR);
      if (tid == 0 && P.lse != nullptr) P.lse[(int64_t)pair.seq * P.hq + qh] = (M + __log2f(lsum)) * LN2;
    }
    if (tid == 0) P.counters[item.pair] = 0;
  }
};

template <int KB, int VB, int G, typename ST>
__global__ void __launch_bounds__(WARPS * 32) decode_kernel(Params P) {
  extern __shared__ __align__(128) unsigned char smem[];
  Kernel<KB, VB, G, ST>::run(P, smem);
}

template <int KB, int VB, int G, typename ST>
int launch(const Params& P, int num_items, cudaStream_t s) {
  using C = Cfg<KB, VB, G, ST>;
  auto fn = decode_kernel<KB, VB, G, ST>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel: cannot reserve %d bytes of shared memory", C::SMEM);
    configured[dev] = true;
  }
  fn<<<num_items, WARPS * 32, C::SMEM, s>>>(P);
  return ucb_host::check_launch("decode_kernel");
}

template <int KB, int VB, int G, typename ST>
int slots(int* out) {
  using C = Cfg<KB, VB, G, ST>;
  auto fn = decode_kernel<KB, VB, G, ST>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel: shared memory attribute failed");
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, WARPS * 32, C::SMEM) != cudaSuccess ||
      cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "decode kernel: occupancy query failed");
  *out = per_sm * sms;
  return UCB_OK;
}

// Dispatch over the packed configuration.
template <template <int, int, int, typename> class Fn, typename... Args>
int dispatch(int kb, int vb, int g, Args... args) {
#define UCB_CASE(KB_, VB_, G_)                                                             \
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
  static int call(int* out) { return slots<KB, VB, G, ST>(out); }
};

// ---------------------------------------------------------------- partial merge
// Merge n_parts partial blocks per pair (layout [part][pair]) into the output.
__global__ void merge_partials_kernel(const float* __restrict__ parts, int n_parts, const ucb_decode_pair* pairs,
                                      int num_pairs, int grp, int num_kv_heads, __nv_bfloat16* out,
                                      int64_t out_stride, float* lse) {
  const int pidx = blockIdx.x, tid = threadIdx.x;
  const ucb_decode_pair pair = pairs[pidx];
  for (int h = 0; h < grp; ++h) {
    float M = -INFINITY;
    for (int p = 0; p < n_parts; ++p)
      M = fmaxf(M, parts[((int64_t)p * num_pairs + pidx) * PARTIAL_FLOATS + h]);
    float acc = 0.f, lsum = 0.f;
    for (int p = 0; p < n_parts; ++p) {
      const float* pp = parts + ((int64_t)p * num_pairs + pidx) * PARTIAL_FLOATS;
      if (pp[h] == -INFINITY) continue;
      const float f = fast_exp2(pp[h] - M);
      acc = fmaf(f, pp[16 + h * D + tid], acc);
      lsum = fmaf(f, pp[8 + h], lsum);
    }
    const int qh = pair.kv_head * grp + h;
    out[pair.seq * out_stride + (int64_t)qh * D + tid] = __float2bfloat16_rn(acc / lsum);
    if (tid == 0 && lse != nullptr) lse[(int64_t)pair.seq * (grp * num_kv_heads) + qh] = (M + __log2f(lsum)) * LN2;
  }
}

}  // namespace decode
}  // namespace ucb

using ucb_host::set_error;

extern "C" int64_t ucb_decode_partial_bytes(int head_dim) {
  return (int64_t)(16 + 8 * head_dim) * 4;
}

extern "C" int ucb_decode_slots(int k_bits, int v_bits, int group_size, int stat_dtype, int* slots) {
  if (!slots) return set_error(UCB_ERR_INVALID, "ucb_decode_slots: null output");
  if (stat_dtype != UCB_BF16) return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_slots: bf16 statistics only");
  return ucb::decode::dispatch<ucb::decode::SlotsFn>(k_bits, v_bits, group_size, slots);
}

extern "C" int ucb_decode_attention(const void* query, int64_t query_stride, int num_q_heads, int num_kv_heads,
                                    int head_dim, const ucb_span* spans, const ucb_decode_item* items,
                                    int num_items, const ucb_decode_pair* pairs, int num_pairs, int k_bits,
                                    int v_bits, int group_size, int stat_dtype, float softmax_scale,
                                    void* partials, int* counters, void* out, int64_t out_stride, float* lse,
                                    void* stream) {
  if (!query || !spans || !items || !pairs || !partials || !counters || !out)
    return set_error(UCB_ERR_INVALID, "ucb_decode_attention: null pointer");
  if (head_dim != 128) return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: head_dim must be 128");
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > 8)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: need q_heads/kv_heads in [1, 8]");
  if (stat_dtype != UCB_BF16)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_decode_attention: packed statistics must be bf16");
  if (num_items <= 0 || num_pairs <= 0) return set_error(UCB_ERR_INVALID, "ucb_decode_attention: empty batch");
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
  P.items = items;
  P.pairs = pairs;
  P.scale_log2 = softmax_scale * ucb::decode::LOG2E;
  P.partials = static_cast<float*>(partials);
  P.counters = counters;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.out_stride = out_stride;
  P.lse = lse;
  P.err = err;
  return ucb::decode::dispatch<ucb::decode::LaunchFn>(k_bits, v_bits, group_size, P, num_items,
                                                      static_cast<cudaStream_t>(stream));
}

extern "C" int ucb_merge_partials(const void* partials, int n_parts, const ucb_decode_pair* pairs, int num_pairs,
                                  int num_q_heads, int num_kv_heads, int head_dim, void* out, int64_t out_stride,
                                  float* lse, void* stream) {
  if (!partials || !pairs || !out || n_parts <= 0 || num_pairs <= 0)
    return set_error(UCB_ERR_INVALID, "ucb_merge_partials: bad arguments");
  if (head_dim != 128) return set_error(UCB_ERR_UNSUPPORTED, "ucb_merge_partials: head_dim must be 128");
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > 8)
    return set_error(UCB_ERR_UNSUPPORTED, "ucb_merge_partials: need q_heads/kv_heads in [1, 8]");
  ucb::decode::merge_partials_kernel<<<num_pairs, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(partials), n_parts, pairs, num_pairs, num_q_heads / num_kv_heads, num_kv_heads,
      static_cast<__nv_bfloat16*>(out), out_stride, lse);
  return ucb_host::check_launch("merge_partials_kernel");
}
