// Long-query attention on the 5th-generation tensor cores (tcgen05).
//
// Replaces the q_len > 1 branch of the physical-cache attention of the
// reference adapter (unicache/adapters/bagel.py:1598-1858, the fused mixed
// path that ends in flash_attn_func(..., causal=False) over the dequantized
// segments) for one KV head group at a time:
//
//   out[h, m, :] = softmax(q[h, m, :] . k[h, :, :]^T * scale) v[h, :, :]
//   lse[h, m]    = log sum_t exp(q . k_t * scale)               (natural log)
//
// q rows are the (query position, head-in-group) pairs of one KV head, so the
// grouped-query structure becomes a plain M x N attention per KV head.
//
// Design: a CTA works on 256 query rows (two 128-row tiles A and B) of one KV
// head at a time -- one such item per CTA, or, in a persistent launch, a list
// of items (pieces of row blocks over key-tile ranges) run back to back --
// warp-specialised so that the tensor core works on one tile while the other
// tile's softmax runs:
//  * warp 8 (one lane) loads Q_A, Q_B once and streams K tiles (128 tokens x
//    128 channels) and V^T tiles (128 channels x 128 tokens) by TMA with
//    128-byte swizzle (the canonical K-major tcgen05 operand layout) through a
//    two-stage ring of full/empty mbarriers;
//  * warp 9 (one lane) issues tcgen05.mma (fp32 accumulators in tensor
//    memory): S_A = Q_A K^T and S_B = Q_B K^T from shared-memory operands,
//    then O_A += P_A V^T and O_B += P_B V^T with P read from tensor memory
//    as the softmax warpgroups hand it over;
//  * warps 0-3 (tile A) and 4-7 (tile B): each thread owns one query row
//    (one TMEM lane), so the row max and sum need no shuffles.  P =
//    exp2(S*scale*log2e - m) is written in bf16 over the first half of its
//    own S columns in tensor memory (no shared-memory round trip); the row
//    sum accumulates the fp32 weights, as FlashAttention's does.  The running
//    max only moves (and O is rescaled in TMEM) when a row's maximum grows by
//    more than 8 (log2 units).
//  * tcgen05.mma operations of one thread execute in issue order, so the
//    PV product that reads P_x(j) completes its reads before S_x(j+1),
//    issued after it, overwrites those columns.
//  * Every wait has a time budget; on expiry the CTA sets the device error
//    word, drains its tensor-core work (bounded) and frees TMEM.
//
// Three launch forms share the kernel: workspace launches (Q, K and V^T by
// TMA from [heads, rows, 128] / [heads, 128, rows] bf16 tensors), segment-
// table launches (SPANS: the query and outputs in the caller's layout, keys
// and values read in place by producer warps 8, 10 and 11, packed KIVI tiles
// restored in shared memory), and staged launches (the caller's layout for
// the query and outputs, keys and values by TMA from a workspace that
// stage_kernel gathered once per launch).  In the caller-layout forms the
// softmax warps (and warps 10-11 of a staged launch) load Q with cp.async.
#include <cstring>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace ucb {
namespace prefill {

constexpr int D = 128;
constexpr int BM = 128;                   // query rows per tile (TMEM lanes)
constexpr int BN = 128;                   // key tokens per K/V tile
constexpr int STAGES = 2;                 // K/V ring depth
constexpr int QTILE = BM * D * 2;         // 32 KB: two 64-channel swizzled halves
constexpr int QHALF = QTILE / 2;          // 16 KB
constexpr int KTILE = BN * D * 2;         // 32 KB: two 64-channel halves of 128 rows
constexpr int KHALF = KTILE / 2;          // 16 KB
constexpr int VTILE = D * BN * 2;         // 32 KB: two 64-token halves of 128 channel rows
constexpr int VHALF = VTILE / 2;          // 16 KB
constexpr int OFF_Q = 0;                  // Q_A, Q_B
constexpr int OFF_K = OFF_Q + 2 * QTILE;
constexpr int OFF_V = OFF_K + STAGES * KTILE;
constexpr int OFF_BAR = OFF_V + STAGES * VTILE;
constexpr int NBAR = 1 + 4 * STAGES + 7;  // q_full, k/v full/empty, s_full[2], p_full[2], o_done[2], drain
constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
constexpr int SMEM = OFF_TMEM + 16;
constexpr int THREADS = 384;              // warps 0-7 softmax, 8 loader, 9 MMA, 10-11 idle
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait
constexpr float RESCALE_THRESHOLD = 8.f;  // log2 units
constexpr uint32_t TMEM_COLS = 512;       // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
constexpr uint32_t S_COL = 0, O_COL = 256; // tile x: S at S_COL + 128x (P_x in its first 64), O at O_COL + 128x

// tcgen05 instruction descriptors, kind::f16: F32 accumulator, BF16 A and B,
// both K-major, M = 128; N = 128 for S = Q K^T and for O += P V.
constexpr uint32_t idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
constexpr uint32_t IDESC_S = idesc(BN);
constexpr uint32_t IDESC_O = idesc(D);

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand
// whose 8-row atoms are 1024 bytes apart (stride byte offset), starting at
// `addr` (16-byte units); leading byte offset unused for this layout (1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (TMEM) += A (TMEM, M rows x 16 bf16 in 8 columns) * B (shared memory).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Row maximum over all 128 S columns (four loads, one wait); the first 64
// columns stay in registers (s0) for the P pass, which reloads only the
// second 64.
template <bool RAGGED>
__device__ __forceinline__ float row_max_keep(uint32_t t_s, int valid, uint32_t (&s0)[2][32]) {
  uint32_t s1[2][32];
  tc_ld32(t_s, s0[0]);
  tc_ld32(t_s + 32, s0[1]);
  tc_ld32(t_s + 64, s1[0]);
  tc_ld32(t_s + 96, s1[1]);
  tc_wait_ld();
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const int col = 32 * c + i;
      const uint32_t a = c < 2 ? s0[c][i] : s1[c - 2][i], b = c < 2 ? s0[c][i + 1] : s1[c - 2][i + 1];
      m0 = fmaxf(m0, (!RAGGED || col < valid) ? __uint_as_float(a) : -INFINITY);
      m1 = fmaxf(m1, (!RAGGED || col + 1 < valid) ? __uint_as_float(b) : -INFINITY);
    }
  return fmaxf(m0, m1);
}

// One 64-column half of P from S values in registers, stored over TMEM
// columns [32 h, 32 h + 32) of the S tile; returns the two partial sums.
template <bool RAGGED>
__device__ __forceinline__ float2 p_half(const uint32_t (&sv)[2][32], uint32_t t_s, int h, int valid, float2 sc,
                                         float2 nm, float2 sum) {
  uint32_t pw[32];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const int col = 64 * h + 32 * c + i;
      const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[c][i]), __uint_as_float(sv[c][i + 1])), sc, nm);
      float2 p;
      if constexpr (RAGGED) {
        p.x = col < valid ? fast_exp2(x.x) : 0.f;
        p.y = col + 1 < valid ? fast_exp2(x.y) : 0.f;
      } else {
        p.x = fast_exp2(x.x);
        p.y = fast_exp2(x.y);
      }
      sum = __fadd2_rn(sum, p);
      pw[16 * c + i / 2] = pack_bf16x2(p.x, p.y);
    }
  tc_st32(t_s + 32 * h, pw);
  return sum;
}

// P = 2^(S * scale_log2 - m): the first half from the registers row_max_keep
// left, the second half reloaded (its S columns are untouched until then:
// the first half's P overwrites S columns 0-31 only).  Returns the fp32 row
// sum of the weights.
template <bool RAGGED>
__device__ __forceinline__ float write_p_keep(const uint32_t (&s0)[2][32], uint32_t t_s, int valid,
                                              float scale_log2, float neg_m) {
  const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(neg_m, neg_m);
  float2 sum = p_half<RAGGED>(s0, t_s, 0, valid, sc, nm, make_float2(0.f, 0.f));
  uint32_t s1[2][32];
  tc_ld32(t_s + 64, s1[0]);
  tc_ld32(t_s + 96, s1[1]);
  tc_wait_ld();
  sum = p_half<RAGGED>(s1, t_s, 1, valid, sc, nm, sum);
  return sum.x + sum.y;
}

// Tiled TMA load of box {x, y, z} of a 3-D tensor map into shared memory.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// One CTA's problem: query rows [q_row0, q_row0 + q_rows) of KV head `head`
// (at most 2*BM rows) against keys [k_row0, k_row0 + n_tokens) of that head.
// mode ITEM_FINAL writes out/lse; a row block whose keys are split in two
// runs as an ITEM_PARTIAL item (writes its normalised fp32 rows and log2 LSE
// to partial slot `slot`, then adds 1 to flags[slot], making it odd) and an
// ITEM_MERGE item (waits for flags[slot] to be odd, merges that partial with
// its own result by LSE, writes out/lse and adds 1 again).  Each item adds
// exactly 1 per launch whatever happens (a timed-out wait included), so every
// flag is even again when a launch ends and a late partial from a failed
// launch can never be taken for the next launch's: kernels on one stream run
// one after the other, and CUDA-graph replays keep the same rule.
struct WorkItem {
  int head, q_row0, q_rows, k_row0, n_tokens, mode, slot, pad;
};
constexpr int ITEM_FINAL = 0, ITEM_PARTIAL = 1, ITEM_MERGE = 2;
constexpr int PARTIAL_SLOT_FLOATS = 2 * BM * D + 2 * BM;  // O [D][256 rows], then log2 LSE [256]

__device__ __forceinline__ bool wait_flag(const unsigned int* flag, uint64_t budget_ns) {
  const uint64_t t0 = global_timer_ns();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v & 1u) return true;
    if (global_timer_ns() - t0 > budget_ns) return false;
    __nanosleep(256);
  }
}

// Item of a segment-table launch (ucb_lq_item): like WorkItem, plus the
// range of spans (in ucb_span order) that hold the item's KV head's keys; the
// item's keys are tokens [k_row0, k_row0 + n_tokens) of the concatenation of
// those spans, and span s covers tokens [unit_begin, unit_begin + tokens).
// Query rows and outputs of a segment-table launch live in the caller's own
// layout: query and out [positions, q_heads, 128], lse [q_heads, positions];
// row m of an item's KV head is position pos0 + m / grp, query head
// head * grp + m % grp.
struct LqItem {
  int head, q_row0, q_rows, k_row0, n_tokens, mode, slot, span_begin, span_count, pos0, pad1, pad2;
};

// ---------------------------------------------------------------- span producers
// In a segment-table launch the keys and values are read in place: threads
// of warps 8, 10 and 11 (96 producers) fill each K and V tile from the item's
// spans.  Both tiles take the layout a 128-byte-swizzled TMA load of
// 64-channel boxes produces: two 16 KB halves (channels 0-63, 64-127), token
// row r at r * 128 bytes, 16-byte chunk c of the row at (c ^ (r & 7)) * 16.
// K is the K-major B operand of S = Q K^T as before; V is read as an
// MN-major B operand of O += P V (channels contiguous), so no transpose is
// needed.  Dense rows are copied with 16-byte cp.async; packed KIVI codes are
// restored as code * scale + minimum with one rounding to bf16 (the
// reference, unicache/storage/physical.py:178-201, rounds the fp32 result
// once more first, which can differ in the last bf16 bit in rare ties) and
// stored with plain shared-memory stores.  Rows past the item's last key are
// zero-filled (the softmax masks them; V must stay finite).
constexpr int PRODUCERS = 96;

__device__ __forceinline__ uint32_t tile_chunk(int row, int chunk) {
  return (uint32_t)((chunk >> 3) * (BN * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// Each producer owns one 16-byte chunk column (pid % 16) and walks every
// sixth row from row pid / 16, so a warp copies two whole rows per
// instruction (coalesced) and the addresses advance by constants.
constexpr int ROW_STEP = PRODUCERS / 16;
__device__ __forceinline__ void dense_rows(const __nv_bfloat16* base, int64_t stride, int off, int r0, int n,
                                           uint32_t tile, int pid) {
  const int c = pid & 15, first = pid >> 4;
  if (first >= n) return;
  const char* src = reinterpret_cast<const char*>(base + (int64_t)(off + first) * stride + 8 * c);
  const int64_t src_step = (int64_t)ROW_STEP * stride * 2;
  const uint32_t half = tile + (uint32_t)((c >> 3) * (BN * 128)), cl = (uint32_t)(c & 7) << 4;
  for (int rr = first; rr < n; rr += ROW_STEP, src += src_step) {
    const int r = r0 + rr;
    cp_async16(half + r * 128 + (cl ^ ((uint32_t)(r & 7) << 4)), src);
  }
}

__device__ __forceinline__ void zero_rows(int r0, unsigned char* tile, int pid) {
  const int c = pid & 15;
  for (int r = r0 + (pid >> 4); r < BN; r += PRODUCERS / 16)
    *reinterpret_cast<uint4*>(tile + tile_chunk(r, c)) = make_uint4(0u, 0u, 0u, 0u);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = bf16lo(w[k]);
    f[2 * k + 1] = bf16hi(w[k]);
  }
}

// Packed codes are restored on bf16 pairs: a code placed in the mantissa of
// a bf16 magic number (M + code, exact) loses M in one exact FMA, and a
// second FMA forms code * scale + minimum with one rounding to bf16 (the
// decode kernel restores its keys the same way).  M = 128, 32 or 8 takes a
// 2-bit code at bits 0-1, 2-3 or 4-5 of a half without a shift.
__device__ __forceinline__ uint32_t restore2(uint32_t z, uint32_t mask_magic_and, uint32_t magic, uint32_t neg_m,
                                             uint32_t s, uint32_t m) {
  return bf16x2_dequant((z & mask_magic_and) | magic, neg_m, s, m);
}

// Keys packed along tokens ([T/f, D] words of this head, f = 32/KB tokens per
// word; statistics [T/G, D]).  Unit = (word row, 8-channel chunk, half of the
// word's tokens): 8 words and the chunk's 8 scales and minima in (channel
// pairs already adjacent), f/2 rows of one 16-byte chunk out.  The loads of
// a thread's next unit are issued before the current unit is restored, so a
// thread waits for memory about once per tile rather than once per unit.
struct KeyUnit {
  uint4 ca, cb, s4, m4;
};

template <int KB>
__device__ void packed_keys(const ucb_span& S, int G, int off, int r0, int n, unsigned char* tile, int pid) {
  constexpr int F = 32 / KB, HALF_TOK = F / 2;
  const int w0 = off / F, w1 = (off + n - 1) / F, nu = (w1 - w0 + 1) * 32;
  const uint32_t* codes = static_cast<const uint32_t*>(S.key_code);
  const uint16_t* sc = static_cast<const uint16_t*>(S.key_scale);
  const uint16_t* mn = static_cast<const uint16_t*>(S.key_minimum);
  auto wanted = [&](int u) {
    const int t_first = (w0 + (u >> 5)) * F + (u & 1) * HALF_TOK;
    return t_first + HALF_TOK > off && t_first < off + n;
  };
  auto next = [&](int u) {
    while (u < nu && !wanted(u)) u += PRODUCERS;
    return u;
  };
  auto load = [&](int u, KeyUnit& d) {
    const int w = w0 + (u >> 5), c = (u >> 1) & 15;
    const uint32_t* cw = codes + (int64_t)w * D + 8 * c;
    const int64_t g = (int64_t)(w * F) / G;
    d.ca = __ldg(reinterpret_cast<const uint4*>(cw));
    d.cb = __ldg(reinterpret_cast<const uint4*>(cw + 4));
    d.s4 = __ldg(reinterpret_cast<const uint4*>(sc + g * D + 8 * c));
    d.m4 = __ldg(reinterpret_cast<const uint4*>(mn + g * D + 8 * c));
  };
  int u = next(pid);
  KeyUnit cur;
  if (u < nu) load(u, cur);
  while (u < nu) {
    const int un = next(u + PRODUCERS);
    KeyUnit nxt;
    if (un < nu) load(un, nxt);
    const int w = w0 + (u >> 5), c = (u >> 1) & 15, hh = u & 1;
    const uint32_t word[8] = {cur.ca.x, cur.ca.y, cur.ca.z, cur.ca.w, cur.cb.x, cur.cb.y, cur.cb.z, cur.cb.w};
    const uint32_t sp[4] = {cur.s4.x, cur.s4.y, cur.s4.z, cur.s4.w}, mp[4] = {cur.m4.x, cur.m4.y, cur.m4.z, cur.m4.w};
#pragma unroll
    for (int b = 0; b < 2; ++b) {  // the two bytes (KB = 2: 4 tokens each; KB = 4: 2 tokens each) of this half
      const int byte = 2 * hh + b;
      const uint32_t sel = byte | (byte << 4) | ((4 + byte) << 8) | ((4 + byte) << 12);
      uint32_t z[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) z[k] = prmt(word[2 * k], word[2 * k + 1], sel);
#pragma unroll
      for (int p = 0; p < 8 / KB; ++p) {  // tokens of the byte
        const int t = w * F + byte * (8 / KB) + p;
        if (t < off || t >= off + n) continue;
        uint32_t out[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (KB == 2) {
            if (p == 0) out[k] = restore2(z[k], 0x00030003u, 0x43004300u, 0xC300C300u, sp[k], mp[k]);
            else if (p == 1) out[k] = restore2(z[k], 0x000C000Cu, 0x42004200u, 0xC200C200u, sp[k], mp[k]);
            else if (p == 2) out[k] = restore2(z[k], 0x00300030u, 0x41004100u, 0xC100C100u, sp[k], mp[k]);
            else out[k] = restore2(z[k] >> 6, 0x00030003u, 0x43004300u, 0xC300C300u, sp[k], mp[k]);
          } else {
            out[k] = restore2(p == 0 ? z[k] : z[k] >> 4, 0x000F000Fu, 0x43004300u, 0xC300C300u, sp[k], mp[k]);
          }
        }
        *reinterpret_cast<uint4*>(tile + tile_chunk(r0 + (t - off), c)) = make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
    cur = nxt;
    u = un;
  }
}

// Values packed along channels ([T, D/f] words, f = 32/VB channels per word;
// statistics [T, D/G]).  Unit = (token, 64-channel half row): the half row's
// words and its groups' statistics in, 8 chunks out; loads of the next unit
// are issued before the current one is restored.
template <int VB>
struct ValueUnit {
  uint32_t word[D / (32 / VB) / 2];
  uint32_t s_a, m_a, s_b, m_b;
};

template <int VB>
__device__ void packed_values(const ucb_span& S, int G, int off, int r0, int n, unsigned char* tile, int pid) {
  constexpr int F = 32 / VB, W = D / F, HW = W / 2;  // words per token, per half row
  const uint32_t* codes = static_cast<const uint32_t*>(S.value_code);
  const uint16_t* sc = static_cast<const uint16_t*>(S.value_scale);
  const uint16_t* mn = static_cast<const uint16_t*>(S.value_minimum);
  const int ng = D / G;
  auto load = [&](int u, ValueUnit<VB>& d) {
    const int64_t t = off + (u >> 1);
    const int hh = u & 1;
#pragma unroll
    for (int k = 0; k < HW; k += 4) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(codes + t * W + hh * HW + k));
      d.word[k] = v.x;
      d.word[k + 1] = v.y;
      d.word[k + 2] = v.z;
      d.word[k + 3] = v.w;
    }
    const int g0 = (64 * hh) / G;  // groups covering channels [64 hh, 64 hh + 64): G = 32 -> 2, else 1
    d.s_a = sc[t * ng + g0];
    d.m_a = mn[t * ng + g0];
    d.s_b = (G == 32) ? (uint32_t)sc[t * ng + g0 + 1] : d.s_a;
    d.m_b = (G == 32) ? (uint32_t)mn[t * ng + g0 + 1] : d.m_a;
  };
  int u = pid;
  ValueUnit<VB> cur;
  if (u < 2 * n) load(u, cur);
  while (u < 2 * n) {
    const int un = u + PRODUCERS;
    ValueUnit<VB> nxt;
    if (un < 2 * n) load(un, nxt);
    const int hh = u & 1, r = r0 + (u >> 1);
    const uint32_t s2a = cur.s_a | (cur.s_a << 16), m2a = cur.m_a | (cur.m_a << 16);
    const uint32_t s2b = cur.s_b | (cur.s_b << 16), m2b = cur.m_b | (cur.m_b << 16);
#pragma unroll
    for (int c = 0; c < 8; ++c) {  // 8-channel chunks of the half row
      const bool second = (8 * c) >= 32;  // second 32-channel group of the half (G = 32)
      const uint32_t s2 = second ? s2b : s2a, m2 = second ? m2b : m2a;
      uint32_t out[4];
      if constexpr (VB == 2) {
        const uint32_t wv = cur.word[c / 2];  // 16 channels per word, chunk = 2 bytes
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int byte = 2 * (c & 1) + b;
          const uint32_t y = prmt(wv, 0u, byte | (byte << 4) | (byte << 8) | (byte << 12));
          // channels 4 byte + {0, 1} at bits 0-1 / 18-19, then + {2, 3} after a 4-bit shift
          out[2 * b] = restore2(y, 0x000C0003u, 0x42004300u, 0xC200C300u, s2, m2);
          out[2 * b + 1] = restore2(y >> 4, 0x000C0003u, 0x42004300u, 0xC200C300u, s2, m2);
        }
      } else {
        const uint32_t wv = cur.word[c], wh = wv >> 4;  // 8 channels per word, chunk = 1 word
#pragma unroll
        for (int k = 0; k < 4; ++k)
          out[k] = restore2(prmt(wv, wh, k | (k << 4) | ((4 + k) << 8) | ((4 + k) << 12)), 0x000F000Fu, 0x43004300u,
                            0xC300C300u, s2, m2);
      }
      *reinterpret_cast<uint4*>(tile + tile_chunk(r, 8 * hh + c)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
    cur = nxt;
    u = un;
  }
}

// Fill rows [0, valid) of a K (keys) or V tile with tokens [tok0, tok0 +
// valid) of the item's spans, then zero rows [valid, BN).
__device__ void fill_tile(bool keys, const ucb_span* spans, int span_count, int tok0, int valid, int kb, int vb,
                          int G, unsigned char* tile, int pid) {
  const uint32_t tile_addr = smem_u32(tile);
  for (int si = 0; si < span_count; ++si) {
    const ucb_span& S = spans[si];
    const int s0 = S.unit_begin, s1 = S.unit_begin + S.tokens;
    const int a = max(tok0, s0), b = min(tok0 + valid, s1);
    if (a >= b) continue;
    const int r0 = a - tok0, off = a - s0, n = b - a;
    if (S.kind == 1) {
      dense_rows(static_cast<const __nv_bfloat16*>(keys ? S.key_code : S.value_code),
                 keys ? S.key_stride : S.value_stride, off, r0, n, tile_addr, pid);
    } else if (keys) {
      if (kb == 2) packed_keys<2>(S, G, off, r0, n, tile, pid);
      else packed_keys<4>(S, G, off, r0, n, tile, pid);
    } else {
      if (vb == 2) packed_values<2>(S, G, off, r0, n, tile, pid);
      else packed_values<4>(S, G, off, r0, n, tile, pid);
    }
  }
  if (valid < BN) zero_rows(valid, tile, pid);
}

// Shared-memory descriptor of the MN-major V operand: 64-channel (128-byte)
// swizzle atoms along N are LBO = 16 KB apart (the two channel halves) and
// 8-token groups along K are SBO = 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((BN * 128) >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
constexpr uint32_t IDESC_O_MN = IDESC_O | (1u << 16);  // B (V) MN-major

struct Params {
  int m_rows;        // query rows per head in q / out / lse (row stride of the head)
  int n_tokens;      // key tokens per head (single-problem launches)
  float scale_log2;  // softmax scale * log2(e)
  const WorkItem* items;  // per-CTA problems (batched launches), or null: CTA (x, y) = rows 2*BM*x.. of head y
  const LqItem* lq_items; // segment-table launches: per-CTA problems reading spans in place
  const ucb_span* spans;  // the spans lq_items refer to
  int k_bits, v_bits, group;  // packed spans of a segment-table launch
  const __nv_bfloat16* q;     // segment-table launches: query [positions, hq, 128]
  int hq, grp, positions;     // query heads, query heads per KV head, positions (lse row length)
  float* partials;        // PARTIAL_SLOT_FLOATS per slot (split row blocks), or null
  unsigned int* flags;    // one per slot, even between launches, or null
  const int32_t* cta_items;  // caller-layout launches: CTA b runs items [cta_items[b], cta_items[b + 1]), or null
  uint64_t* trace;           // optional: per CTA 32 words, see ucb_prefill_set_trace
  __nv_bfloat16* out;  // [heads, m_rows, D]
  float* lse;          // [heads, m_rows], may be null
  unsigned int* err;
};

// Q_A and Q_B of a caller-layout item straight from the query [positions,
// hq, 128] into the swizzled Q tiles (zero rows past the item's last row):
// thread pid of `threads` (a multiple of 16) owns 16-byte chunk column
// pid % 16 and every (threads / 16)-th row from pid / 16; the row's
// (position, head-in-group) pair advances by an add and one wrap per step
// rather than a division.  The caller waits for its cp.async group and
// fences the async proxy before publishing.
__device__ __forceinline__ void load_q_caller(const Params& P, unsigned char* smem, int m0, int m_end, int pos0,
                                              int head, int pid, int threads) {
  const uint32_t q_addr = smem_u32(smem + OFF_Q);
  const int c = pid & 15, step = threads >> 4;
  const uint32_t cl = (uint32_t)(c & 7) << 4;
  const int step_pos = step / P.grp, step_g = step % P.grp;
  int rb = pid >> 4, pos = (m0 + rb) / P.grp, g = (m0 + rb) % P.grp;
  const int64_t row_stride = (int64_t)P.hq * D;
  const __nv_bfloat16* qh = P.q + (int64_t)pos0 * row_stride + (int64_t)head * P.grp * D + 8 * c;
  for (; rb < 2 * BM; rb += step) {
    const int x = rb >> 7, rr = rb & (BM - 1);
    const uint32_t dst = x * QTILE + (c >> 3) * QHALF + rr * 128 + (cl ^ ((uint32_t)(rr & 7) << 4));
    if (m0 + rb < m_end)
      cp_async16(q_addr + dst, qh + (int64_t)pos * row_stride + g * D);
    else
      *reinterpret_cast<uint4*>(smem + OFF_Q + dst) = make_uint4(0u, 0u, 0u, 0u);
    pos += step_pos;
    g += step_g;
    if (g >= P.grp) {
      g -= P.grp;
      ++pos;
    }
  }
}
// Threads that load Q in a caller-layout launch: the softmax warps, idle
// until the first S tile of an item, which needs Q.
constexpr int Q_THREADS = 256;

// ---------------------------------------------------------------- staging
// A staged launch first gathers each key space (the keys of one KV head of
// one sample: the span list of its items) once into a bf16 workspace, K as
// rows [heads, ws_rows, 128] and V transposed [heads, 128, ws_rows], rows
// [ws_row0, ws_row0 + rows) of the job's head with tokens past `tokens`
// zeroed; the attention kernel then streams both by TMA.  Dense spans are
// copied; packed spans are restored with the arithmetic of the in-tile
// restore (code * scale + minimum, one rounding to bf16), so a staged launch
// and a segment-table launch see the same key and value values.  Restoring
// once per launch rather than once per row block pays when several row
// blocks read the same keys (the configuration-4 layer has 28 per KV head).
struct StageJob {
  int head, span_begin, span_count, tokens, ws_row0, rows, pad0, pad1;
};
constexpr int STAGE_T = 32;          // tokens per staging block
constexpr int STAGE_THREADS = 128;
constexpr int STAGE_PITCH = D + 8;   // bf16 per token row of a block's value rows

// Block (x, job): tokens [32 x, 32 x + 32) of the job's key space.  The job's
// span records are staged in shared memory (STAGE_SPANS at a time) and each
// token is mapped to its span once; each thread then issues the loads of all
// its (token, 8-channel chunk) items before restoring any, so a block waits
// for memory about once per span batch.  K rows go straight to the workspace
// (16-byte chunks, coalesced); value rows gather in shared memory and leave
// as V^T rows of 32 tokens (64 bytes per channel).
constexpr int STAGE_SPANS = 16;
constexpr int STAGE_ITEMS = STAGE_T * 16 / STAGE_THREADS;  // items per thread per block

struct StageLoad {
  uint4 a, b, c, d;  // dense: key, value chunk; packed: key code words (a, b), key scales (c), key minima (d)
  uint32_t vword, vs, vm;
};

template <int KB, int VB>
__global__ void __launch_bounds__(STAGE_THREADS) stage_kernel(const StageJob* __restrict__ jobs,
                                                              const ucb_span* __restrict__ spans, int G,
                                                              __nv_bfloat16* __restrict__ k_ws,
                                                              __nv_bfloat16* __restrict__ vt_ws, int64_t ws_rows) {
  __shared__ __align__(16) __nv_bfloat16 vblk[STAGE_T * STAGE_PITCH];
  __shared__ __align__(16) ucb_span sps[STAGE_SPANS];
  __shared__ int span_of[STAGE_T];
  const StageJob J = jobs[blockIdx.y];
  const int c0 = blockIdx.x * STAGE_T;
  if (c0 >= J.rows) return;
  const int tid = threadIdx.x;
  __nv_bfloat16* kdst = k_ws + ((int64_t)J.head * ws_rows + J.ws_row0 + c0) * D;
  constexpr int KF = 32 / KB, VF = 32 / VB, VW = D / VF;
  constexpr uint32_t KMASK = (1u << KB) - 1u, VMASK = (1u << VB) - 1u;
  const int ng = D / G;
  for (int sb = 0; sb < J.span_count; sb += STAGE_SPANS) {
    const int nb = min(STAGE_SPANS, J.span_count - sb);
    __syncthreads();  // the previous batch's records are no longer read
    for (int i = tid; i < nb * (int)(sizeof(ucb_span) / 8); i += STAGE_THREADS)
      reinterpret_cast<uint64_t*>(sps)[i] = reinterpret_cast<const uint64_t*>(spans + J.span_begin + sb)[i];
    __syncthreads();
    if (tid < STAGE_T) {
      const int tok = c0 + tid;
      int found = -1;
      for (int k = 0; k < nb; ++k)
        if (tok < J.tokens && tok >= sps[k].unit_begin && tok < sps[k].unit_begin + sps[k].tokens) found = k;
      span_of[tid] = found;
    }
    __syncthreads();
    StageLoad L[STAGE_ITEMS];
#pragma unroll
    for (int it = 0; it < STAGE_ITEMS; ++it) {
      const int i = tid + it * STAGE_THREADS, t = i >> 4, cc = i & 15, k = span_of[t];
      if (k < 0) continue;
      const ucb_span& S = sps[k];
      const int off = c0 + t - S.unit_begin;
      if (S.kind == 1) {
        L[it].a = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(S.key_code) +
                                                       (int64_t)off * S.key_stride + 8 * cc));
        L[it].b = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(S.value_code) +
                                                       (int64_t)off * S.value_stride + 8 * cc));
      } else {
        const uint32_t* cw = static_cast<const uint32_t*>(S.key_code) + (int64_t)(off / KF) * D + 8 * cc;
        const int64_t g = off / G;
        L[it].a = __ldg(reinterpret_cast<const uint4*>(cw));
        L[it].b = __ldg(reinterpret_cast<const uint4*>(cw + 4));
        L[it].c = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(S.key_scale) + g * D + 8 * cc));
        L[it].d = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(S.key_minimum) + g * D + 8 * cc));
        L[it].vword = __ldg(static_cast<const uint32_t*>(S.value_code) + (int64_t)off * VW + (8 * cc) / VF);
        L[it].vs = __ldg(static_cast<const uint16_t*>(S.value_scale) + (int64_t)off * ng + (8 * cc) / G);
        L[it].vm = __ldg(static_cast<const uint16_t*>(S.value_minimum) + (int64_t)off * ng + (8 * cc) / G);
      }
    }
#pragma unroll
    for (int it = 0; it < STAGE_ITEMS; ++it) {
      const int i = tid + it * STAGE_THREADS, t = i >> 4, cc = i & 15, k = span_of[t];
      if (k < 0) continue;
      uint4 kv, vv;
      if (sps[k].kind == 1) {
        kv = L[it].a;
        vv = L[it].b;
      } else {
        // keys: code of token `off` in each of the 8 channel words (restore as in the operand tiles)
        const int sh = KB * ((c0 + t - sps[k].unit_begin) % KF);
        const uint32_t w[8] = {L[it].a.x, L[it].a.y, L[it].a.z, L[it].a.w, L[it].b.x, L[it].b.y, L[it].b.z, L[it].b.w};
        const uint32_t sp[4] = {L[it].c.x, L[it].c.y, L[it].c.z, L[it].c.w};
        const uint32_t mp[4] = {L[it].d.x, L[it].d.y, L[it].d.z, L[it].d.w};
        uint32_t ko[4], vo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t code = ((w[2 * q] >> sh) & KMASK) | (((w[2 * q + 1] >> sh) & KMASK) << 16);
          ko[q] = bf16x2_dequant(code | 0x43004300u, 0xC300C300u, sp[q], mp[q]);
        }
        // values: channels 8 cc .. 8 cc + 7 of the token, one word
        const int base = VB * ((8 * cc) % VF);
        const uint32_t s2 = L[it].vs | (L[it].vs << 16), m2 = L[it].vm | (L[it].vm << 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t a = (L[it].vword >> (base + VB * 2 * q)) & VMASK;
          const uint32_t b = (L[it].vword >> (base + VB * (2 * q + 1))) & VMASK;
          vo[q] = bf16x2_dequant((a | (b << 16)) | 0x43004300u, 0xC300C300u, s2, m2);
        }
        kv = make_uint4(ko[0], ko[1], ko[2], ko[3]);
        vv = make_uint4(vo[0], vo[1], vo[2], vo[3]);
      }
      *reinterpret_cast<uint4*>(kdst + (int64_t)t * D + 8 * cc) = kv;
      *reinterpret_cast<uint4*>(&vblk[t * STAGE_PITCH + 8 * cc]) = vv;
    }
  }
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < STAGE_T * 16; i += STAGE_THREADS) {  // tokens past the key space
    const int t = i >> 4, cc = i & 15;
    if (c0 + t >= J.tokens) {
      *reinterpret_cast<uint4*>(kdst + (int64_t)t * D + 8 * cc) = zero;
      *reinterpret_cast<uint4*>(&vblk[t * STAGE_PITCH + 8 * cc]) = zero;
    }
  }
  __syncthreads();
  const uint16_t* vb = reinterpret_cast<const uint16_t*>(vblk);
  for (int i = tid; i < D * (STAGE_T / 8); i += STAGE_THREADS) {
    const int ch = i % D, q = i / D;
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = (uint32_t)vb[(8 * q + 2 * k) * STAGE_PITCH + ch] | ((uint32_t)vb[(8 * q + 2 * k + 1) * STAGE_PITCH + ch] << 16);
    *reinterpret_cast<uint4*>(vt_ws + ((int64_t)J.head * D + ch) * ws_rows + J.ws_row0 + c0 + 8 * q) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// One problem of a CTA, decoded from whichever table the launch uses.
struct Item {
  int head, m0, m_end, k0, n_tokens, mode, slot, nparts, span_begin, span_count, pos0;
};

// Item `idx` of the launch.  Segment-table and staged launches read LqItem
// records (a staged item's key space starts at workspace row reserved[0]; a
// merge item folds in reserved[1] partials, at least one, from slots
// [slot, slot + reserved[1])); batched workspace launches read WorkItem
// records; single-problem launches derive the item from the grid.
template <bool SPANS>
__device__ __forceinline__ Item load_item(const Params& P, bool staged, int idx, int tid) {
  Item I;
  I.nparts = 1;
  I.span_begin = I.span_count = I.pos0 = 0;
  I.mode = ITEM_FINAL;
  I.slot = 0;
  if (SPANS || staged) {
    const LqItem it = P.lq_items[idx];
    I.head = it.head;
    I.m0 = it.q_row0;
    I.m_end = it.q_row0 + it.q_rows;
    I.k0 = it.k_row0 + (staged ? it.pad1 : 0);
    I.n_tokens = it.n_tokens;
    I.mode = it.mode;
    I.slot = it.slot;
    I.nparts = max(1, it.pad2);
    I.span_begin = it.span_begin;
    I.span_count = it.span_count;
    I.pos0 = it.pos0;
  } else if (P.items) {
    const WorkItem it = P.items[idx];
    I.head = it.head;
    I.m0 = it.q_row0;
    I.m_end = it.q_row0 + it.q_rows;
    I.k0 = it.k_row0;
    I.n_tokens = it.n_tokens;
    I.mode = it.mode;
    I.slot = it.slot;
  } else {
    I.head = blockIdx.y;
    I.m0 = blockIdx.x * 2 * BM;
    I.m_end = P.m_rows;
    I.k0 = 0;
    I.n_tokens = P.n_tokens;
  }
  if (I.mode != ITEM_FINAL && (!P.partials || !P.flags || I.slot < 0)) {
    if (tid == 0) atomicOr(P.err, DEVERR_BAD_DESCRIPTOR);
    I.mode = ITEM_FINAL;
  }
  return I;
}

// The flag additions an item owes each launch (a partial's own slot; a
// merge item's partner slots), made even when the item could not run.
__device__ __forceinline__ void settle_flags(const Params& P, const Item& I) {
  if (I.mode == ITEM_PARTIAL) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(P.flags + I.slot), "r"(1u) : "memory");
  } else if (I.mode == ITEM_MERGE) {
    for (int k = 0; k < I.nparts; ++k)
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(P.flags + I.slot + k), "r"(1u) : "memory");
  }
}

// The item's result from its O accumulators (this thread's TMEM lane t_o)
// and running max / sum: a partial item writes its normalised fp32 rows and
// log2 LSE to its slot; a final or merge item (the latter after folding in
// its partners' partials, which it waits for) writes bf16 rows and the
// natural-log LSE in the launch's layout.  Called by every softmax thread.
__device__ __forceinline__ void write_item_result(const Params& P, const Item& I, bool caller_layout, bool good,
                                                  int nt, int r_blk, int lane, uint32_t t_o, float m_run,
                                                  float l_run, int* failed) {
  const int m = I.m0 + r_blk;
  const bool live = m < I.m_end;
  bool merged = false;
  if (!good) {
    if (lane == 0) atomicOr(failed, 1);
  } else if (nt == 0) {
    // an item without keys writes nothing (the host never builds one)
  } else if (I.mode == ITEM_PARTIAL) {
    float* part = P.partials + (int64_t)I.slot * PARTIAL_SLOT_FLOATS;
    const float inv = 1.f / l_run;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t ov[32];
      tc_ld32(t_o + 32 * c, ov);
      tc_wait_ld();
      if (live) {
#pragma unroll
        for (int i = 0; i < 32; ++i) part[(32 * c + i) * (2 * BM) + r_blk] = __uint_as_float(ov[i]) * inv;
      }
    }
    if (live) part[D * 2 * BM + r_blk] = m_run + __log2f(l_run);
    __threadfence();
  } else {
    // ITEM_FINAL, or ITEM_MERGE: fold in the partners' rows once published.
    float w_own = 1.f, lse2 = m_run + __log2f(l_run), mx = lse2, inv_sum = 1.f;
    if (I.mode == ITEM_MERGE) {
      bool all_in = true;
      for (int k = 0; k < I.nparts; ++k) all_in = all_in && wait_flag(P.flags + I.slot + k, WAIT_NS);
      merged = __all_sync(0xffffffffu, all_in);
      if (!merged) {
        if (lane == 0) atomicOr(failed, 1);
      } else if (live) {
        for (int k = 0; k < I.nparts; ++k)
          mx = fmaxf(mx, __ldcg(P.partials + (int64_t)(I.slot + k) * PARTIAL_SLOT_FLOATS + D * 2 * BM + r_blk));
        float sum = fast_exp2(lse2 - mx);
        for (int k = 0; k < I.nparts; ++k)
          sum += fast_exp2(__ldcg(P.partials + (int64_t)(I.slot + k) * PARTIAL_SLOT_FLOATS + D * 2 * BM + r_blk) - mx);
        inv_sum = 1.f / sum;
        w_own = fast_exp2(lse2 - mx) * inv_sum;
        lse2 = mx + __log2f(sum);
      }
    }
    const float inv = w_own / l_run;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t ov[32];
      tc_ld32(t_o + 32 * c, ov);
      tc_wait_ld();
      if (live) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(ov[i]) * inv;
        if (merged) {
#pragma unroll 2
          for (int k = 0; k < I.nparts; ++k) {
            const float* part = P.partials + (int64_t)(I.slot + k) * PARTIAL_SLOT_FLOATS;
            const float wp = fast_exp2(__ldcg(part + D * 2 * BM + r_blk) - mx) * inv_sum;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fmaf(wp, __ldcg(part + (32 * c + i) * (2 * BM) + r_blk), v[i]);
          }
        }
        __nv_bfloat16* dst =
            caller_layout
                ? P.out + ((int64_t)(I.pos0 + m / P.grp) * P.hq + I.head * P.grp + m % P.grp) * D + 32 * c
                : P.out + ((int64_t)I.head * P.m_rows + m) * D + 32 * c;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w4;
          w4.x = pack_bf16x2(v[i], v[i + 1]);
          w4.y = pack_bf16x2(v[i + 2], v[i + 3]);
          w4.z = pack_bf16x2(v[i + 4], v[i + 5]);
          w4.w = pack_bf16x2(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(dst + i) = w4;
        }
      }
    }
    if (live && P.lse) {
      const int64_t at = caller_layout
                             ? (int64_t)(I.head * P.grp + m % P.grp) * P.positions + I.pos0 + m / P.grp
                             : (int64_t)I.head * P.m_rows + m;
      P.lse[at] = lse2 * 0.6931471805599453f;
    }
  }
}

// SPANS: keys and values come from the item's spans (producer warps 8, 10,
// 11); otherwise from the K / V^T tensor maps (loader warp 8), with the query
// from the Q tensor map (workspace launches) or the caller's layout (staged
// launches: P.lq_items set).
//
// A CTA runs the items [cta_items[b], cta_items[b + 1]) of P.cta_items one
// after the other when that table is given (segment-table and staged
// launches), else item blockIdx.x.  Across items the K/V ring, the S/P/O
// hand-offs and their mbarrier phases simply continue (tile counters run
// over the CTA's whole item list); at an item boundary the softmax warps
// write the item's result, then load the next item's query rows, which the
// MMA thread waits for before the next S tile.
template <bool SPANS>
__global__ void __launch_bounds__(THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, Params P) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* trace = P.trace ? P.trace + 32 * (size_t)blockIdx.x : nullptr;
  if (trace && tid == 0) {
    trace[0] = global_timer_ns();
    trace[2] = sm_id();
  }
  // A staged launch: LqItem problems in the caller's layout, keys and values
  // by TMA from the staging workspace.
  const bool staged = !SPANS && P.lq_items != nullptr;
  const bool caller_layout = SPANS || staged;
  int ib = blockIdx.x, ie = blockIdx.x + 1;
  if (caller_layout && P.cta_items) {
    ib = P.cta_items[blockIdx.x];
    ie = P.cta_items[blockIdx.x + 1];
  }
  const int n_items = max(0, ie - ib);
  auto tiles_of = [](const Item& I) { return (I.n_tokens + BN - 1) / BN; };
  // The swizzled operand layout needs a 1024-byte aligned base.
  if (smem_u32(smem) & 1023) {
    if (tid == 0) {
      atomicOr(P.err, DEVERR_BAD_DESCRIPTOR);
      for (int it = ib; it < ie; ++it) settle_flags(P, load_item<SPANS>(P, staged, it, 1));  // keep the parity rule
    }
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* v_full = k_empty + STAGES;
  uint64_t* v_empty = v_full + STAGES;
  uint64_t* s_full = v_empty + STAGES;  // [2]
  uint64_t* p_full = s_full + 2;        // [2]
  uint64_t* o_done = p_full + 2;        // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
  __shared__ int failed;
  __shared__ int stop_items;

  if (tid == 0) {
    failed = 0;
    stop_items = 0;
    mbar_init(q_full, caller_layout ? Q_THREADS : 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&k_full[i], SPANS ? PRODUCERS : 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], SPANS ? PRODUCERS : 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], BM);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(drain, 1);
    fence_mbarrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (trace && tid == 0) trace[1] = global_timer_ns();
  auto fail = [&]() { atomicOr(&failed, 1); };
  auto is_failed = [&]() { return *reinterpret_cast<volatile int*>(&failed) != 0; };

  if (SPANS && (warp == 8 || warp == 10 || warp == 11)) {
    // ---------------- span producers.  Half-tiles h = 2g (K of the CTA's
    // g-th tile) and 2g + 1 (V of it) are filled in order, each as one
    // cp.async group; half-tile h - 1 is published (its copies waited for,
    // proxy fence, arrive) only once half-tile h is in flight, so K and V
    // loads overlap like TMA loads do.  A half-tile's stage is released by
    // the MMA thread; the producer runs at most one half-tile ahead of what
    // it has published, which is what the MMA loop needs to release that
    // stage, so the two cannot wait on each other.
    const int pid = (warp == 8 ? 0 : warp - 9) * 32 + lane;
    auto publish = [&](int h) {
      fence_proxy_async_smem();  // generic-proxy writes, read by the tensor core (async proxy)
      mbar_arrive((h & 1) ? &v_full[(h >> 1) % STAGES] : &k_full[(h >> 1) % STAGES]);
    };
    int filled = 0, g0 = 0;
    bool ok = true;
    for (int it = ib; it < ie && ok; ++it) {
      const Item I = load_item<SPANS>(P, staged, it, tid);
      const ucb_span* spans = P.spans + I.span_begin;
      const int nt = tiles_of(I);
      for (int h = 2 * g0; h < 2 * (g0 + nt); ++h) {
        if (is_failed()) {
          ok = false;
          break;
        }
        const int g = h >> 1, j = g - g0, st = g % STAGES;
        const bool keys = (h & 1) == 0;
        if (g >= STAGES && !mbar_wait_for(keys ? &k_empty[st] : &v_empty[st], ((g / STAGES) - 1) & 1, WAIT_NS)) {
          fail();
          ok = false;
          break;
        }
        const int tok0 = I.k0 + j * BN, valid = min(BN, I.n_tokens - j * BN);
        fill_tile(keys, spans, I.span_count, tok0, valid, P.k_bits, P.v_bits, P.group,
                  smem + (keys ? OFF_K + st * KTILE : OFF_V + st * VTILE), pid);
        cp_async_commit();
        filled = h + 1;
        if (h > 0) {
          cp_async_wait_one();  // every group but the newest (half-tile h) has landed
          publish(h - 1);
        }
      }
      g0 += nt;
    }
    cp_async_wait_all();
    if (filled > 0) publish(filled - 1);
  } else if (!SPANS && warp == 8) {
    // ---------------- loader
    if (lane == 0) {
      int issued = 0, g = 0;
      bool ok = true;
      for (int it = ib; it < ie && ok; ++it) {
        const Item I = load_item<SPANS>(P, staged, it, tid);
        if (!staged) {  // workspace launches run one item
          mbar_arrive_expect_tx(q_full, 2 * QTILE);
          for (int x = 0; x < 2; ++x) {
            tma_load_3d(smem + OFF_Q + x * QTILE, &tm_q, 0, I.m0 + x * BM, I.head, q_full);
            tma_load_3d(smem + OFF_Q + x * QTILE + QHALF, &tm_q, 64, I.m0 + x * BM, I.head, q_full);
          }
        }
        const int nt = tiles_of(I);
        for (int j = 0; j < nt; ++j, ++g) {
          const int st = g % STAGES;
          const uint32_t ph = ((g / STAGES) - 1) & 1;
          if (is_failed() ||
              (g >= STAGES && (!mbar_wait_for(&k_empty[st], ph, WAIT_NS) || !mbar_wait_for(&v_empty[st], ph, WAIT_NS)))) {
            fail();
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], KTILE);
          tma_load_3d(smem + OFF_K + st * KTILE, &tm_k, 0, I.k0 + j * BN, I.head, &k_full[st]);
          tma_load_3d(smem + OFF_K + st * KTILE + KHALF, &tm_k, 64, I.k0 + j * BN, I.head, &k_full[st]);
          mbar_arrive_expect_tx(&v_full[st], VTILE);
          tma_load_3d(smem + OFF_V + st * VTILE, &tm_v, I.k0 + j * BN, 0, I.head, &v_full[st]);
          tma_load_3d(smem + OFF_V + st * VTILE + VHALF, &tm_v, I.k0 + j * BN + 64, 0, I.head, &v_full[st]);
          issued = g + 1;
        }
        if (!staged) break;
      }
      // Copies still in flight must land before the shared memory is released.
      if (!staged) mbar_wait_for(q_full, 0, WAIT_NS);
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j) {
        mbar_wait_for(&k_full[j % STAGES], (j / STAGES) & 1, WAIT_NS);
        mbar_wait_for(&v_full[j % STAGES], (j / STAGES) & 1, WAIT_NS);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer.  Order on the tensor core per item: S_A(0)
    // S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ..., so that while one
    // tile's softmax runs the other tile's products are in flight.  g counts
    // the CTA's tiles over all its items (ring stages and phases).
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(smem + OFF_Q);
      auto issue_s = [&](int g, int x) {
        const uint32_t k_addr = smem_u32(smem + OFF_K + (g % STAGES) * KTILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t col = (kk & 3) * 32;
          tc_mma(tmem + S_COL + 128 * x, sw128_desc(q_addr + x * QTILE + (kk >> 2) * QHALF + col),
                 sw128_desc(k_addr + (kk >> 2) * KHALF + col), IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[x]);
      };
      auto issue_pv = [&](int g, int j, int x) {
        const uint32_t v_addr = smem_u32(smem + OFF_V + (g % STAGES) * VTILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {  // P_x: 8 TMEM columns (16 tokens) per step
          if constexpr (SPANS)  // V rows = tokens: 16 tokens = two 8-row groups = 2048 bytes
            tc_mma_ts(tmem + O_COL + 128 * x, tmem + S_COL + 128 * x + 8 * kk, sw128_mn_desc(v_addr + kk * 2048),
                      IDESC_O_MN, (j > 0 || kk > 0) ? 1u : 0u);
          else  // V^T rows = channels: 16 tokens = 32 bytes of a 64-token half
            tc_mma_ts(tmem + O_COL + 128 * x, tmem + S_COL + 128 * x + 8 * kk,
                      sw128_desc(v_addr + (kk >> 2) * VHALF + (kk & 3) * 32), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&o_done[x]);
      };
      bool ok = true;
      int g = 0;
      uint64_t wait_kv = 0, wait_p = 0;  // diagnostics (trace): time spent waiting for K/V tiles and for P
      auto timed_wait = [&](uint64_t* bar, uint32_t ph, uint64_t& acc) {
        if (!trace) return mbar_wait_for(bar, ph, WAIT_NS);
        const uint64_t t0 = global_timer_ns();
        const bool r = mbar_wait_for(bar, ph, WAIT_NS);
        acc += global_timer_ns() - t0;
        return r;
      };
      for (int it = ib, n = 0; it < ie && ok; ++it, ++n) {
        const Item I = load_item<SPANS>(P, staged, it, tid);
        const int nt = tiles_of(I);
        ok = mbar_wait_for(q_full, n & 1, WAIT_NS) &&
             (nt == 0 || mbar_wait_for(&k_full[g % STAGES], (g / STAGES) & 1, WAIT_NS));
        if (!ok || nt == 0) continue;
        tc_fence_after();
        issue_s(g, 0);
        issue_s(g, 1);
        tc_commit(&k_empty[g % STAGES]);
        for (int j = 0; j < nt && ok; ++j) {
          const int gj = g + j, st = gj % STAGES, st1 = (gj + 1) % STAGES;
          const bool more = j + 1 < nt;
          ok = timed_wait(&v_full[st], (gj / STAGES) & 1, wait_kv) && timed_wait(&p_full[0], gj & 1, wait_p);
          if (!ok) break;
          tc_fence_after();
          issue_pv(gj, j, 0);
          if (more) {
            ok = timed_wait(&k_full[st1], ((gj + 1) / STAGES) & 1, wait_kv);
            if (!ok) break;
            tc_fence_after();
            issue_s(gj + 1, 0);
          }
          ok = timed_wait(&p_full[1], gj & 1, wait_p);
          if (!ok) break;
          tc_fence_after();
          issue_pv(gj, j, 1);
          tc_commit(&v_empty[st]);
          if (more) {
            issue_s(gj + 1, 1);
            tc_commit(&k_empty[st1]);
          }
        }
        g += nt;
      }
      if (!ok) fail();
      if (trace) {
        trace[30] = wait_kv;
        trace[31] = wait_p;
      }
      // Everything issued has finished before TMEM can be released.
      tc_commit(drain);
      mbar_wait_for(drain, 0, WAIT_NS);
    }
  } else if (warp < 8) {
    // ---------------- softmax warpgroups
    const int x = warp >> 2;             // tile
    const int row = tid & (BM - 1);      // query row in the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t t_s = tmem + S_COL + 128 * x + lane_off, t_o = tmem + O_COL + 128 * x + lane_off;
    const int r_blk = x * BM + row;  // row within the item's 2*BM-row block
    int g = 0, it = ib;
    for (; it < ie; ++it) {
      const Item I = load_item<SPANS>(P, staged, it, tid);
      const int nt = tiles_of(I);
      if (caller_layout) {
        // caller-layout Q_A and Q_B of this item: every tensor-core operation
        // of the previous item has completed (its last O hand-off was
        // waited for), so the Q tiles are free
        load_q_caller(P, smem, I.m0, I.m_end, I.pos0, I.head, tid, Q_THREADS);
        cp_async_wait_all();
        fence_proxy_async_smem();  // generic-proxy writes, read by the tensor core (async proxy)
        mbar_arrive(q_full);
      }
      if (trace && tid == 0 && it - ib < 12) trace[6 + 2 * (it - ib)] = global_timer_ns();
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        const int gj = g + j;
        ok = mbar_wait_for(&s_full[x], gj & 1, WAIT_NS);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        const int valid = min(BN, I.n_tokens - j * BN);
        uint32_t s0[2][32];
        const float mx =
            (valid < BN ? row_max_keep<true>(t_s, valid, s0) : row_max_keep<false>(t_s, valid, s0)) * P.scale_log2;
        // P_x(j-1) consumed and O_x(j-1) complete before this tile writes either.
        if (j > 0) {
          ok = mbar_wait_for(&o_done[x], (gj - 1) & 1, WAIT_NS);
          if (!__all_sync(0xffffffffu, ok)) break;
          tc_fence_after();
        }
        const bool move = mx > m_run + RESCALE_THRESHOLD || m_run == -INFINITY;
        if (__any_sync(0xffffffffu, move)) {
          const float m_new = move ? fmaxf(mx, m_run) : m_run;
          const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
          if (j > 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t ov[32];
              tc_ld32(t_o + 32 * c, ov);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float2 v = __fmul2_rn(make_float2(__uint_as_float(ov[i]), __uint_as_float(ov[i + 1])),
                                            make_float2(alpha, alpha));
                ov[i] = __float_as_uint(v.x);
                ov[i + 1] = __float_as_uint(v.y);
              }
              tc_st32(t_o + 32 * c, ov);
            }
            tc_wait_st();
          }
          l_run *= alpha;
          m_run = m_new;
        }
        l_run += valid < BN ? write_p_keep<true>(s0, t_s, valid, P.scale_log2, -m_run)
                            : write_p_keep<false>(s0, t_s, valid, P.scale_log2, -m_run);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
      }
      if (ok && nt > 0) ok = mbar_wait_for(&o_done[x], (g + nt - 1) & 1, WAIT_NS);
      tc_fence_after();
      const bool good = __all_sync(0xffffffffu, ok);
      write_item_result(P, I, caller_layout, good, nt, r_blk, lane, t_o, m_run, l_run, &failed);
      // The softmax warps meet once per item: a partial is published after
      // every row is written; consumed partials' flags advance after every
      // row is read.  A failed item still settles its flags (its CTA has set
      // the error word), so the parity stays in step.
      // After a failure anywhere in the CTA every softmax warp stops at the
      // same item (thread 0's reading of the failure word, shared between
      // two barriers), so no warp waits at a barrier the others have left.
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (tid == 0) {
        settle_flags(P, I);
        stop_items = is_failed() ? 1 : 0;
        if (trace && it - ib < 12) trace[6 + 2 * (it - ib) + 1] = global_timer_ns();
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      g += nt;
      if (stop_items) {
        ++it;
        break;
      }
    }
    // items this CTA could not reach after a failure still settle their flags
    if (tid == 0)
      for (; it < ie; ++it) settle_flags(P, load_item<SPANS>(P, staged, it, 1));
  }
  tc_fence_before();
  __syncthreads();
  if (failed && tid == 0) atomicOr(P.err, DEVERR_MBAR_TIMEOUT);
  if (trace && tid == 0) {
    trace[3] = global_timer_ns();
    trace[4] = (uint64_t)n_items;
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D bf16 tensor map {x: inner, y, z} with a {64, box_y, 1} box and 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint32_t box_y) {
  auto fn = encode_fn();
  if (!fn) return ucb_host::set_error(UCB_ERR_CUDA, "prefill: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {x, y, z};
  const cuuint64_t strides[2] = {x * 2, x * y * 2};
  const cuuint32_t box[3] = {64, box_y, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ucb_host::set_error(UCB_ERR_CUDA, "prefill: tensor map encoding failed (%d)", (int)r);
  return UCB_OK;
}

}  // namespace prefill
}  // namespace ucb

namespace {
uint64_t* g_prefill_trace = nullptr;  // diagnostics only; see ucb_prefill_set_trace
}  // namespace

extern "C" int ucb_prefill_set_trace(void* trace_dev) {
  g_prefill_trace = static_cast<uint64_t*>(trace_dev);
  return UCB_OK;
}

namespace {
// q == k == vt == nullptr: a segment-table launch (keys and values from
// P.spans).  q == nullptr with k and vt: a staged launch (caller-layout query
// in P.q, keys and values from the staging workspace k [heads, n_padded, 128]
// and vt [heads, 128, n_padded]).
int launch_prefill(const void* q, const void* k, const void* vt, int heads, int m_rows, int n_padded,
                   ucb::prefill::Params P, dim3 grid, void* stream) {
  using namespace ucb::prefill;
  const bool spans = (q == nullptr && k == nullptr);
  const bool staged = (q == nullptr && k != nullptr);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(vt)) & 15)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention: operands must be 16-byte aligned");
  if (!spans && n_padded % 8)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention: n_padded must be a multiple of 8");
  unsigned int* err = ucb_host::device_error_word();
  if (!err) return ucb_host::set_error(UCB_ERR_CUDA, "ucb_prefill_attention: device error word unavailable");
  CUtensorMap tq, tk, tv;
  if (spans) {
    memset(&tq, 0, sizeof(tq));  // unused by the segment-table kernel
    tk = tv = tq;
  } else if (staged) {
    memset(&tq, 0, sizeof(tq));  // the query is loaded in the caller's layout
    int rc = make_map(&tk, k, D, (uint64_t)n_padded, (uint64_t)heads, BN);
    if (!rc) rc = make_map(&tv, vt, (uint64_t)n_padded, D, (uint64_t)heads, D);
    if (rc) return rc;
  } else {
    int rc = make_map(&tq, q, D, (uint64_t)m_rows, (uint64_t)heads, BM);
    if (!rc) rc = make_map(&tk, k, D, (uint64_t)n_padded, (uint64_t)heads, BN);
    if (!rc) rc = make_map(&tv, vt, (uint64_t)n_padded, D, (uint64_t)heads, D);
    if (rc) return rc;
  }
  static bool configured[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[spans][dev]) {
    const cudaError_t e = spans ? cudaFuncSetAttribute(prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM)
                                : cudaFuncSetAttribute(prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess)
      return ucb_host::set_error(UCB_ERR_CUDA, "prefill: cannot reserve %d bytes of shared memory", SMEM);
    if (dev >= 0 && dev < 64) configured[spans][dev] = true;
  }
  P.err = err;
  P.trace = g_prefill_trace;
  if (spans)
    prefill_kernel<true><<<grid, THREADS, SMEM, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, P);
  else
    prefill_kernel<false><<<grid, THREADS, SMEM, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, P);
  return ucb_host::check_launch("prefill_kernel");
}
}  // namespace

extern "C" int ucb_prefill_attention(const void* q, const void* k, const void* vt, int heads, int m_rows,
                                     int n_tokens, int n_padded, float softmax_scale, void* out, float* lse,
                                     void* stream) {
  using namespace ucb::prefill;
  if (!q || !k || !vt || !out) return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention: null pointer");
  if (heads <= 0 || m_rows <= 0 || n_tokens <= 0)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention: empty problem");
  if (n_padded < n_tokens)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention: n_padded must be >= n_tokens");
  Params P;
  P.m_rows = m_rows;
  P.n_tokens = n_tokens;
  P.scale_log2 = softmax_scale * 1.4426950408889634f;
  P.items = nullptr;
  P.lq_items = nullptr;
  P.spans = nullptr;
  P.k_bits = P.v_bits = P.group = 0;
  P.q = nullptr;
  P.hq = P.grp = P.positions = 0;
  P.partials = nullptr;
  P.flags = nullptr;
  P.cta_items = nullptr;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.lse = lse;
  return launch_prefill(q, k, vt, heads, m_rows, n_padded, P, dim3((m_rows + 2 * BM - 1) / (2 * BM), heads), stream);
}

extern "C" int ucb_prefill_attention_items(const void* q, const void* k, const void* vt, int heads, int m_rows,
                                           int n_padded, const void* items, int num_items, float softmax_scale,
                                           void* out, float* lse, float* partials, unsigned int* flags,
                                           void* stream) {
  using namespace ucb::prefill;
  if (!q || !k || !vt || !out || !items)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention_items: null pointer");
  if (heads <= 0 || m_rows <= 0 || n_padded <= 0 || num_items <= 0)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention_items: empty problem");
  if ((partials == nullptr) != (flags == nullptr))
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_prefill_attention_items: partials and flags go together");
  Params P;
  P.m_rows = m_rows;
  P.n_tokens = 0;
  P.scale_log2 = softmax_scale * 1.4426950408889634f;
  P.items = static_cast<const WorkItem*>(items);
  P.lq_items = nullptr;
  P.spans = nullptr;
  P.k_bits = P.v_bits = P.group = 0;
  P.q = nullptr;
  P.hq = P.grp = P.positions = 0;
  P.partials = partials;
  P.flags = flags;
  P.cta_items = nullptr;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.lse = lse;
  return launch_prefill(q, k, vt, heads, m_rows, n_padded, P, dim3(num_items), stream);
}

extern "C" int ucb_prefill_attention_batched(const void* q, const void* k, const void* vt, int heads, int m_rows,
                                             int n_padded, const void* items, int num_items, float softmax_scale,
                                             void* out, float* lse, void* stream) {
  return ucb_prefill_attention_items(q, k, vt, heads, m_rows, n_padded, items, num_items, softmax_scale, out, lse,
                                     nullptr, nullptr, stream);
}

extern "C" int64_t ucb_prefill_partial_bytes() {
  return (int64_t)ucb::prefill::PARTIAL_SLOT_FLOATS * (int64_t)sizeof(float);
}

namespace {
int check_lq_common(const char* fn, const void* q, int positions, int num_q_heads, int num_kv_heads,
                    const void* items, int num_items, const ucb_span* spans, int num_spans, int k_bits, int v_bits,
                    int group_size, const void* out, const float* partials, const unsigned int* flags) {
  if (!q || !items || !spans || !out) return ucb_host::set_error(UCB_ERR_INVALID, "%s: null pointer", fn);
  if (positions <= 0 || num_items <= 0 || num_spans <= 0)
    return ucb_host::set_error(UCB_ERR_INVALID, "%s: empty problem", fn);
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads)
    return ucb_host::set_error(UCB_ERR_INVALID, "%s: query heads must be a multiple of KV heads", fn);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return ucb_host::set_error(UCB_ERR_INVALID, "%s: query/out must be 16-byte aligned", fn);
  if ((k_bits != 2 && k_bits != 4) || (v_bits != 2 && v_bits != 4))
    return ucb_host::set_error(UCB_ERR_UNSUPPORTED, "%s: packed spans must be 2- or 4-bit", fn);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return ucb_host::set_error(UCB_ERR_UNSUPPORTED, "%s: group_size must be 32, 64 or 128", fn);
  if ((partials == nullptr) != (flags == nullptr))
    return ucb_host::set_error(UCB_ERR_INVALID, "%s: partials and flags go together", fn);
  return UCB_OK;
}
}  // namespace

extern "C" int ucb_long_query_attention(const void* q, int positions, int num_q_heads, int num_kv_heads,
                                        const void* items, int num_items, const ucb_span* spans, int num_spans,
                                        int k_bits, int v_bits, int group_size, float softmax_scale, void* out,
                                        float* lse, float* partials, unsigned int* flags, void* stream) {
  using namespace ucb::prefill;
  const int rc = check_lq_common("ucb_long_query_attention", q, positions, num_q_heads, num_kv_heads, items,
                                 num_items, spans, num_spans, k_bits, v_bits, group_size, out, partials, flags);
  if (rc) return rc;
  Params P;
  P.m_rows = 0;
  P.n_tokens = 0;
  P.scale_log2 = softmax_scale * 1.4426950408889634f;
  P.items = nullptr;
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.hq = num_q_heads;
  P.grp = num_q_heads / num_kv_heads;
  P.positions = positions;
  P.lq_items = static_cast<const LqItem*>(items);
  P.spans = spans;
  P.k_bits = k_bits;
  P.v_bits = v_bits;
  P.group = group_size;
  P.partials = partials;
  P.flags = flags;
  P.cta_items = nullptr;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.lse = lse;
  return launch_prefill(nullptr, nullptr, nullptr, 0, 0, 0, P, dim3(num_items), stream);
}


extern "C" int ucb_long_query_stage(const ucb_span* spans, int num_spans, const void* jobs, int num_jobs,
                                    int max_chunks, int k_bits, int v_bits, int group_size, void* k_ws,
                                    void* vt_ws, int64_t ws_rows, void* stream) {
  using namespace ucb::prefill;
  if (!spans || !jobs || !k_ws || !vt_ws) return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_stage: null pointer");
  if (num_spans <= 0 || num_jobs <= 0 || max_chunks <= 0 || num_jobs > 65535)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_stage: bad job grid");
  if (ws_rows <= 0 || ws_rows % BN || (int64_t)max_chunks * STAGE_T > ws_rows)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_stage: ws_rows must be a positive multiple of 128 "
                                                "covering max_chunks * 64 rows");
  if ((reinterpret_cast<uintptr_t>(k_ws) | reinterpret_cast<uintptr_t>(vt_ws)) & 15)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_stage: workspaces must be 16-byte aligned");
  if ((k_bits != 2 && k_bits != 4) || (v_bits != 2 && v_bits != 4))
    return ucb_host::set_error(UCB_ERR_UNSUPPORTED, "ucb_long_query_stage: packed spans must be 2- or 4-bit");
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return ucb_host::set_error(UCB_ERR_UNSUPPORTED, "ucb_long_query_stage: group_size must be 32, 64 or 128");
  const dim3 grid(max_chunks, num_jobs);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const StageJob* J = static_cast<const StageJob*>(jobs);
  __nv_bfloat16* K = static_cast<__nv_bfloat16*>(k_ws);
  __nv_bfloat16* VT = static_cast<__nv_bfloat16*>(vt_ws);
  if (k_bits == 2 && v_bits == 2) stage_kernel<2, 2><<<grid, STAGE_THREADS, 0, st>>>(J, spans, group_size, K, VT, ws_rows);
  else if (k_bits == 2) stage_kernel<2, 4><<<grid, STAGE_THREADS, 0, st>>>(J, spans, group_size, K, VT, ws_rows);
  else if (v_bits == 2) stage_kernel<4, 2><<<grid, STAGE_THREADS, 0, st>>>(J, spans, group_size, K, VT, ws_rows);
  else stage_kernel<4, 4><<<grid, STAGE_THREADS, 0, st>>>(J, spans, group_size, K, VT, ws_rows);
  return ucb_host::check_launch("stage_kernel");
}

extern "C" int ucb_long_query_attention_staged(const void* q, int positions, int num_q_heads, int num_kv_heads,
                                               const void* items, int num_items, const int32_t* cta_items,
                                               int num_ctas, const ucb_span* spans, int num_spans, const void* jobs,
                                               int num_jobs, int max_chunks, int k_bits, int v_bits,
                                               int group_size, float softmax_scale, void* k_ws, void* vt_ws,
                                               int64_t ws_rows, void* out, float* lse, float* partials,
                                               unsigned int* flags, void* stream) {
  using namespace ucb::prefill;
  int rc = check_lq_common("ucb_long_query_attention_staged", q, positions, num_q_heads, num_kv_heads, items,
                           num_items, spans, num_spans, k_bits, v_bits, group_size, out, partials, flags);
  if (rc) return rc;
  if (ws_rows > (int64_t)1 << 30)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_attention_staged: workspace too large");
  if (cta_items && (num_ctas <= 0 || num_ctas > num_items))
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_long_query_attention_staged: num_ctas must be in [1, num_items]");
  rc = ucb_long_query_stage(spans, num_spans, jobs, num_jobs, max_chunks, k_bits, v_bits, group_size, k_ws, vt_ws,
                            ws_rows, stream);
  if (rc) return rc;
  Params P;
  P.m_rows = 0;
  P.n_tokens = 0;
  P.scale_log2 = softmax_scale * 1.4426950408889634f;
  P.items = nullptr;
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.hq = num_q_heads;
  P.grp = num_q_heads / num_kv_heads;
  P.positions = positions;
  P.lq_items = static_cast<const LqItem*>(items);
  P.spans = spans;
  P.k_bits = k_bits;
  P.v_bits = v_bits;
  P.group = group_size;
  P.partials = partials;
  P.flags = flags;
  P.cta_items = cta_items;
  P.out = static_cast<__nv_bfloat16*>(out);
  P.lse = lse;
  return launch_prefill(nullptr, k_ws, vt_ws, num_kv_heads, 0, (int)ws_rows, P, dim3(cta_items ? num_ctas : num_items), stream);
}
