// Sequence-split merge over NVLink peer memory.
//
// A sequence split across GPUs ends every decode step with an exchange of each
// rank's (out, LSE) summary and an LSE merge (the reference's
// merge_attention_summaries, unicache/adapters/bagel.py:57-72, applied across
// ranks).  Instead of a library all-gather followed by a merge kernel, one
// kernel per rank does both:
//
//  * every rank owns one exchange buffer (cudaMalloc'd, shared with its peers
//    through CUDA IPC handles); rank r sends its summary into slot r of every
//    peer's buffer with plain 8-byte peer stores over NVLink (no multicast),
//    each word carrying 4 bytes of data and the step's epoch, so a word is
//    valid exactly when its epoch matches: no fence and no separate flag;
//  * it then reads every peer's words from its OWN buffer, polling each until
//    its epoch matches (bounded), and merges them with its own summary in rank
//    order with the arithmetic of ucb_lse_merge.
//
// Buffer layout: [epoch counter u32 | pad to 256 B][slots: 2 parities x
// MAX_RANKS x rows * 65 words of 8 bytes (rows * 64 data words of two bf16,
// then rows LSE words)].  The epoch is a device-side counter in the buffer that
// the kernel itself increments, so replays of a captured graph advance it too;
// every rank makes the same sequence of calls, so epochs agree.  Slots
// alternate by epoch parity: a rank can send step e+2 (the parity of step e)
// only after every peer sent step e+1, which a peer does only after its merge
// of step e finished, so no send overwrites a word still to be read.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"

namespace ucb {
namespace peer {

constexpr int MAX_RANKS = 8;
constexpr int HEADER_BYTES = 256;            // epoch counter at 0
constexpr uint64_t WAIT_NS = 1000000000ull;  // 1 s
constexpr int THREADS = 512;

struct PeerArgs {
  unsigned char* bufs[MAX_RANKS];  // every rank's buffer as mapped here; bufs[rank] is local
};

__host__ __device__ constexpr int64_t slot_words(int64_t rows) { return rows * 65; }

__device__ __forceinline__ void st_word(uint64_t* p, uint32_t data, uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | data;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Polls one word until its epoch matches; false once the deadline has passed.
__device__ __forceinline__ bool ld_word(const uint64_t* p, uint32_t epoch, uint64_t deadline, uint32_t& data) {
  while (true) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    if ((uint32_t)(v >> 32) == epoch) {
      data = (uint32_t)v;
      return true;
    }
    if (global_timer_ns() > deadline) return false;
  }
}

// rows = B * Hq summary rows of 128 channels.
__global__ void __launch_bounds__(THREADS, 1)
    split_merge_kernel(PeerArgs a, int rank, int world, const __nv_bfloat16* __restrict__ out_local,
                       const float* __restrict__ lse_local, int rows, __nv_bfloat16* __restrict__ out,
                       float* __restrict__ lse, unsigned int* err) {
  __shared__ unsigned int epoch_s;
  unsigned char* own = a.bufs[rank];
  if (threadIdx.x == 0) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(own);
    epoch_s = *counter + 1u;
    *counter = epoch_s;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int64_t sw = slot_words(rows);
  const int64_t parity_off = (int64_t)(epoch & 1u) * MAX_RANKS * sw;
  const uint32_t* o32 = reinterpret_cast<const uint32_t*>(out_local);
  // 1. send this rank's words into slot `rank` of every peer's buffer
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    uint64_t* dst = reinterpret_cast<uint64_t*>(a.bufs[p] + HEADER_BYTES) + parity_off + rank * sw;
    for (int w = threadIdx.x; w < rows * 64; w += blockDim.x) st_word(dst + w, o32[w], epoch);
    for (int r = threadIdx.x; r < rows; r += blockDim.x)
      st_word(dst + rows * 64 + r, __float_as_uint(lse_local[r]), epoch);
  }
  // 2. merge: warp per summary row, rank order, the arithmetic of ucb_lse_merge
  const uint64_t deadline = global_timer_ns() + WAIT_NS;
  const uint64_t* slots = reinterpret_cast<const uint64_t*>(own + HEADER_BYTES) + parity_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  bool ok = true;
  for (int r = warp; r < rows; r += warps) {
    float lp[MAX_RANKS];
    uint32_t d0[MAX_RANKS], d1[MAX_RANKS];
    float peak = -INFINITY;
    for (int p = 0; p < world; ++p) {
      if (p == rank) {
        lp[p] = lse_local[r];
        d0[p] = o32[(int64_t)r * 64 + 2 * lane];
        d1[p] = o32[(int64_t)r * 64 + 2 * lane + 1];
      } else {
        const uint64_t* sp = slots + p * sw;
        uint32_t lbits = 0;
        ok = ok && ld_word(sp + rows * 64 + r, epoch, deadline, lbits);
        ok = ok && ld_word(sp + (int64_t)r * 64 + 2 * lane, epoch, deadline, d0[p]);
        ok = ok && ld_word(sp + (int64_t)r * 64 + 2 * lane + 1, epoch, deadline, d1[p]);
        lp[p] = __uint_as_float(lbits);
      }
      peak = fmaxf(peak, lp[p]);
    }
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    float sum = 0.f;
    if (peak != -INFINITY) {
      for (int p = 0; p < world; ++p) sum += expf(lp[p] - peak);
    }
    const float total = (peak == -INFINITY) ? -INFINITY : peak + logf(sum);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < world; ++p) {
      const float w = expf(lp[p] - total);
      const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&d0[p]);
      const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&d1[p]);
      acc[0] = fmaf(__bfloat162float(lo.x), w, acc[0]);
      acc[1] = fmaf(__bfloat162float(lo.y), w, acc[1]);
      acc[2] = fmaf(__bfloat162float(hi.x), w, acc[2]);
      acc[3] = fmaf(__bfloat162float(hi.y), w, acc[3]);
    }
    __nv_bfloat162 o0 = __floats2bfloat162_rn(acc[0], acc[1]);
    __nv_bfloat162 o1 = __floats2bfloat162_rn(acc[2], acc[3]);
    uint2 o;
    o.x = *reinterpret_cast<unsigned int*>(&o0);
    o.y = *reinterpret_cast<unsigned int*>(&o1);
    reinterpret_cast<uint2*>(out)[(int64_t)r * 32 + lane] = o;
    if (lane == 0 && lse) lse[r] = total;
  }
  if (!__syncthreads_and(ok) && threadIdx.x == 0) atomicOr(err, DEVERR_MBAR_TIMEOUT);
}

}  // namespace peer
}  // namespace ucb

using ucb_host::check_launch;
using ucb_host::set_error;

extern "C" int64_t ucb_peer_buffer_bytes(int64_t rows) {
  if (rows <= 0) return 0;
  return ucb::peer::HEADER_BYTES + 2LL * ucb::peer::MAX_RANKS * ucb::peer::slot_words(rows) * 8;
}

extern "C" int ucb_peer_buffer_alloc(int64_t bytes, void** ptr, void* handle_out) {
  if (bytes <= 0 || !ptr || !handle_out) return set_error(UCB_ERR_INVALID, "ucb_peer_buffer_alloc: bad arguments");
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess)
    return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_alloc: cudaMalloc of %lld bytes failed", (long long)bytes);
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_alloc: clearing the buffer failed");
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_alloc: cudaIpcGetMemHandle failed");
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return UCB_OK;
}

extern "C" int ucb_peer_buffer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return set_error(UCB_ERR_INVALID, "ucb_peer_buffer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_open: cudaIpcOpenMemHandle failed");
  *ptr = p;
  return UCB_OK;
}

extern "C" int ucb_peer_buffer_close(void* ptr) {
  if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_close failed");
  return UCB_OK;
}

extern "C" int ucb_peer_buffer_free(void* ptr) {
  if (ptr && cudaFree(ptr) != cudaSuccess) return set_error(UCB_ERR_CUDA, "ucb_peer_buffer_free failed");
  return UCB_OK;
}

extern "C" int ucb_split_merge_peer(int rank, int world, void* const* bufs, const void* out_local,
                                    const float* lse_local, int64_t rows, int head_dim, void* out, float* lse,
                                    void* stream) {
  if (world < 1 || world > ucb::peer::MAX_RANKS || rank < 0 || rank >= world)
    return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: rank/world out of range (world <= %d)",
                     ucb::peer::MAX_RANKS);
  if (head_dim != 128) return set_error(UCB_ERR_UNSUPPORTED, "ucb_split_merge_peer: head_dim must be 128");
  if (rows <= 0 || rows > (1 << 20)) return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: bad row count");
  if (!bufs || !out_local || !lse_local || !out)
    return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: null pointer");
  if ((reinterpret_cast<uintptr_t>(out_local) | reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: out rows must be 16-byte aligned");
  // The kernel sends a row's words to the peers and merges without a barrier
  // in between, so the merged result must not overwrite the rank's own summary.
  if (out == out_local || (lse != nullptr && lse == lse_local))
    return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: out/lse must not alias out_local/lse_local");
  ucb::peer::PeerArgs a;
  for (int i = 0; i < ucb::peer::MAX_RANKS; ++i) a.bufs[i] = nullptr;
  for (int i = 0; i < world; ++i) {
    if (!bufs[i] || (reinterpret_cast<uintptr_t>(bufs[i]) & 255))
      return set_error(UCB_ERR_INVALID, "ucb_split_merge_peer: buffer %d missing or not 256-byte aligned", i);
    a.bufs[i] = static_cast<unsigned char*>(bufs[i]);
  }
  unsigned int* err = ucb_host::device_error_word();
  if (!err) return set_error(UCB_ERR_CUDA, "ucb_split_merge_peer: device error word unavailable");
  ucb::peer::split_merge_kernel<<<1, ucb::peer::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      a, rank, world, static_cast<const __nv_bfloat16*>(out_local), lse_local, (int)rows,
      static_cast<__nv_bfloat16*>(out), lse, err);
  return check_launch("split_merge_kernel");
}
