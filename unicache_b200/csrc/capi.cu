// Error reporting, device status word and the tensor-core self test.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = {0};

// Device error word: kernels OR DeviceError bits into it instead of trapping.
__device__ unsigned int g_error_word = 0;

constexpr int kMaxDevices = 64;
unsigned int* g_error_word_ptr[kMaxDevices] = {nullptr};
}  // namespace

namespace ucb_host {

int set_error(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(UCB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return UCB_OK;
}

unsigned int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_error_word_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_error_word) != cudaSuccess) return nullptr;
    g_error_word_ptr[dev] = static_cast<unsigned int*>(ptr);
  }
  return g_error_word_ptr[dev];
}

}  // namespace ucb_host

extern "C" const char* ucb_last_error(void) { return g_last_error; }

extern "C" int ucb_version(void) { return 100; }

extern "C" int ucb_device_status(unsigned int* flags, void* stream) {
  unsigned int* word = ucb_host::device_error_word();
  if (word == nullptr) return ucb_host::set_error(UCB_ERR_CUDA, "device error word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int value = 0;
  if (cudaMemcpyAsync(&value, word, sizeof(value), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemsetAsync(word, 0, sizeof(unsigned int), s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    return ucb_host::set_error(UCB_ERR_CUDA, "reading the device error word failed");
  }
  if (flags) *flags = value;
  return UCB_OK;
}

// One warp: A = codes c in [0,3] placed at bit 2*(row%4) of an fp16 subnormal,
// B = ordinary fp16 values; compare mma.sync against an fp32 sum.
__global__ void selftest_mma_kernel(float* max_err) {
  const int lane = threadIdx.x;
  const int r = lane >> 2, c = lane & 3;
  __shared__ float A[16][16], B[16][8];
  __shared__ float err[32];
  for (int i = lane; i < 256; i += 32) {
    int row = i / 16, col = i % 16;
    int code = (row * 7 + col * 3) & 3;
    A[row][col] = ldexpf(static_cast<float>(code), 2 * (row % 4) - 24);
  }
  for (int i = lane; i < 128; i += 32) {
    int k = i / 8, n = i % 8;
    B[k][n] = __half2float(__float2half_rn(0.37f * (k - 7) + 0.11f * n * n - 0.5f));
  }
  __syncwarp();
  auto h2 = [](float lo, float hi) { return ucb::pack_f16x2(lo, hi); };
  uint32_t a[4] = {h2(A[r][2 * c], A[r][2 * c + 1]), h2(A[r + 8][2 * c], A[r + 8][2 * c + 1]),
                   h2(A[r][2 * c + 8], A[r][2 * c + 9]), h2(A[r + 8][2 * c + 8], A[r + 8][2 * c + 9])};
  uint32_t b0 = h2(B[2 * c][r], B[2 * c + 1][r]);
  uint32_t b1 = h2(B[2 * c + 8][r], B[2 * c + 9][r]);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  ucb::mma_f16(d, a, b0, b1);
  float worst = 0.f;
  const int rows[4] = {r, r, r + 8, r + 8};
  const int cols[4] = {2 * c, 2 * c + 1, 2 * c, 2 * c + 1};
  for (int e = 0; e < 4; ++e) {
    float ref = 0.f;
    for (int k = 0; k < 16; ++k) ref += A[rows[e]][k] * B[k][cols[e]];
    // Compare at unit scale: undo the 2^-24 subnormal offset of the codes.
    worst = fmaxf(worst, fabsf(ldexpf(d[e] - ref, 24)));
  }
  err[lane] = worst;
  __syncwarp();
  if (lane == 0) {
    float m = 0.f;
    for (int i = 0; i < 32; ++i) m = fmaxf(m, err[i]);
    *max_err = m;
  }
}

extern "C" int ucb_selftest_mma_subnormal(float* max_abs_err, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* d_err = nullptr;
  // The self test is a diagnostic outside the hot path; it owns its tiny buffer.
  if (cudaMallocAsync(&d_err, sizeof(float), s) != cudaSuccess)
    return ucb_host::set_error(UCB_ERR_CUDA, "selftest allocation failed");
  selftest_mma_kernel<<<1, 32, 0, s>>>(d_err);
  int rc = ucb_host::check_launch("selftest_mma_kernel");
  float h = -1.f;
  if (rc == UCB_OK) {
    if (cudaMemcpyAsync(&h, d_err, sizeof(float), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      rc = ucb_host::set_error(UCB_ERR_CUDA, "selftest readback failed");
  }
  cudaFreeAsync(d_err, s);
  if (max_abs_err) *max_abs_err = h;
  return rc;
}

// ---------------------------------------------------------------- host transfers
namespace {
constexpr int MAX_RANGES = 8;
struct CopyRanges {
  unsigned char* dst[MAX_RANGES];
  const unsigned char* src[MAX_RANGES];
  int64_t bytes[MAX_RANGES];
  int n;
};

// Grid-stride copy in 16-byte chunks of every range, then the tail bytes.
// Either side may be device memory or pinned host memory mapped into the
// device address space.
__global__ void copy_ranges_kernel(const CopyRanges R) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int r = 0; r < R.n; ++r) {
    const int64_t n16 = R.bytes[r] / 16;
    for (int64_t i = first; i < n16; i += stride)
      reinterpret_cast<uint4*>(R.dst[r])[i] = reinterpret_cast<const uint4*>(R.src[r])[i];
    const int64_t tail = R.bytes[r] - n16 * 16;
    if (first < tail) R.dst[r][n16 * 16 + first] = R.src[r][n16 * 16 + first];
  }
}
}  // namespace

extern "C" int ucb_host_device_pointer(const void* host, void** dev) {
  if (!host || !dev) return ucb_host::set_error(UCB_ERR_INVALID, "ucb_host_device_pointer: null pointer");
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0);
  if (e != cudaSuccess || d == nullptr) {
    cudaGetLastError();  // clear the (non-sticky) error the failed query left behind
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_host_device_pointer: memory is not mapped pinned host memory (%s)",
                               cudaGetErrorString(e));
  }
  *dev = d;
  return UCB_OK;
}

extern "C" int ucb_copy_ranges(int n, void* const* dst, const void* const* src, const int64_t* bytes, void* stream) {
  if (n < 1 || n > MAX_RANGES || !dst || !src || !bytes)
    return ucb_host::set_error(UCB_ERR_INVALID, "ucb_copy_ranges: need 1..%d ranges", MAX_RANGES);
  CopyRanges R;
  R.n = n;
  int64_t most = 0;
  for (int r = 0; r < n; ++r) {
    if (!dst[r] || !src[r] || bytes[r] < 0) return ucb_host::set_error(UCB_ERR_INVALID, "ucb_copy_ranges: bad range %d", r);
    if ((reinterpret_cast<uintptr_t>(dst[r]) | reinterpret_cast<uintptr_t>(src[r])) & 15)
      return ucb_host::set_error(UCB_ERR_INVALID, "ucb_copy_ranges: range %d is not 16-byte aligned", r);
    R.dst[r] = static_cast<unsigned char*>(dst[r]);
    R.src[r] = static_cast<const unsigned char*>(src[r]);
    R.bytes[r] = bytes[r];
    most = bytes[r] > most ? bytes[r] : most;
  }
  const int64_t chunks = (most + 15) / 16;
  const int blocks = (int)((chunks + 255) / 256 < 148 ? (chunks + 255) / 256 : 148);
  copy_ranges_kernel<<<blocks > 0 ? blocks : 1, 256, 0, static_cast<cudaStream_t>(stream)>>>(R);
  return ucb_host::check_launch("copy_ranges_kernel");
}
