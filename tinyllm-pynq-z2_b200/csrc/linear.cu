// q6w_linear: y[n, rows] = x[n, cols] @ dequant(W)^T, the Q6W nn.Linear.
#include <string.h>

#include <mutex>

#include "launch.cuh"

namespace q6w {

// General fallback for shapes the tiled kernels do not take (odd rows,
// cols % 16 != 0, unaligned pointers): one warp per output element, byte
// loads of 3-byte groups.  Same per-element dequantisation as the fast path.
__global__ void linear_general_kernel(const uint8_t* __restrict__ packed,
                                      const float* __restrict__ scales, const float* __restrict__ x,
                                      float* __restrict__ y, int64_t rows, int64_t cols, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t groups = cols >> 2;
  for (int64_t o = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); o < n * rows;
       o += warps) {
    const int64_t m = o / rows, r = o % rows;
    const uint8_t* row = packed + r * groups * 3;
    const float s = __ldg(scales + r);
    const float* xr = x + m * cols;
    float acc = 0.0f;
    for (int64_t g = lane; g < groups; g += 32) {
      const uint32_t v = load_group(row + 3 * g);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc = fmaf(__fmul_rn((float)group_code(v, i), s), xr[4 * g + i], acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) y[o] = acc;
  }
}

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ out, int n, int len, float eps) {
  __shared__ float red[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int b = blockIdx.x; b < n; b += gridDim.x) {
    const float* xr = x + (int64_t)b * len;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < len; k += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xr[k], xr[k]));
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    const float r = rms_scale(t, len, eps);
    for (int k = threadIdx.x; k < len; k += blockDim.x)
      out[(int64_t)b * len + k] = __fmul_rn(__fmul_rn(xr[k], r), __ldg(w + k));
    __syncthreads();
  }
}

__global__ void keys_to_index_kernel(int n, unsigned long long* keys, int32_t* argmax) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n; b += gridDim.x * blockDim.x) {
    argmax[b] = argmax_index(keys[b]);
    keys[b] = 0ull;
  }
}

}  // namespace q6w

using namespace q6w;

extern "C" int32_t q6w_rmsnorm(const float* x, const float* weight, float* out, int32_t n,
                               int32_t length, float eps, q6w_stream_t stream) {
  clear_error();
  if (n < 0 || length <= 0 || !(eps >= 0.0f)) return fail(Q6W_ERR_ARG, "q6w_rmsnorm: bad shape or epsilon");
  if (n == 0) return Q6W_OK;
  if (!x || !weight || !out) return fail(Q6W_ERR_ARG, "q6w_rmsnorm: null pointer");
  if (!aligned(x, 4) || !aligned(weight, 4) || !aligned(out, 4)) return fail(Q6W_ERR_ALIGN, "q6w_rmsnorm: 4-byte alignment required");
  rmsnorm_kernel<<<n < 4096 ? n : 4096, 256, 0, (cudaStream_t)stream>>>(x, weight, out, n, length, eps);
  Q6W_LAUNCH_CHECK("rmsnorm_kernel");
  return Q6W_OK;
}

extern "C" int32_t q6w_linear_argmax(const uint8_t* packed, const float* scales, const float* x,
                                     float* logits, int32_t* argmax, void* scratch,
                                     size_t scratch_bytes, int64_t rows, int64_t cols, int64_t n,
                                     q6w_stream_t stream) {
  clear_error();
  if (rows <= 0 || cols <= 0 || n < 0) return fail(Q6W_ERR_ARG, "q6w_linear_argmax: bad shape");
  if (cols % 16 || rows % 2) return fail(Q6W_ERR_ARG, "q6w_linear_argmax: cols %% 16 == 0 and even rows required");
  if (rows > INT32_MAX / 2 || cols > INT32_MAX / 2 || n > INT32_MAX) return fail(Q6W_ERR_ARG, "q6w_linear_argmax: shape too large");
  if (n == 0) return Q6W_OK;
  if (!packed || !scales || !x || !argmax || !scratch) return fail(Q6W_ERR_ARG, "q6w_linear_argmax: null pointer");
  if (!aligned(packed, 4) || !aligned(scales, 4) || !aligned(x, 16) || !aligned(scratch, 8) ||
      (logits && !aligned(logits, 8)) || !aligned(argmax, 4))
    return fail(Q6W_ERR_ALIGN, "q6w_linear_argmax: misaligned pointer");
  if (scratch_bytes < (size_t)n * 8) return fail(Q6W_ERR_ARG, "q6w_linear_argmax: scratch needs 8*n bytes");
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long* keys = (unsigned long long*)scratch;
  Q6W_CUDA_TRY(cudaMemsetAsync(keys, 0, (size_t)n * 8, st));
  MatSet ms = {packed, nullptr, nullptr, scales, nullptr, nullptr,
               (int32_t)rows, (int32_t)rows, (int32_t)cols, 0, (int32_t)(rows / 2)};
  EpiArgs ep;
  memset(&ep, 0, sizeof(ep));
  ep.y = logits;
  ep.ldy = (int32_t)rows;
  ep.keys = keys;
  cudaError_t e = LinearLauncher<false, EPI_VOCAB>::run(x, (int)cols, (int)n, nullptr, 0.f, ms, ep, st);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "q6w_linear_argmax launch: %s", cudaGetErrorString(e));
  keys_to_index_kernel<<<grid_for(n, 256), 256, 0, st>>>((int)n, keys, argmax);
  Q6W_LAUNCH_CHECK("keys_to_index_kernel");
  return Q6W_OK;
}

extern "C" int32_t q6w_linear(const uint8_t* packed, const float* scales, const float* x, float* y,
                              int64_t rows, int64_t cols, int64_t n, q6w_stream_t stream) {
  clear_error();
  if (rows < 0 || cols < 0 || n < 0) return fail(Q6W_ERR_ARG, "q6w_linear: negative shape");
  if (cols % 4) return fail(Q6W_ERR_ARG, "Q6 row width must be divisible by four");
  if (rows == 0 || n == 0) return Q6W_OK;
  if (!packed || !scales || !x || !y) return fail(Q6W_ERR_ARG, "q6w_linear: null pointer");
  if (!aligned(scales, 4) || !aligned(x, 4) || !aligned(y, 4))
    return fail(Q6W_ERR_ALIGN, "q6w_linear: scales, x and y must be 4-byte aligned");
  if (rows > INT32_MAX / 2 || n > INT32_MAX || cols > INT32_MAX / 2)
    return fail(Q6W_ERR_ARG, "q6w_linear: shape too large");
  cudaStream_t st = (cudaStream_t)stream;
  const bool fast = cols > 0 && cols % 16 == 0 && rows % 2 == 0 && aligned(packed, 4) &&
                    aligned(x, 16) && aligned(y, 8);
  if (!fast) {
    linear_general_kernel<<<grid_for(n * rows * 32, 256), 256, 0, st>>>(packed, scales, x, y, rows,
                                                                          cols, n);
    Q6W_LAUNCH_CHECK("linear_general_kernel");
    return Q6W_OK;
  }
  MatSet ms = {packed, nullptr, nullptr, scales, nullptr, nullptr,
               (int32_t)rows, (int32_t)rows, (int32_t)cols, 0, (int32_t)(rows / 2)};
  EpiArgs ep;
  memset(&ep, 0, sizeof(ep));
  ep.y = y;
  ep.ldy = (int32_t)rows;
  cudaError_t e = LinearLauncher<false, EPI_STORE>::run(x, (int)cols, (int)n, nullptr, 0.f, ms, ep, st);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "q6w_linear launch: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

// ---- q6w_linear_argmax_noalloc ----------------------------------------------
//
// Same computation as q6w_linear_argmax, with its scratch (one 64-bit argmax
// key per activation row) in a library-owned device array instead of caller
// memory, for callers that cannot allocate device memory: hosts that bind
// this library through a plain FFI (ctypes, JNI, cgo) and own no CUDA
// allocator, and serving loops that run under a fixed device-memory budget
// where a per-call cudaMalloc can fail and a cudaFree synchronises the
// device.  Every GPU that loads the library holds the array (256 KiB) until
// the process exits.
namespace q6w {

constexpr int64_t kNoAllocMaxRows = 32768;  // activation rows per call
static __device__ __align__(256) unsigned long long g_noalloc_keys[kNoAllocMaxRows];

// Device address of g_noalloc_keys (the host-side name is only a stand-in
// for the symbol, not a device pointer).  The address belongs to the CUDA
// context that loaded this module, so it is looked up with cudaGetSymbolAddress
// once per context -- the first call on each device, and again after the
// context changes (a cudaDeviceReset, or a driver-API context the caller made
// current) -- and cached under the context's unique id.
static unsigned long long* noalloc_keys_ptr(int32_t* status) {
  struct Entry {
    unsigned long long ctx;
    unsigned long long* ptr;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  unsigned long long ctx = context_id();
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].ctx == ctx) {
        *status = Q6W_OK;
        return cache[i].ptr;
      }
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_keys);
  if (e != cudaSuccess || !p) {
    *status = fail(Q6W_ERR_CUDA, "q6w_linear_argmax_noalloc: cudaGetSymbolAddress failed: %s",
                   cudaGetErrorString(e));
    return nullptr;
  }
  if (!ctx) ctx = context_id();  // the lookup made the primary context current
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    cache[used < 64 ? used++ : (int)(ctx % 64)] = {ctx, (unsigned long long*)p};
  }
  *status = Q6W_OK;
  return (unsigned long long*)p;
}

}  // namespace q6w

extern "C" int32_t q6w_linear_argmax_noalloc(const uint8_t* packed, const float* scales,
                                             const float* x, float* logits, int32_t* argmax,
                                             int64_t rows, int64_t cols, int64_t n,
                                             q6w_stream_t stream) {
  clear_error();
  if (n > kNoAllocMaxRows)
    return fail(Q6W_ERR_ARG,
                "q6w_linear_argmax_noalloc: n = %lld activation rows exceeds the built-in maximum of %lld",
                (long long)n, (long long)kNoAllocMaxRows);
  if (rows <= 0 || cols <= 0 || n < 0) return fail(Q6W_ERR_ARG, "q6w_linear_argmax_noalloc: bad shape");
  if (cols % 16 || rows % 2)
    return fail(Q6W_ERR_ARG, "q6w_linear_argmax_noalloc: cols %% 16 == 0 and even rows required");
  if (rows > INT32_MAX / 2 || cols > INT32_MAX / 2) return fail(Q6W_ERR_ARG, "q6w_linear_argmax_noalloc: shape too large");
  if (n == 0) return Q6W_OK;
  if (!packed || !scales || !x || !argmax) return fail(Q6W_ERR_ARG, "q6w_linear_argmax_noalloc: null pointer");
  if (!aligned(packed, 4) || !aligned(scales, 4) || !aligned(x, 16) || (logits && !aligned(logits, 8)) ||
      !aligned(argmax, 4))
    return fail(Q6W_ERR_ALIGN, "q6w_linear_argmax_noalloc: misaligned pointer");
  int32_t st = Q6W_OK;
  unsigned long long* keys = noalloc_keys_ptr(&st);
  if (!keys) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // The array keeps the previous call's contents: the keys must start at 0.
  Q6W_CUDA_TRY(cudaMemsetAsync(keys, 0, (size_t)n * sizeof(unsigned long long), s));
  MatSet ms = {packed, nullptr, nullptr, scales, nullptr, nullptr,
               (int32_t)rows, (int32_t)rows, (int32_t)cols, 0, (int32_t)(rows / 2)};
  EpiArgs ep;
  memset(&ep, 0, sizeof(ep));
  ep.y = logits;
  ep.ldy = (int32_t)rows;
  ep.keys = keys;
  cudaError_t e = LinearLauncher<false, EPI_VOCAB>::run(x, (int)cols, (int)n, nullptr, 0.f, ms, ep, s);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "q6w_linear_argmax_noalloc launch: %s", cudaGetErrorString(e));
  keys_to_index_kernel<<<grid_for(n, 256), 256, 0, s>>>((int)n, keys, argmax);
  Q6W_LAUNCH_CHECK("keys_to_index_kernel");
  return Q6W_OK;
}
