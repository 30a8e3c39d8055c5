// Q6W codec entry points: q6w_unpack, q6w_dequant, and the library's error state.
//
// Both kernels are pure HBM streams (3/4 byte in, 1 or 4 bytes out per
// value).  A thread owns one 3-byte group (4 values) so any cols % 4 == 0
// layout is handled without alignment assumptions; the grid is sized in
// multiples of the SM count and grid-strides over the groups.
#include <stdarg.h>
#include <stdio.h>

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace q6w {

static thread_local char g_msg[512] = "";

int32_t fail(int32_t code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_msg[0] = 0; }

// Multiprocessor count of the current device (cached per device).
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = 148;
    }
    cache[dev] = v;
  }
  return cache[dev];
}

// Unique id of the CUDA context current on this host thread (0 when none is
// current or the driver entry points are unavailable).  A __device__
// symbol's address belongs to the context that loaded the module: a new
// primary context after cudaDeviceReset, or a driver-API context the caller
// made current, has its own.  Caches of symbol addresses are keyed by it.
unsigned long long context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_cur = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    cudaGetLastError();
  });
  if (!get_cur || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

cudaError_t symbol_address(const void* symbol, void** out) {
  struct Entry {
    unsigned long long ctx;
    const void* sym;
    void* addr;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  *out = nullptr;
  unsigned long long ctx = context_id();
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].ctx == ctx && cache[i].sym == symbol) {
        *out = cache[i].addr;
        return cudaSuccess;
      }
  }
  // (with no context current yet, the lookup itself makes the device's
  // primary context current; its id is read afterwards)
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, symbol);
  if (e != cudaSuccess || !p) return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
  *out = p;
  if (!ctx) ctx = context_id();
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    cache[used < 64 ? used++ : (int)(ctx % 64)] = {ctx, symbol, p};
  }
  return cudaSuccess;
}

namespace stream {
// Bit 4 is set by a streaming-kernel wait that ran out of time (a
// should-never-happen diagnostic; the kernel then skips the rest of its work).
__device__ int32_t g_error_word;

// Device address of g_error_word in the current context, or null (with the
// CUDA error left for the caller) when the lookup fails.
int32_t* error_word() {
  void* p = nullptr;
  if (symbol_address(&g_error_word, &p) != cudaSuccess) return nullptr;
  return static_cast<int32_t*>(p);
}
}  // namespace stream

int grid_for(int64_t work, int threads) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  int64_t blocks = (work + threads - 1) / threads;
  int64_t cap = (int64_t)sms * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int8_t* __restrict__ out,
                              int64_t groups) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    uint32_t w = load_group(packed + 3 * g);
    char4 v = make_char4((signed char)group_code(w, 0), (signed char)group_code(w, 1),
                         (signed char)group_code(w, 2), (signed char)group_code(w, 3));
    reinterpret_cast<char4*>(out)[g] = v;
  }
}

// Unaligned-output variant (int8 output not 4-byte aligned).
__global__ void unpack_bytes_kernel(const uint8_t* __restrict__ packed, int8_t* __restrict__ out,
                                    int64_t groups) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    uint32_t w = load_group(packed + 3 * g);
    for (int i = 0; i < 4; ++i) out[4 * g + i] = (int8_t)group_code(w, i);
  }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scales,
                               float* __restrict__ out, int64_t groups, int64_t groups_per_row,
                               bool vec_out) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    uint32_t w = load_group(packed + 3 * g);
    float s = __ldg(scales + g / groups_per_row);
    float v0 = __fmul_rn((float)group_code(w, 0), s), v1 = __fmul_rn((float)group_code(w, 1), s);
    float v2 = __fmul_rn((float)group_code(w, 2), s), v3 = __fmul_rn((float)group_code(w, 3), s);
    if (vec_out) {
      reinterpret_cast<float4*>(out)[g] = make_float4(v0, v1, v2, v3);
    } else {
      out[4 * g] = v0;
      out[4 * g + 1] = v1;
      out[4 * g + 2] = v2;
      out[4 * g + 3] = v3;
    }
  }
}

// ---- row-wise quantization (the Q6W writer) ----------------------------------
//
// quantize_rows of quantization/q6w_format.py:84-98 with the same FP32
// operations, so codes and scales are bit-identical:
//   scale = max|w| / 31 (one rounded division; 1.0 for an all-zero row)
//   q     = clamp(round-half-even(w / scale), -31, 31)
// and packs the codes low-bit-first (pack_signed_int6, :52-64).  One CTA per
// row (grid-stride): a max reduction, then each thread turns 4-value groups
// into 3 bytes.  With row_err set, the reconstruction error of every row
// (max |q*s - w|, sum |q*s - w|, sum (q*s - w)^2, the last two in FP64) is
// written for the statistics kernel.
constexpr int kQuantThreads = 256;

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  __syncthreads();
  return t;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kQuantThreads) quantize_rows_kernel(const float* __restrict__ w, int64_t rows,
                                                                      int64_t cols, uint8_t* __restrict__ packed,
                                                                      float* __restrict__ scales,
                                                                      double* __restrict__ row_err) {
  __shared__ float redf[32];
  __shared__ double redd[32];
  const int64_t groups = cols >> 2;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* wr = w + r * cols;
    float mx = 0.0f;
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) mx = fmaxf(mx, fabsf(wr[k]));
    mx = block_max(mx, redf);
    const float s = mx > 0.0f ? __fdiv_rn(mx, 31.0f) : 1.0f;
    float emax = 0.0f;
    double esum = 0.0, esq = 0.0;
    uint8_t* pr = packed + r * groups * 3;
    for (int64_t g = threadIdx.x; g < groups; g += blockDim.x) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = wr[4 * g + i];
        const float qf = fminf(fmaxf(rintf(__fdiv_rn(v, s)), -31.0f), 31.0f);
        word |= ((uint32_t)(int32_t)qf & 0x3Fu) << (6 * i);
        const float e = __fsub_rn(__fmul_rn(qf, s), v);
        emax = fmaxf(emax, fabsf(e));
        esum += (double)fabsf(e);
        esq += (double)e * (double)e;
      }
      pr[3 * g] = (uint8_t)word;
      pr[3 * g + 1] = (uint8_t)(word >> 8);
      pr[3 * g + 2] = (uint8_t)(word >> 16);
    }
    if (row_err) {
      emax = block_max(emax, redf);
      esum = block_sum(esum, redd);
      esq = block_sum(esq, redd);
      if (threadIdx.x == 0) {
        row_err[3 * r] = (double)emax;
        row_err[3 * r + 1] = esum;
        row_err[3 * r + 2] = esq;
      }
    }
    if (threadIdx.x == 0) scales[r] = s;
  }
}

// Whole-matrix statistics from the per-row errors, in one fixed order
// (deterministic): stats = {max_abs_error, mean_abs_error, rmse}.
__global__ void __launch_bounds__(kQuantThreads) quantize_stats_kernel(const double* __restrict__ row_err,
                                                                       int64_t rows, int64_t values,
                                                                       double* __restrict__ stats) {
  __shared__ float redf[32];
  __shared__ double redd[32];
  float emax = 0.0f;
  double esum = 0.0, esq = 0.0;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    emax = fmaxf(emax, (float)row_err[3 * r]);
    esum += row_err[3 * r + 1];
    esq += row_err[3 * r + 2];
  }
  emax = block_max(emax, redf);
  esum = block_sum(esum, redd);
  esq = block_sum(esq, redd);
  if (threadIdx.x == 0) {
    stats[0] = (double)emax;
    stats[1] = esum / (double)values;
    stats[2] = sqrt(esq / (double)values);
  }
}

}  // namespace q6w

using namespace q6w;

extern "C" int32_t q6w_quantize_rows(const float* weights, int64_t rows, int64_t cols, uint8_t* packed,
                                     float* scales, double* row_err, double* stats, q6w_stream_t stream) {
  clear_error();
  if (rows < 0 || cols < 0) return fail(Q6W_ERR_ARG, "q6w_quantize_rows: negative shape");
  if (cols % 4) return fail(Q6W_ERR_ARG, "Q6 rows must be 2D and have a width divisible by four");
  if (stats && !row_err) return fail(Q6W_ERR_ARG, "q6w_quantize_rows: stats need the row_err scratch");
  if (rows == 0 || cols == 0) return Q6W_OK;
  if (!weights || !packed || !scales) return fail(Q6W_ERR_ARG, "q6w_quantize_rows: null pointer");
  if (!aligned(weights, 4) || !aligned(scales, 4) || (row_err && !aligned(row_err, 8)) ||
      (stats && !aligned(stats, 8)))
    return fail(Q6W_ERR_ALIGN, "q6w_quantize_rows: weights/scales 4-byte and row_err/stats 8-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t cap = (int64_t)sm_count() * 16;
  const int grid = (int)(rows < cap ? rows : cap);
  quantize_rows_kernel<<<grid, kQuantThreads, 0, st>>>(weights, rows, cols, packed, scales, row_err);
  Q6W_LAUNCH_CHECK("quantize_rows_kernel");
  if (stats) {
    quantize_stats_kernel<<<1, kQuantThreads, 0, st>>>(row_err, rows, rows * cols, stats);
    Q6W_LAUNCH_CHECK("quantize_stats_kernel");
  }
  return Q6W_OK;
}

extern "C" const char* q6w_last_error(void) { return g_msg; }
extern "C" int32_t q6w_abi_version(void) { return 1; }

extern "C" int32_t q6w_unpack(const uint8_t* packed, int8_t* out, int64_t rows, int64_t cols,
                              q6w_stream_t stream) {
  clear_error();
  if (rows < 0 || cols < 0) return fail(Q6W_ERR_ARG, "q6w_unpack: negative shape");
  if (cols % 4) return fail(Q6W_ERR_ARG, "Q6 row width must be divisible by four");
  int64_t groups = rows * (cols / 4);
  if (groups == 0) return Q6W_OK;
  if (!packed || !out) return fail(Q6W_ERR_ARG, "q6w_unpack: null pointer");
  int g = grid_for(groups, 256);
  if (aligned(out, 4))
    unpack_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(packed, out, groups);
  else
    unpack_bytes_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(packed, out, groups);
  Q6W_LAUNCH_CHECK("unpack_kernel");
  return Q6W_OK;
}

extern "C" int32_t q6w_dequant(const uint8_t* packed, const float* scales, float* out, int64_t rows,
                               int64_t cols, q6w_stream_t stream) {
  clear_error();
  if (rows < 0 || cols < 0) return fail(Q6W_ERR_ARG, "q6w_dequant: negative shape");
  if (cols % 4) return fail(Q6W_ERR_ARG, "Q6 row width must be divisible by four");
  int64_t groups = rows * (cols / 4);
  if (groups == 0) return Q6W_OK;
  if (!packed || !scales || !out) return fail(Q6W_ERR_ARG, "q6w_dequant: null pointer");
  if (!aligned(scales, 4) || !aligned(out, 4)) return fail(Q6W_ERR_ALIGN, "q6w_dequant: scales/out must be 4-byte aligned");
  dequant_kernel<<<grid_for(groups, 256), 256, 0, (cudaStream_t)stream>>>(
      packed, scales, out, groups, cols / 4, aligned(out, 16));
  Q6W_LAUNCH_CHECK("dequant_kernel");
  return Q6W_OK;
}
