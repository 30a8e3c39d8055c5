// Q6W codec entry points: q6w_unpack, q6w_dequant, and the library's error state.
//
// Both kernels are pure HBM streams (3/4 byte in, 1 or 4 bytes out per
// value).  A thread owns one 3-byte group (4 values) so any cols % 4 == 0
// layout is handled without alignment assumptions; the grid is sized in
// multiples of the SM count and grid-strides over the groups.
#include <stdarg.h>
#include <stdio.h>

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

namespace stream {
// Bit 4 is set by a streaming-kernel wait that ran out of time (a
// should-never-happen diagnostic; the kernel then skips the rest of its work).
__device__ int32_t g_error_word;

int32_t* error_word() {
  static int32_t* cache[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) cudaGetLastError();
    cache[dev] = static_cast<int32_t*>(p);
  }
  return cache[dev];
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

}  // namespace q6w

using namespace q6w;

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
