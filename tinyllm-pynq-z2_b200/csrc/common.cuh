// Shared device helpers and host error plumbing for the Q6W sm_100a library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q6w_b200.h"

namespace q6w {

// ---- host-side status ------------------------------------------------------

// Record a formatted message for this host thread and return `code`.
int32_t fail(int32_t code, const char* fmt, ...);
void clear_error();

#define Q6W_CUDA_TRY(expr)                                                              \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return ::q6w::fail(Q6W_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

#define Q6W_LAUNCH_CHECK(what)                                                          \
  do {                                                                                  \
    cudaError_t e_ = cudaGetLastError();                                                \
    if (e_ != cudaSuccess)                                                              \
      return ::q6w::fail(Q6W_ERR_CUDA, "launch of %s failed: %s", what,                 \
                         cudaGetErrorString(e_));                                       \
  } while (0)

int sm_count();
// Id of the CUDA context current on this host thread (0 if none / unknown).
unsigned long long context_id();
// Device address of a __device__ symbol in the current context, looked up
// once per (context, symbol) and cached.
cudaError_t symbol_address(const void* symbol, void** out);
namespace stream {
int32_t* error_word();
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ---- Q6W decode --------------------------------------------------------------
//
// A packed row is a little-endian stream of 6-bit two's-complement fields:
// value i sits at bits [6i, 6i+6).  Sixteen values fill exactly three 32-bit
// words, the unit every kernel here loads.
//
// Field -> float without an integer conversion: (u ^ 0x20) maps the signed
// code v in [-32, 31] to v + 32 in [0, 63]; OR-ing it under the exponent of
// 1.5 * 2^23 (0x4B400000, ulp 1) gives the float 12582944 + v exactly, and
// one subtraction leaves v.  `(u & 0x3F) ^ 0x4B400020` does the mask, the
// bias and the exponent in one logic op.
__device__ __forceinline__ float code_to_float(uint32_t field) {
  return __int_as_float((field & 0x3Fu) ^ 0x4B400020u) - 12582944.0f;
}

// Decode the 16 codes held in words (w0, w1, w2) and multiply each by the
// row scale with one rounded FP32 product -- the reference's
// float32(q) * scale (quantization/q6w_format.py:258), bit for bit.
__device__ __forceinline__ void dequant16(uint32_t w0, uint32_t w1, uint32_t w2, float s,
                                          float (&w)[16]) {
  w[0] = __fmul_rn(code_to_float(w0), s);
  w[1] = __fmul_rn(code_to_float(w0 >> 6), s);
  w[2] = __fmul_rn(code_to_float(w0 >> 12), s);
  w[3] = __fmul_rn(code_to_float(w0 >> 18), s);
  w[4] = __fmul_rn(code_to_float(w0 >> 24), s);
  w[5] = __fmul_rn(code_to_float(__funnelshift_r(w0, w1, 30)), s);
  w[6] = __fmul_rn(code_to_float(w1 >> 4), s);
  w[7] = __fmul_rn(code_to_float(w1 >> 10), s);
  w[8] = __fmul_rn(code_to_float(w1 >> 16), s);
  w[9] = __fmul_rn(code_to_float(w1 >> 22), s);
  w[10] = __fmul_rn(code_to_float(__funnelshift_r(w1, w2, 28)), s);
  w[11] = __fmul_rn(code_to_float(w2 >> 2), s);
  w[12] = __fmul_rn(code_to_float(w2 >> 8), s);
  w[13] = __fmul_rn(code_to_float(w2 >> 14), s);
  w[14] = __fmul_rn(code_to_float(w2 >> 20), s);
  w[15] = __fmul_rn(code_to_float(w2 >> 26), s);
}

// Signed code of field i (0..3) of a 3-byte group.
__device__ __forceinline__ int32_t group_code(uint32_t g24, int i) {
  int32_t f = (int32_t)((g24 >> (6 * i)) & 0x3Fu);
  return f >= 32 ? f - 64 : f;
}

__device__ __forceinline__ uint32_t load_group(const uint8_t* p) {
  return (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 8) | ((uint32_t)__ldg(p + 2) << 16);
}

// Order-preserving 32-bit image of a float (larger float -> larger key).
// Every NaN maps to the canonical +NaN first, so it ranks above +inf as
// torch.argmax ranks NaN (a NaN with the sign bit set would otherwise sort
// below -inf).  Every float then has a key > 0: a key of 0 means "no value
// seen", which argmax_index turns into -1.
__device__ __forceinline__ uint32_t float_key(float v) {
  uint32_t u = v != v ? 0x7FC00000u : __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Argmax key: max over keys picks the largest value, and among equal values
// the smallest index -- the first-maximum rule of torch.argmax.
__device__ __forceinline__ unsigned long long argmax_key(float v, int32_t idx) {
  return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int32_t argmax_index(unsigned long long key) {
  return (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

}  // namespace q6w
