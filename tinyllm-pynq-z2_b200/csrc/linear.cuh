// Q6W linear kernels (FP32 SIMT) with fused prologues and epilogues.
//
// Output rows are produced in PAIRS.  A pair is either two adjacent rows of
// one matrix (the RoPE pair (2j, 2j+1) of torch_benchmark.py:79-85 falls in
// one pair) or, in GLU mode, row j of W1 and row j of W3 (the SwiGLU gate and
// up projections of torch_benchmark.py:123, computed together).  A "matrix
// set" concatenates up to three matrices that share the input (wq | wk | wv).
//
// Two kernels:
//   gemv_kernel  n <= 8 activation rows (decode of few sequences).  The
//                normalised activations sit in shared memory; lane groups of
//                G lanes split a row pair's 16-value units (12 bytes = three
//                32-bit loads), dequantise in registers and reduce with
//                shuffles.  Weight bytes are read once per launch.
//   gemm_kernel  n > 8.  128 x 64 (seqs x rows) CTA tiles, K in steps of 32:
//                the weight tile is decoded + dequantised once into shared
//                memory and reused by all 128 activation rows.
//
// Weights are dequantised exactly as the reference does
// (float32(q) * scale, quantization/q6w_format.py:258) and accumulated in
// FP32 FMA, so results differ from the reference only by summation order.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace q6w {

enum { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_GLU = 3, EPI_VOCAB = 4 };
enum { SEQ_DONE = 1, SEQ_INVALID = 2 };
constexpr int kMaxStop = 8;

struct MatSet {
  const uint8_t* q0;
  const uint8_t* q1;
  const uint8_t* q2;
  const float* s0;
  const float* s1;
  const float* s2;
  int32_t end0, end1;  // cumulative row ends of matrices 0 and 1 (concat mode)
  int32_t cols;
  int32_t glu;         // 1: pair p = (matrix 0 row p, matrix 1 row p)
  int32_t n_pairs;
};

struct EpiArgs {
  float* y;  // STORE / RESID / GLU output, VOCAB logits (may be null)
  int32_t ldy;
  // QKV
  float* qbuf;
  int32_t ldq;
  float* kc;
  float* vc;
  int64_t cache_stride;
  int64_t layer_off;
  const int32_t* seq;  // cache row of activation row m (null: row m); prefill rows are tokens
  const float* rope_cos;
  const float* rope_sin;
  int32_t hd, q_rows, kv_rows;
  int32_t kv_half;     // the cache holds FP16 (kc / vc point at __half; offsets stay in elements)
  // per-sequence state
  const int32_t* pos;
  const int32_t* flags;
  // VOCAB
  unsigned long long* keys;
  const int32_t* gen;
  const int32_t* plen;
  float* step_logits;
  int32_t new_tokens, vocab, min_new, n_stop;
  int32_t stop_ids[kMaxStop];
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- KV cache elements: FP32, or FP16 (round to nearest even, as torch's
// copy_ of an FP32 row into a float16 cache; quantization/compare_kv_cache.py:57-58)

// Two consecutive elements (offset even) of a cache row.
__device__ __forceinline__ void store_kv2(float* base, int64_t off, int half, float a, float b) {
  if (half)
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + off) = __floats2half2_rn(a, b);
  else
    *reinterpret_cast<float2*>(base + off) = make_float2(a, b);
}

// Eight consecutive elements (offset a multiple of 8) of a cache row.
__device__ __forceinline__ void store_kv8(float* base, int64_t off, int half, float4 p0, float4 p1) {
  if (half) {
    const __half2 h0 = __floats2half2_rn(p0.x, p0.y), h1 = __floats2half2_rn(p0.z, p0.w);
    const __half2 h2 = __floats2half2_rn(p1.x, p1.y), h3 = __floats2half2_rn(p1.z, p1.w);
    uint4 u;
    u.x = *reinterpret_cast<const uint32_t*>(&h0);
    u.y = *reinterpret_cast<const uint32_t*>(&h1);
    u.z = *reinterpret_cast<const uint32_t*>(&h2);
    u.w = *reinterpret_cast<const uint32_t*>(&h3);
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(base) + off) = u;
  } else {
    reinterpret_cast<float4*>(base + off)[0] = p0;
    reinterpret_cast<float4*>(base + off)[1] = p1;
  }
}

// Four consecutive cache elements as FP32 (FP16 converts exactly).
template <typename KT>
__device__ __forceinline__ float4 load_kv4(const KT* p);
template <>
__device__ __forceinline__ float4 load_kv4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 load_kv4<__half>(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Sixteen consecutive cache elements as four float4.
template <typename KT>
__device__ __forceinline__ void load_kv16(const KT* p, float4 (&o)[4]);
template <>
__device__ __forceinline__ void load_kv16<float>(const float* p, float4 (&o)[4]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = q[i];
}
template <>
__device__ __forceinline__ void load_kv16<__half>(const __half* p, float4 (&o)[4]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 u = q[i];
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
    o[2 * i] = make_float4(a.x, a.y, b.x, b.y);
    o[2 * i + 1] = make_float4(c.x, c.y, d.x, d.y);
  }
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

__device__ __forceinline__ void pair_rows(const MatSet& ms, int p, const uint8_t*& ra, float& sa,
                                          const uint8_t*& rb, float& sb) {
  const int64_t rbytes = (int64_t)ms.cols * 3 / 4;
  if (ms.glu) {
    ra = ms.q0 + p * rbytes;
    rb = ms.q1 + p * rbytes;
    sa = __ldg(ms.s0 + p);
    sb = __ldg(ms.s1 + p);
  } else {
    const int v = 2 * p;
    const uint8_t* q;
    const float* s;
    int r;
    if (v < ms.end0) {
      q = ms.q0; s = ms.s0; r = v;
    } else if (v < ms.end1) {
      q = ms.q1; s = ms.s1; r = v - ms.end0;
    } else {
      q = ms.q2; s = ms.s2; r = v - ms.end1;
    }
    ra = q + r * rbytes;
    rb = ra + rbytes;
    sa = __ldg(s + r);
    sb = __ldg(s + r + 1);
  }
}

// silu(a) * b with the rounding steps of torch's CPU silu (x / (1 + exp(-x))).
__device__ __forceinline__ float swiglu(float a, float b) {
  float sig = __fdiv_rn(a, __fadd_rn(1.0f, expf(-a)));
  return __fmul_rn(sig, b);
}

// Apply the epilogue to output pair p of activation row m; returns the
// pair's argmax key for EPI_VOCAB (0 otherwise).
template <int EPI>
__device__ __forceinline__ unsigned long long epilogue(const EpiArgs& ep, int m, int p, float a,
                                                       float b) {
  if (EPI == EPI_STORE) {
    float* y = ep.y + (int64_t)m * ep.ldy + 2 * p;
    y[0] = a;
    y[1] = b;
  } else if (EPI == EPI_RESID) {
    float* y = ep.y + (int64_t)m * ep.ldy + 2 * p;
    y[0] = __fadd_rn(y[0], a);
    y[1] = __fadd_rn(y[1], b);
  } else if (EPI == EPI_GLU) {
    ep.y[(int64_t)m * ep.ldy + p] = swiglu(a, b);
  } else if (EPI == EPI_QKV) {
    if (ep.flags[m] & SEQ_INVALID) return 0;
    const int v = 2 * p;
    const int pos = ep.pos[m];
    if (v < ep.q_rows + ep.kv_rows) {
      // RoPE of torch_benchmark.py:84 with each product rounded before the
      // add/subtract, as torch evaluates it.
      const int j = (v % ep.hd) >> 1;
      const float c = __ldg(ep.rope_cos + (int64_t)pos * (ep.hd >> 1) + j);
      const float s = __ldg(ep.rope_sin + (int64_t)pos * (ep.hd >> 1) + j);
      const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
      const float rb = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
      a = ra;
      b = rb;
    }
    const int64_t crow = ep.seq ? ep.seq[m] : m;
    if (v < ep.q_rows) {
      float* dst = ep.qbuf + (int64_t)m * ep.ldq + v;
      dst[0] = a;
      dst[1] = b;
    } else {
      const bool kr = v < ep.q_rows + ep.kv_rows;
      const int64_t off = crow * ep.cache_stride + ep.layer_off + (int64_t)pos * ep.kv_rows +
                          (kr ? v - ep.q_rows : v - ep.q_rows - ep.kv_rows);
      float* base = kr ? ep.kc : ep.vc;
      store_kv2(base, off, ep.kv_half, a, b);
    }
  } else if (EPI == EPI_VOCAB) {
    const int r = 2 * p;
    if (ep.y) {
      float* y = ep.y + (int64_t)m * ep.ldy + r;
      y[0] = a;
      y[1] = b;
    }
    if (ep.step_logits && !(ep.flags[m] & (SEQ_DONE | SEQ_INVALID)) && ep.pos[m] >= ep.plen[m] - 1) {
      float* y = ep.step_logits + ((int64_t)m * ep.new_tokens + ep.gen[m]) * ep.vocab + r;
      y[0] = a;
      y[1] = b;
    }
    if (ep.n_stop && ep.gen[m] < ep.min_new) {
      for (int i = 0; i < ep.n_stop; ++i) {
        if (ep.stop_ids[i] == r) a = -INFINITY;
        if (ep.stop_ids[i] == r + 1) b = -INFINITY;
      }
    }
    return umax64(argmax_key(a, r), argmax_key(b, r + 1));
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Prologue: stage activation row(s) with optional RMSNorm
// (torch_benchmark.py:22-24: x * rsqrt(mean(x^2) + eps), then * weight; the
// reciprocal square root is a correctly rounded sqrt and divide, as torch's
// CPU rsqrt).
__device__ __forceinline__ float rms_scale(float ss, int K, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
}

template <int NB, int G, bool RMS, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(const float* __restrict__ x, int32_t ldx,
                                                   int32_t n, const float* __restrict__ gnorm,
                                                   float eps, MatSet ms, EpiArgs ep) {
  extern __shared__ __align__(16) float4 xs4[];  // [NB][4][U] float4, unit-interleaved
  __shared__ float red[32];
  const int K = ms.cols, U = K >> 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  float* xs = reinterpret_cast<float*>(xs4);

  for (int b = 0; b < NB; ++b) {
    const bool live = b < n;
    const float* xr = x + (int64_t)b * ldx;
    float rstd = 1.0f;
    if (RMS && live) {
      float ss = 0.0f;
      for (int k = tid; k < K; k += blockDim.x) {
        float v = xr[k];
        ss = __fadd_rn(ss, __fmul_rn(v, v));
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float t = lane < nwarps ? red[lane] : 0.0f;
      t = warp_sum(t);
      rstd = rms_scale(t, K, eps);
      __syncthreads();
    }
    for (int k = tid; k < K; k += blockDim.x) {
      float v = live ? xr[k] : 0.0f;
      if (RMS && live) v = __fmul_rn(__fmul_rn(v, rstd), __ldg(gnorm + k));
      const int u = k >> 4, j = (k >> 2) & 3, e = k & 3;
      xs[(((b * 4 + j) * U + u) << 2) + e] = v;
    }
  }
  __syncthreads();

  constexpr int GPW = 32 / G;
  const int gl = lane & (G - 1), grp = lane / G;
  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = 0ull;

  for (int pb = (blockIdx.x * nwarps + warp) * GPW; pb < ms.n_pairs;
       pb += gridDim.x * nwarps * GPW) {
    const int p = pb + grp;
    const bool act = p < ms.n_pairs;
    float acc0[NB], acc1[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc0[b] = acc1[b] = 0.0f;
    if (act) {
      const uint8_t *ra, *rb;
      float sa, sb;
      pair_rows(ms, p, ra, sa, rb, sb);
#pragma unroll 2
      for (int u = gl; u < U; u += G) {
        const uint32_t* pa = reinterpret_cast<const uint32_t*>(ra + 12 * u);
        const uint32_t* pq = reinterpret_cast<const uint32_t*>(rb + 12 * u);
        const uint32_t a0 = __ldg(pa), a1 = __ldg(pa + 1), a2 = __ldg(pa + 2);
        const uint32_t b0 = __ldg(pq), b1 = __ldg(pq + 1), b2 = __ldg(pq + 2);
        float wa[16], wb[16];
        dequant16(a0, a1, a2, sa, wa);
        dequant16(b0, b1, b2, sb, wb);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 xv = xs4[(b * 4 + j) * U + u];
            acc0[b] = fmaf(wa[4 * j + 0], xv.x, acc0[b]);
            acc0[b] = fmaf(wa[4 * j + 1], xv.y, acc0[b]);
            acc0[b] = fmaf(wa[4 * j + 2], xv.z, acc0[b]);
            acc0[b] = fmaf(wa[4 * j + 3], xv.w, acc0[b]);
            acc1[b] = fmaf(wb[4 * j + 0], xv.x, acc1[b]);
            acc1[b] = fmaf(wb[4 * j + 1], xv.y, acc1[b]);
            acc1[b] = fmaf(wb[4 * j + 2], xv.z, acc1[b]);
            acc1[b] = fmaf(wb[4 * j + 3], xv.w, acc1[b]);
          }
        }
      }
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        acc0[b] += __shfl_xor_sync(0xffffffffu, acc0[b], o);
        acc1[b] += __shfl_xor_sync(0xffffffffu, acc1[b], o);
      }
    }
    if (act && gl == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (b < n) best[b] = umax64(best[b], epilogue<EPI>(ep, b, p, acc0[b], acc1[b]));
    }
  }
  if (EPI == EPI_VOCAB) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      unsigned long long k = best[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) k = umax64(k, __shfl_xor_sync(0xffffffffu, k, o));
      if (lane == 0 && b < n && k) atomicMax(ep.keys + b, k);
    }
  }
}

template <bool RMS, int EPI>
__global__ void __launch_bounds__(256) gemm_kernel(const float* __restrict__ x, int32_t ldx,
                                                   int32_t n, const float* __restrict__ gnorm,
                                                   float eps, MatSet ms, EpiArgs ep) {
  constexpr int BM = 128, BP = 32, BN = 64, BK = 32;
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  __shared__ float rs[BM];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.y * BM, p0 = blockIdx.x * BP;
  const int K = ms.cols;

  if (RMS) {
    for (int r = warp; r < BM; r += 8) {
      const int m = m0 + r;
      float ss = 0.0f;
      if (m < n) {
        const float* xr = x + (int64_t)m * ldx;
        for (int k = lane; k < K; k += 32) {
          const float v = xr[k];
          ss = __fadd_rn(ss, __fmul_rn(v, v));
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) rs[r] = rms_scale(ss, K, eps);
    }
    __syncthreads();
  }

  // Weight-load role: threads 0..127 own one (row, 16-column unit) slot.
  const int lr = tid >> 1, lu = tid & 1;
  const uint8_t* wrow = nullptr;
  float wsc = 0.0f;
  if (tid < 128) {
    const int p = p0 + (lr >> 1);
    if (p < ms.n_pairs) {
      const uint8_t *ra, *rb;
      float sa, sb;
      pair_rows(ms, p, ra, sa, rb, sb);
      wrow = (lr & 1) ? rb : ra;
      wsc = (lr & 1) ? sb : sa;
    }
  }

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int k0 = 0; k0 < K; k0 += BK) {
    if (tid < 128) {
      float w[16];
      const int k = k0 + 16 * lu;
      if (wrow && k < K) {
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(wrow + (k >> 4) * 12);
        dequant16(__ldg(pw), __ldg(pw + 1), __ldg(pw + 2), wsc, w);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) Bs[16 * lu + i][lr] = w[i];
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + 256 * it;
      const int r = idx & (BM - 1), kc = idx >> 7;
      const int m = m0 + r, k = k0 + 4 * kc;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < n && k < K) {
        v = *reinterpret_cast<const float4*>(x + (int64_t)m * ldx + k);
        if (RMS) {
          const float rr = rs[r];
          v.x = __fmul_rn(__fmul_rn(v.x, rr), __ldg(gnorm + k));
          v.y = __fmul_rn(__fmul_rn(v.y, rr), __ldg(gnorm + k + 1));
          v.z = __fmul_rn(__fmul_rn(v.z, rr), __ldg(gnorm + k + 2));
          v.w = __fmul_rn(__fmul_rn(v.w, rr), __ldg(gnorm + k + 3));
        }
      }
      As[4 * kc + 0][r] = v.x;
      As[4 * kc + 1][r] = v.y;
      As[4 * kc + 2][r] = v.z;
      As[4 * kc + 3][r] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(bw[j], av[i], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + ty * 8 + i;
    unsigned long long best = 0ull;
#pragma unroll
    for (int jp = 0; jp < 2; ++jp) {
      const int p = p0 + 2 * tx + jp;
      if (m < n && p < ms.n_pairs)
        best = umax64(best, epilogue<EPI>(ep, m, p, acc[i][2 * jp], acc[i][2 * jp + 1]));
    }
    if (EPI == EPI_VOCAB) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
      if (tx == 0 && m < n && best) atomicMax(ep.keys + m, best);
    }
  }
}

}  // namespace q6w
