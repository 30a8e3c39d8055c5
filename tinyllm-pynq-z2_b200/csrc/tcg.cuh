// Tensor-core (tcgen05) linears for models of any width (dim, hidden and K
// multiples of 64): the batched step of the 1.1B-shape config at B = 64 and
// the like.
//
// Roles are swapped against the dim-128 kernel in tc.cuh: the weights are the
// MMA's M operand (128 rows per tile) and the activations its N operand, the
// three bf16 parts (hi, mid, lo) of 64 activation rows stacked as N = 192:
//   D[128 weight rows, 192] = W[128, K] . [A_hi; A_mid; A_lo][192, K]^T
// and y[a][r] = ((D[r][a] + D[r][64+a]) + D[r][128+a]) * scale[r], which is
// sum_k q_k u_k with exact bf16 products and FP32 accumulation (the parts hold
// u's 24-bit significand), times the row scale once.
//
// Two rings, per K step of 64 columns (one 128-byte swizzle atom):
//  * packed weights: the 128 rows x 48 bytes of int6 codes arrive by one 2-D
//    TMA tensor load (no multicast) per step (two 64-row boxes in GLU mode),
//    12 steps deep, so a CTA keeps 72 KB of weight reads in flight;
//  * MMA stages (3): the weight rows expanded to bf16 by the decode warps
//    (16 KB) and the 192 activation rows, bulk-copied from the pre-swizzled
//    activation image (24 KB).
// Warps 0-3 expand and later run the epilogue (TMEM lane quadrants 0-3), warp
// 4 issues the copies (lane 0 the weight loads, lane 1 the activation loads),
// warp 5 issues the MMAs and owns TMEM.  Every wait is bounded; a timeout sets
// an error bit and the CTA stops.
#pragma once

#include <cuda.h>

#include "async.cuh"
#include "linear.cuh"
#include "tc.cuh"

namespace q6w {
namespace tcg {

constexpr int kWR = 128;          // weight rows per tile (MMA M)
constexpr int kAR = 64;           // activation rows per tile (x 3 parts = MMA N)
constexpr int kN = 3 * kAR;       // 192
constexpr int kS = 3;             // MMA stages
constexpr int kP = 12;            // packed-weight stages
constexpr int kThreads = 192;     // 6 warps
constexpr uint32_t kAT = kWR * 128;   // bytes of a decoded weight tile (one K step)
constexpr uint32_t kBT = kN * 128;    // bytes of an activation tile (one K step)
constexpr uint32_t kMS = kAT + kBT;   // 40960, a multiple of 1024
constexpr uint32_t kPT = kWR * 48;    // packed bytes of a weight tile (one K step)
constexpr size_t kSmem = 1024 + (size_t)kS * kMS + (size_t)kP * kPT;

enum { GEPI_QKV = 0, GEPI_RESID = 1, GEPI_GLU = 2, GEPI_VOCAB = 3 };

struct GArgs {
  const uint8_t* img;   // activation image (tc.cuh layout) of K columns
  int32_t n, K;
  MatSet ms;            // weights; GLU: pairs (W1 row j, W3 row j)
  EpiArgs ep;
  int32_t* err;
};

// Tensor maps of the (up to three) weight matrices: 2-D uint8 [rows][K*3/4],
// box 48 bytes x 128 rows (64 rows in GLU mode).
struct GMaps {
  CUtensorMap m[3];
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Weight tile t's row j (0..127): matrix index (0..2), row in that matrix.
__device__ __forceinline__ void weight_row(const MatSet& ms, bool glu, int t, int j, int& mi, int& r) {
  if (glu) {
    mi = j < kWR / 2 ? 0 : 1;
    r = t * (kWR / 2) + (j & (kWR / 2 - 1));
    return;
  }
  const int v = t * kWR + j;
  if (v < ms.end0) {
    mi = 0; r = v;
  } else if (v < ms.end1) {
    mi = 1; r = v - ms.end0;
  } else {
    mi = 2; r = v - ms.end1;
  }
}

__device__ __forceinline__ const float* scale_ptr(const MatSet& ms, int mi) {
  return mi == 0 ? ms.s0 : (mi == 1 ? ms.s1 : ms.s2);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) tcg_kernel(GArgs a, const __grid_constant__ GMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t pk_full[kP], pk_empty[kP], act_full[kS], a_full[kS], mma_empty[kS];
  __shared__ uint64_t tmem_full, tmem_empty, glu_ready, glu_free, drain;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ float glu_x[kWR / 2][kAR + 1];  // GLU: W3 values handed to the W1 lanes
  constexpr bool kGlu = EPI == GEPI_GLU;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* packed = smem + (size_t)kS * kMS;
  const int nks = a.K / 64;
  const int wtiles = kGlu ? a.ms.n_pairs / (kWR / 2) : (2 * a.ms.n_pairs) / kWR;
  const int atiles = (a.n + kAR - 1) / kAR;
  const int items = wtiles * atiles;

  if (warp == 5) {
    tc::tmem_alloc(&tmem_base, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int p = 0; p < kP; ++p) {
      mbar_init(pk_full + p, 1);
      mbar_init(pk_empty + p, 4);
    }
    for (int s = 0; s < kS; ++s) {
      mbar_init(act_full + s, 1);
      mbar_init(a_full + s, 4);
      mbar_init(mma_empty + s, 1);
    }
    mbar_init(&tmem_full, 1);
    mbar_init(&tmem_empty, 4);
    mbar_init(&glu_ready, 2);
    mbar_init(&glu_free, 2);
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t taddr = tmem_base;

  if (warp == 4) {
    if (lane == 0) {
      // ---- weight loads: one TMA box (two in GLU mode) per K step, kP steps ahead
      int g = 0;
      for (int it = blockIdx.x; it < items && !abort_flag; it += gridDim.x) {
        const int wt = it % wtiles;
        int mi, r0;
        weight_row(a.ms, kGlu, wt, 0, mi, r0);
        for (int ks = 0; ks < nks; ++ks, ++g) {
          const int p = g % kP;
          if (g >= kP && !mbar_wait(pk_empty + p, ((g / kP) - 1) & 1)) {
            abort_flag = 1;
            atomicOr(a.err, tc::kErrTimeout);
            break;
          }
          uint8_t* dst = packed + (size_t)p * kPT;
          mbar_expect_tx(pk_full + p, kPT);
          if (kGlu) {
            tma_load_2d(dst, &maps.m[0], ks * 48, r0, pk_full + p);
            tma_load_2d(dst + (kWR / 2) * 48, &maps.m[1], ks * 48, r0, pk_full + p);
          } else {
            tma_load_2d(dst, &maps.m[mi], ks * 48, r0, pk_full + p);
          }
        }
      }
    } else if (lane == 1) {
      // ---- activation loads: 3 bulk copies (one per part) per K step
      int g = 0;
      for (int it = blockIdx.x; it < items && !abort_flag; it += gridDim.x) {
        const int at = it / wtiles;
        const int64_t arow = (int64_t)at * kAR;
        const uint8_t* isrc = a.img + (arow >> 7) * (3 * (int64_t)a.K * 256) + (arow & 127) * 128;
        for (int ks = 0; ks < nks; ++ks, ++g) {
          const int s = g % kS;
          if (g >= kS && !mbar_wait(mma_empty + s, ((g / kS) - 1) & 1)) {
            abort_flag = 1;
            atomicOr(a.err, tc::kErrTimeout);
            break;
          }
          uint8_t* st = smem + (size_t)s * kMS + kAT;
          mbar_expect_tx(act_full + s, kBT);
#pragma unroll
          for (int p = 0; p < 3; ++p)
            bulk_g2s(st + p * (kAR * 128), isrc + (int64_t)p * a.K * 256 + (int64_t)ks * 16384, kAR * 128,
                     act_full + s);
        }
      }
    }
  } else if (warp == 5) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) |
                             ((uint32_t)(kWR >> 4) << 24);
      int g = 0, idx = 0;
      for (int it = blockIdx.x; it < items && !abort_flag; it += gridDim.x, ++idx) {
        if (idx > 0 && !mbar_wait(&tmem_empty, (idx - 1) & 1)) {
          abort_flag = 1;
          atomicOr(a.err, tc::kErrTimeout);
          break;
        }
        tc::tc_fence_after();
        bool ok = true;
        for (int ks = 0; ks < nks; ++ks, ++g) {
          const int s = g % kS;
          if (!mbar_wait(act_full + s, (g / kS) & 1) || !mbar_wait(a_full + s, (g / kS) & 1)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = smem_u32(smem + (size_t)s * kMS), b0 = a0 + kAT;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::umma(taddr, tc::sdesc(a0 + kk * 32), tc::sdesc(b0 + kk * 32), idesc, (ks | kk) != 0);
          tc::umma_commit(mma_empty + s);
        }
        if (!ok) {
          abort_flag = 1;
          atomicOr(a.err, tc::kErrTimeout);
          break;
        }
        tc::umma_commit(&tmem_full);
      }
      // every MMA this thread issued has finished before TMEM is released
      tc::umma_commit(&drain);
      if (!mbar_wait(&drain, 0)) atomicOr(a.err, tc::kErrTimeout);
    }
  } else {
    // ---- warps 0-3: expand weights, then the epilogue of each item
    const int j = tid;  // weight row of the tile this thread expands / owns in TMEM
    int g = 0, idx = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++idx) {
      const int wt = it % wtiles, at = it / wtiles;
      bool ok = true;
      for (int ks = 0; ks < nks; ++ks, ++g) {
        const int p = g % kP, s = g % kS;
        bool got = !abort_flag && mbar_wait(pk_full + p, (g / kP) & 1);
        if (!__all_sync(0xffffffffu, got)) {  // warp-uniform: the warp leaves together
          ok = false;
          break;
        }
        const uint4* pp = reinterpret_cast<const uint4*>(packed + (size_t)p * kPT + j * 48);
        const uint4 p0 = pp[0], p1 = pp[1], p2 = pp[2];
        __syncwarp();
        if (lane == 0) mbar_arrive(pk_empty + p);  // the packed stage is in registers
        // the MMA of this stage's previous use has finished reading its weight tile
        got = g < kS || mbar_wait(mma_empty + s, ((g / kS) - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t w[12] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w, p2.x, p2.y, p2.z, p2.w};
        uint8_t* line = smem + (size_t)s * kMS + j * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t w0 = w[3 * u], w1 = w[3 * u + 1], w2 = w[3 * u + 2];
          const uint32_t f[16] = {w0, w0 >> 6, w0 >> 12, w0 >> 18, w0 >> 24, __funnelshift_r(w0, w1, 30),
                                  w1 >> 4, w1 >> 10, w1 >> 16, w1 >> 22, __funnelshift_r(w1, w2, 28),
                                  w2 >> 2, w2 >> 8, w2 >> 14, w2 >> 20, w2 >> 26};
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            pk[e] = (__float_as_uint(code_to_float(f[2 * e])) >> 16) |
                    (__float_as_uint(code_to_float(f[2 * e + 1])) & 0xFFFF0000u);
          const int lu = 2 * u;
          reinterpret_cast<uint4*>(line)[lu ^ (j & 7)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(line)[(lu + 1) ^ (j & 7)] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + s);
      }
      bool full = ok && mbar_wait(&tmem_full, idx & 1);
      if (!__all_sync(0xffffffffu, full)) {
        if (lane == 0) {
          abort_flag = 1;
          atomicOr(a.err, tc::kErrTimeout);
        }
        break;
      }
      tc::tc_fence_after();
      // ---- epilogue: this thread holds weight row j of the tile, all 192 columns
      int mi, r;
      weight_row(a.ms, kGlu, wt, j, mi, r);
      const float scale = __ldg(scale_ptr(a.ms, mi) + r);
      const uint32_t lane_addr = taddr + ((uint32_t)(warp * 32) << 16);
      float y[kAR];
#pragma unroll
      for (int c = 0; c < kAR; c += 32) {
        float d0[32], d1[32], d2[32];
        tc::tmem_ld32(lane_addr + c, d0);
        tc::tmem_ld32(lane_addr + kAR + c, d1);
        tc::tmem_ld32(lane_addr + 2 * kAR + c, d2);
#pragma unroll
        for (int i = 0; i < 32; ++i) y[c + i] = __fmul_rn(__fadd_rn(__fadd_rn(d0[i], d1[i]), d2[i]), scale);
      }
      // TMEM is free for the next item's MMAs
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty);
      const int a0 = at * kAR;
      if (EPI == GEPI_GLU) {
        // rows 64..127 (warps 2, 3) hold W3: hand them to the W1 lanes (warps 0, 1)
        // through shared memory, with bounded waits on both hand-offs
        bool fine = true;
        if (j >= kWR / 2) {
          if (idx > 0) fine = mbar_wait(&glu_free, (idx - 1) & 1);
          fine = __all_sync(0xffffffffu, fine);
          if (fine)
#pragma unroll
            for (int i = 0; i < kAR; ++i) glu_x[j - kWR / 2][i] = y[i];
          __syncwarp();
          if (lane == 0) mbar_arrive(&glu_ready);
        } else {
          fine = __all_sync(0xffffffffu, mbar_wait(&glu_ready, idx & 1));
          if (fine) {
            const int p = wt * (kWR / 2) + j;
#pragma unroll
            for (int i = 0; i < kAR; ++i)
              if (a0 + i < a.n) epilogue<EPI_GLU>(a.ep, a0 + i, p, y[i], glu_x[j][i]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&glu_free);
        }
        if (!fine) {
          if (lane == 0) {
            abort_flag = 1;
            atomicOr(a.err, tc::kErrTimeout);
          }
          break;
        }
      } else {
        // pairs (2p, 2p+1) sit on adjacent lanes
        const int vrow = wt * kWR + j;  // row of the concatenation
#pragma unroll
        for (int i = 0; i < kAR; ++i) {
          const float other = __shfl_xor_sync(0xffffffffu, y[i], 1);
          unsigned long long key = 0ull;
          if (!(j & 1) && a0 + i < a.n) {
            if (EPI == GEPI_QKV) key = epilogue<EPI_QKV>(a.ep, a0 + i, vrow >> 1, y[i], other);
            if (EPI == GEPI_RESID) key = epilogue<EPI_RESID>(a.ep, a0 + i, vrow >> 1, y[i], other);
            if (EPI == GEPI_VOCAB) key = epilogue<EPI_VOCAB>(a.ep, a0 + i, vrow >> 1, y[i], other);
          }
          if (EPI == GEPI_VOCAB) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, o));
            if (lane == 0 && key && a0 + i < a.n) atomicMax(a.ep.keys + a0 + i, key);
          }
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc::tc_fence_after();
    tc::tmem_dealloc(taddr, 256);
  }
}

// Activation image (tc.cuh layout, K columns) of rows x[0..n): RMSNorm with
// weight g when g is given (torch_benchmark.py:22-24), else the rows as they
// are.  One warp per row; rows beyond n are left as they are (never used).
__global__ void image_kernel(const float* __restrict__ x, int ldx, int n, int K, const float* __restrict__ g,
                             float eps, uint8_t* __restrict__ img) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  const float* xr = x + row * ldx;
  float r = 1.0f;
  if (g) {
    float ss = 0.0f;
    for (int k = lane * 4; k < K; k += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + k);
      ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
      ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
      ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
      ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    }
    ss = warp_sum(ss);
    r = rms_scale(ss, K, eps);
  }
  for (int k0 = lane * 8; k0 < K; k0 += 256) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float xv = xr[k0 + i];
      v[i] = g ? __fmul_rn(__fmul_rn(xv, r), __ldg(g + k0 + i)) : xv;
    }
    tc::img_store8(img, row, k0, K, v);
  }
}

}  // namespace tcg
}  // namespace q6w
