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
//  * packed weights: the 128 rows x 48 bytes of int6 codes of a K step arrive
//    by one 2-D TMA tensor load (no multicast; two 64-row boxes in GLU mode),
//    6 steps deep;
//  * MMA stages (4): the weight rows expanded to bf16 by the decode warps
//    (16 KB) and the 192 activation rows, bulk-copied from the pre-swizzled
//    activation image (24 KB).
// Split K.  A matrix with few tiles (wq|wk|wv, wo, w2 of the 1.1B shape: 16-20
// tiles of 128 rows) would occupy 16-20 SMs; instead a thread-block cluster of
// C CTAs (C = 2, 4 or 8) shares one tile, each CTA taking K steps
// [c nks/C, (c+1) nks/C).  After its MMAs a CTA writes its partial tile
// (128 rows x 64 activations, FP32, the three parts already added) to its own
// shared memory slot of the CTA owning each activation slice (stores through
// distributed shared memory); after a cluster barrier CTA c sums, in rank
// order, the C partials of activations [c 64/C, (c+1) 64/C) and runs the
// epilogue for them.  No multicast.
// Warps 0-7 expand (warps w and w+4 take the two halves of row 32(w%4)+lane)
// and later run the epilogue (TMEM lane quadrant w%4; warps 0-3 activations
// 0-31, warps 4-7 activations 32-63), warp 8 issues the copies (lane 0 the
// weight loads, lane 1 the activation loads), warp 9 issues the MMAs and owns
// TMEM.  Every wait is bounded; a timeout sets an error bit and the CTA stops.
#pragma once

#include <cooperative_groups.h>
#include <cuda.h>

#include "async.cuh"
#include "linear.cuh"
#include "tc.cuh"

namespace q6w {
namespace tcg {

constexpr int kWR = 128;          // weight rows per tile (MMA M)
constexpr int kAR = 64;           // activation rows per tile (x 3 parts = MMA N)
constexpr int kN = 3 * kAR;       // 192
constexpr int kS = 4;             // MMA stages
constexpr int kMaxSplit = 8;      // CTAs of a cluster splitting one tile's K range
constexpr int kG = 1;             // K steps per packed-weight group (one TMA box)
constexpr int kP = 6;             // packed-weight groups in the ring
// Boxes wider than 128 bytes per row (kG > 2) delivered wrong bytes in the
// parity tests here; 48 and 96 bytes were exact and equally fast.
static_assert(48 * kG <= 128, "TMA box rows of at most 128 bytes");
constexpr int kThreads = 320;     // 10 warps
constexpr int kDW = 8;            // expand / epilogue warps
constexpr uint32_t kAT = kWR * 128;   // bytes of a decoded weight tile (one K step)
constexpr uint32_t kBT = kN * 128;    // bytes of an activation tile (one K step)
constexpr uint32_t kMS = kAT + kBT;   // 40960, a multiple of 1024
constexpr uint32_t kPT = kWR * 48 * kG;  // packed bytes of a weight tile (one group of K steps)
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
// box 48 kG bytes x 128 rows (64 rows in GLU mode).
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
  __shared__ uint64_t tmem_full, glu_ready, drain;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ float glu_x[kWR / 2][kAR + 1];  // GLU: W3 values handed to the W1 lanes
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr bool kGlu = EPI == GEPI_GLU;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* packed = smem + (size_t)kS * kMS;
  const int C = (int)cl.num_blocks(), c = (int)cl.block_rank();
  const int nks = a.K / 64;
  const int wtiles = kGlu ? a.ms.n_pairs / (kWR / 2) : (2 * a.ms.n_pairs) / kWR;
  const int it = blockIdx.x / C;  // one item (weight tile, activation tile) per cluster
  const int wt = it % wtiles, at = it / wtiles;
  const int ks0 = c * (nks / C), nk = nks / C;  // this CTA's K steps

  if (warp == kDW + 1) {
    tc::tmem_alloc(&tmem_base, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int p = 0; p < kP; ++p) {
      mbar_init(pk_full + p, 1);
      mbar_init(pk_empty + p, kDW);
    }
    for (int s = 0; s < kS; ++s) {
      mbar_init(act_full + s, 1);
      mbar_init(a_full + s, kDW);
      mbar_init(mma_empty + s, 1);
    }
    mbar_init(&tmem_full, 1);
    mbar_init(&glu_ready, kDW / 2);
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t taddr = tmem_base;

  if (warp == kDW) {
    if (lane == 0) {
      // ---- weight loads: one TMA box (two in GLU mode) per K step
      int mi, r0;
      weight_row(a.ms, kGlu, wt, 0, mi, r0);
      for (int g = 0; g < nk && !abort_flag; ++g) {
        const int p = g % kP;
        if (g >= kP && !mbar_wait(pk_empty + p, ((g / kP) - 1) & 1)) {
          abort_flag = 1;
          atomicOr(a.err, tc::kErrTimeout);
          break;
        }
        uint8_t* dst = packed + (size_t)p * kPT;
        const int x = (ks0 + g) * 48;
        mbar_expect_tx(pk_full + p, kPT);
        if (kGlu) {
          tma_load_2d(dst, &maps.m[0], x, r0, pk_full + p);
          tma_load_2d(dst + (kWR / 2) * 48, &maps.m[1], x, r0, pk_full + p);
        } else {
          tma_load_2d(dst, &maps.m[mi], x, r0, pk_full + p);
        }
      }
    } else if (lane == 1) {
      // ---- activation loads: 3 bulk copies (one per part) per K step
      const int64_t arow = (int64_t)at * kAR;
      const uint8_t* isrc = a.img + (arow >> 7) * (3 * (int64_t)a.K * 256) + (arow & 127) * 128;
      for (int g = 0; g < nk && !abort_flag; ++g) {
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
          bulk_g2s(st + p * (kAR * 128), isrc + (int64_t)p * a.K * 256 + (int64_t)(ks0 + g) * 16384, kAR * 128,
                   act_full + s);
      }
    }
  } else if (warp == kDW + 1) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) |
                             ((uint32_t)(kWR >> 4) << 24);
      bool ok = true;
      for (int g = 0; g < nk && !abort_flag; ++g) {
        const int s = g % kS;
        if (!mbar_wait(act_full + s, (g / kS) & 1) || !mbar_wait(a_full + s, (g / kS) & 1)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t a0 = smem_u32(smem + (size_t)s * kMS), b0 = a0 + kAT;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::umma(taddr, tc::sdesc(a0 + kk * 32), tc::sdesc(b0 + kk * 32), idesc, (g | kk) != 0);
        tc::umma_commit(mma_empty + s);
      }
      if (!ok) {
        abort_flag = 1;
        atomicOr(a.err, tc::kErrTimeout);
      } else {
        tc::umma_commit(&tmem_full);
      }
      // every MMA this thread issued has finished before TMEM is released
      tc::umma_commit(&drain);
      if (!mbar_wait(&drain, 0)) atomicOr(a.err, tc::kErrTimeout);
    }
  } else {
    // ---- warps 0-7: expand weights
    const int j = ((warp & 3) << 5) | lane;  // weight row this thread expands
    const int half = warp >> 2;               // units 2 half, 2 half + 1 of the step
    for (int g = 0; g < nk; ++g) {
      const int p = g % kP, s = g % kS;
      bool got = !abort_flag && mbar_wait(pk_full + p, (g / kP) & 1);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform: the warp leaves together
      const uint2* pp = reinterpret_cast<const uint2*>(packed + (size_t)p * kPT + j * 48 + half * 24);
      const uint2 p0 = pp[0], p1 = pp[1], p2 = pp[2];
      __syncwarp();
      if (lane == 0) mbar_arrive(pk_empty + p);  // the packed step is in registers
      // the MMA of this stage's previous use has finished reading its weight tile
      got = g < kS || mbar_wait(mma_empty + s, ((g / kS) - 1) & 1);
      if (!__all_sync(0xffffffffu, got)) break;
      const uint32_t w[6] = {p0.x, p0.y, p1.x, p1.y, p2.x, p2.y};
      uint8_t* line = smem + (size_t)s * kMS + j * 128;
#pragma unroll
      for (int uu = 0; uu < 2; ++uu) {
        const uint32_t w0 = w[3 * uu], w1 = w[3 * uu + 1], w2 = w[3 * uu + 2];
        const uint32_t f[16] = {w0, w0 >> 6, w0 >> 12, w0 >> 18, w0 >> 24, __funnelshift_r(w0, w1, 30),
                                w1 >> 4, w1 >> 10, w1 >> 16, w1 >> 22, __funnelshift_r(w1, w2, 28),
                                w2 >> 2, w2 >> 8, w2 >> 14, w2 >> 20, w2 >> 26};
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          pk[e] = (__float_as_uint(code_to_float(f[2 * e])) >> 16) |
                  (__float_as_uint(code_to_float(f[2 * e + 1])) & 0xFFFF0000u);
        const int lu = 2 * (2 * half + uu);
        reinterpret_cast<uint4*>(line)[lu ^ (j & 7)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        reinterpret_cast<uint4*>(line)[(lu + 1) ^ (j & 7)] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      tc::fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full + s);
    }
  }

  // ---- partial tile -> the shared memory of the CTA that owns each activation
  // slice: CTA q receives, for activations [q SA, (q+1) SA), one slot per rank
  // (stage memory, free once this CTA's MMAs are done; a peer writes into it
  // only after its own K loop, and every CTA's MMAs finish before the barrier)
  const int SA = kAR / C, SH = SA / 2;
  float* recv = reinterpret_cast<float*>(smem);  // [C ranks][128 rows][SA]
  const int j = ((warp & 3) << 5) | lane;
  const int half = (warp >> 2) & 1;
  // every CTA's MMAs are done before any peer writes into its stage memory
  if (warp < kDW) {
    const bool full = __all_sync(0xffffffffu, !abort_flag && mbar_wait(&tmem_full, 0));
    if (!full && lane == 0) {
      abort_flag = 1;
      atomicOr(a.err, tc::kErrTimeout);
    }
  }
  tc::tc_fence_before();
  cl.sync();
  if (warp < kDW) {
    tc::tc_fence_after();
    const uint32_t lane_addr = taddr + ((uint32_t)((warp & 3) * 32) << 16);
    float d0[32], d1[32], d2[32];
    tc::tmem_ld32(lane_addr + half * 32, d0);
    tc::tmem_ld32(lane_addr + kAR + half * 32, d1);
    tc::tmem_ld32(lane_addr + 2 * kAR + half * 32, d2);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int la = half * 32 + i;  // local activation
      const int q = la / SA;         // owner rank
      float* dst = C == 1 ? recv : cl.map_shared_rank(recv, q);
      dst[((size_t)c * kWR + j) * SA + (la - q * SA)] = __fadd_rn(__fadd_rn(d0[i], d1[i]), d2[i]);
    }
  }
  tc::tc_fence_before();
  cl.sync();  // every partial has landed in its owner

  // ---- this CTA's activations: [c SA, (c+1) SA); warps w, w+4 take halves
  if (warp < kDW) {
    int mi, r;
    weight_row(a.ms, kGlu, wt, j, mi, r);
    const float scale = __ldg(scale_ptr(a.ms, mi) + r);
    const int a0 = at * kAR + c * SA + half * SH;  // global activation row of y[0]
    float y[kAR / 2];
#pragma unroll
    for (int i = 0; i < kAR / 2; ++i) {
      float v = 0.f;
      if (i < SH)
        for (int q = 0; q < C; ++q) {  // rank order: one summation order everywhere
          const float pv = recv[((size_t)q * kWR + j) * SA + half * SH + i];
          v = q == 0 ? pv : __fadd_rn(v, pv);
        }
      y[i] = __fmul_rn(v, scale);
    }
    const EpiArgs& ep = a.ep;
    if (EPI == GEPI_GLU) {
      // rows 64..127 (warps 2, 3, 6, 7) hold W3: hand them to the W1 rows
      if (j >= kWR / 2) {
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i)
          if (i < SH) glu_x[j - kWR / 2][half * SH + i] = y[i];
        __syncwarp();
        if (lane == 0) mbar_arrive(&glu_ready);
      } else if (__all_sync(0xffffffffu, mbar_wait(&glu_ready, 0))) {
        const int p = wt * (kWR / 2) + j;
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i)
          if (i < SH && a0 + i < a.n) epilogue<EPI_GLU>(ep, a0 + i, p, y[i], glu_x[j][half * SH + i]);
      } else if (lane == 0) {
        atomicOr(a.err, tc::kErrTimeout);
      }
    } else {
      // pairs (2p, 2p+1) sit on adjacent lanes; the even lane finishes the pair.
      // Every global value needed is loaded for all of the thread's activations
      // before any store, so the loads overlap.
      const int vrow = wt * kWR + j;
      const bool lead = !(j & 1);
      float other[kAR / 2];
#pragma unroll
      for (int i = 0; i < kAR / 2; ++i) other[i] = __shfl_xor_sync(0xffffffffu, y[i], 1);
      if (EPI == GEPI_RESID) {
        float2 old[kAR / 2];
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i)
          old[i] = i < SH && lead && a0 + i < a.n
                       ? *reinterpret_cast<const float2*>(ep.y + (int64_t)(a0 + i) * ep.ldy + vrow)
                       : make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i)
          if (i < SH && lead && a0 + i < a.n)
            *reinterpret_cast<float2*>(ep.y + (int64_t)(a0 + i) * ep.ldy + vrow) =
                make_float2(__fadd_rn(old[i].x, y[i]), __fadd_rn(old[i].y, other[i]));
      } else if (EPI == GEPI_QKV) {
        // RoPE of torch_benchmark.py:84 (each product rounded before the add);
        // q to the query buffer, k and v to the cache row of the activation's sequence
        const bool rope = vrow < ep.q_rows + ep.kv_rows;
        const int jr = (vrow % ep.hd) >> 1;
        int pos[kAR / 2];
        int64_t crow[kAR / 2];
        bool live[kAR / 2];
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i) {
          const int m = a0 + i;
          live[i] = i < SH && lead && m < a.n && !(ep.flags[m] & SEQ_INVALID);
          pos[i] = live[i] ? ep.pos[m] : 0;
          crow[i] = live[i] && ep.seq ? ep.seq[m] : m;
        }
        float cs[kAR / 2], sn[kAR / 2];
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i) {
          cs[i] = live[i] && rope ? __ldg(ep.rope_cos + (int64_t)pos[i] * (ep.hd >> 1) + jr) : 0.f;
          sn[i] = live[i] && rope ? __ldg(ep.rope_sin + (int64_t)pos[i] * (ep.hd >> 1) + jr) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i) {
          if (!live[i]) continue;
          float ra = y[i], rb = other[i];
          if (rope) {
            ra = __fsub_rn(__fmul_rn(y[i], cs[i]), __fmul_rn(other[i], sn[i]));
            rb = __fadd_rn(__fmul_rn(y[i], sn[i]), __fmul_rn(other[i], cs[i]));
          }
          float* dst;
          if (vrow < ep.q_rows)
            dst = ep.qbuf + (int64_t)(a0 + i) * ep.ldq + vrow;
          else if (vrow < ep.q_rows + ep.kv_rows)
            dst = ep.kc + crow[i] * ep.cache_stride + ep.layer_off + (int64_t)pos[i] * ep.kv_rows + (vrow - ep.q_rows);
          else
            dst = ep.vc + crow[i] * ep.cache_stride + ep.layer_off + (int64_t)pos[i] * ep.kv_rows +
                  (vrow - ep.q_rows - ep.kv_rows);
          *reinterpret_cast<float2*>(dst) = make_float2(ra, rb);
        }
      } else {  // GEPI_VOCAB: logits, dumped step logits, stop masking, first-maximum key
        int gen[kAR / 2], fl[kAR / 2], pos[kAR / 2], plen[kAR / 2];
        const bool need = ep.step_logits || ep.n_stop;
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i) {
          const int m = a0 + i;
          const bool in = need && i < SH && lead && m < a.n;
          gen[i] = in ? ep.gen[m] : 0;
          fl[i] = in ? ep.flags[m] : 0;
          pos[i] = in && ep.step_logits ? ep.pos[m] : 0;
          plen[i] = in && ep.step_logits ? ep.plen[m] : 0;
        }
#pragma unroll
        for (int i = 0; i < kAR / 2; ++i) {
          if (i >= SH) break;
          const int m = a0 + i;
          unsigned long long key = 0ull;
          if (lead && m < a.n) {
            float va = y[i], vb = other[i];
            if (ep.y) *reinterpret_cast<float2*>(ep.y + (int64_t)m * ep.ldy + vrow) = make_float2(va, vb);
            if (ep.step_logits && !(fl[i] & (SEQ_DONE | SEQ_INVALID)) && pos[i] >= plen[i] - 1)
              *reinterpret_cast<float2*>(ep.step_logits + ((int64_t)m * ep.new_tokens + gen[i]) * ep.vocab + vrow) =
                  make_float2(va, vb);
            if (ep.n_stop && gen[i] < ep.min_new) {
              for (int t = 0; t < ep.n_stop; ++t) {
                if (ep.stop_ids[t] == vrow) va = -INFINITY;
                if (ep.stop_ids[t] == vrow + 1) vb = -INFINITY;
              }
            }
            key = umax64(argmax_key(va, vrow), argmax_key(vb, vrow + 1));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, o));
          if (lane == 0 && key && m < a.n) atomicMax(ep.keys + m, key);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kDW + 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(taddr, 256);
  }
}

// Activation image (tc.cuh layout, K columns) of rows x[0..n): RMSNorm with
// weight g when g is given (torch_benchmark.py:22-24), else the rows as they
// are.  One CTA of 256 threads per row, each thread 8-column chunks
// k0 = 8 tid + 2048 i (K <= 6144: at most three per thread), all loaded before
// the reduction; rows beyond n are left as they are (never used).
constexpr int kImgThreads = 256;
constexpr int kImgChunks = 3;

__global__ void __launch_bounds__(kImgThreads) image_kernel(const float* __restrict__ x, int ldx, int n, int K,
                                                            const float* __restrict__ g, float eps,
                                                            uint8_t* __restrict__ img) {
  __shared__ float red[kImgThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  const float* xr = x + row * ldx;
  float v[kImgChunks][8];
#pragma unroll
  for (int c = 0; c < kImgChunks; ++c) {
    const int k0 = 8 * tid + 8 * kImgThreads * c;
    if (k0 < K) {
      const float4 lo = *reinterpret_cast<const float4*>(xr + k0);
      const float4 hi = *reinterpret_cast<const float4*>(xr + k0 + 4);
      v[c][0] = lo.x; v[c][1] = lo.y; v[c][2] = lo.z; v[c][3] = lo.w;
      v[c][4] = hi.x; v[c][5] = hi.y; v[c][6] = hi.z; v[c][7] = hi.w;
    }
  }
  if (g) {
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < kImgChunks; ++c)
      if (8 * tid + 8 * kImgThreads * c < K)
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[c][i], v[c][i]));
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = lane < kImgThreads / 32 ? red[lane] : 0.0f;
    t = warp_sum(t);
    const float r = rms_scale(t, K, eps);
#pragma unroll
    for (int c = 0; c < kImgChunks; ++c) {
      const int k0 = 8 * tid + 8 * kImgThreads * c;
      if (k0 < K)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = __fmul_rn(__fmul_rn(v[c][i], r), __ldg(g + k0 + i));
    }
  }
#pragma unroll
  for (int c = 0; c < kImgChunks; ++c) {
    const int k0 = 8 * tid + 8 * kImgThreads * c;
    if (k0 < K) tc::img_store8(img, row, k0, K, v[c]);
  }
}

}  // namespace tcg
}  // namespace q6w
