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
// Per K step of 128 columns (two 128-byte swizzle atoms), three rings:
//  * packed weights: the 128 rows x 96 bytes of int6 codes of a K step arrive
//    by one 2-D TMA tensor load (no multicast; two 64-row boxes in GLU mode),
//    6 steps deep;
//  * expanded weights (3 stages of 64 columns) in tensor memory: the decode
//    warps write the bf16 rows with tcgen05.st (row r on TMEM lane r, two K
//    elements per column, in the pair order of expand_group) and the MMA
//    reads its A operand from there, so the expansion costs no shared-memory
//    bandwidth;
//  * activations (3 stages of 48 KB): the 192 rows of both 64-column chunks,
//    bulk-copied from the pre-swizzled activation image, the MMA's B operand.
// One commit per step frees a weight stage and an activation stage together.
// Every K step pays a fixed handshake latency (barrier waits and arrivals,
// the commit); 128 columns a step halve its share against 64.
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
// 0-31, warps 4-7 activations 32-63), warp 8 issues the weight loads, warp
// 9 the MMAs (and owns TMEM), warp 10 the activation loads: each waiting role
// has a warp of its own, so no role's wait holds up another's issue.
// Every wait is bounded; a timeout sets an error bit and the CTA stops.
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
constexpr int kG = 2;             // 64-column chunks per K step (one TMA box of 48 kG bytes a row)
constexpr int kS = 3;             // K-step stages: activations (shared memory) + expanded weights (TMEM)
constexpr int kMaxSplit = 8;      // CTAs of a cluster splitting one tile's K range
constexpr int kP = 6;             // packed-weight K steps in the ring
// Boxes wider than 128 bytes per row (kG > 2) delivered wrong bytes in the
// parity tests here; 48 and 96 bytes were exact.
static_assert(48 * kG <= 128, "TMA box rows of at most 128 bytes");
constexpr int kThreads = 352;     // 11 warps
constexpr int kDW = 8;            // expand / epilogue warps
constexpr uint32_t kBT = kG * kN * 128;  // activation bytes of a K step: [chunk][part][64 rows][128 B]
constexpr uint32_t kTmemCols = 512;      // accumulator [0, 192), weight stages from kAcol
constexpr uint32_t kAcol = 256;
constexpr uint32_t kAS = 32 * kG;        // TMEM columns of an expanded weight stage
static_assert(kAcol + kAS * kS <= kTmemCols && kN <= kAcol, "tensor memory columns");
constexpr uint32_t kPT = kWR * 48 * kG;  // packed bytes of a weight tile (one group of K steps)
constexpr size_t kSmem = 1024 + (size_t)kS * kBT + (size_t)kP * kPT;
// the partial tiles of every rank ([C][64 / C][128] floats) fit in the stage memory
static_assert((size_t)kWR * kAR * 4 <= (size_t)kS * kBT, "partial tiles exceed the stages");

enum { GEPI_QKV = 0, GEPI_RESID = 1, GEPI_GLU = 2, GEPI_VOCAB = 3, GEPI_STORE = 4 };

// Weight tiles of a launch: whole 128-row tiles, except the plain linear
// (GEPI_STORE), whose last tile may be partial (the TMA box reads zeros past
// the last row and the epilogue stores only rows that exist).
__host__ __device__ inline int weight_tiles(int epi, const MatSet& ms) {
  if (epi == GEPI_GLU) return ms.n_pairs / (kWR / 2);
  if (epi == GEPI_STORE) return (2 * ms.n_pairs + kWR - 1) / kWR;
  return (2 * ms.n_pairs) / kWR;
}

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

// ---- weight expansion -------------------------------------------------------
// A 12-byte group (words w0, w1, w2) holds codes 0..15 at bits 6f.  Codes whose
// bits start at the same offset inside their byte (0, 2, 4 or 6) are paired:
// one byte permute puts the pair's bytes in the two 16-bit halves of a word,
// one shift brings both codes to bits 0-5 and 16-21, one mask/xor makes each
// half the bf16 of 128 + (c ^ 32) (the 7-bit mantissa holds it), and one bf16x2
// subtraction of 160 leaves the signed value (c ^ 32) - 32 exactly.  The pairs, as TMEM columns
// 0..7 of the group, hold codes (0,4) (8,12) (3,7) (11,15) (2,6) (10,14)
// (1,5) (9,13): K order {0, 4, 8, 12, 3, 7, 11, 15, 2, 6, 10, 14, 1, 5, 9, 13}
// inside each group, the order in which image_kernel writes the activations,
// so the dot products are unchanged.
__device__ __forceinline__ uint32_t code_pair_bf16(uint32_t t) {
  // codes are two's complement: (c ^ 32) - 32 is the value (bit 5 flipped, as code_to_float)
  const uint32_t u = (t & 0x003F003Fu) ^ 0x43204320u;  // bf16x2 (128 + (c0 ^ 32), 128 + (c1 ^ 32))
  __nv_bfloat162_raw k;
  k.x = 0x4320;  // 160
  k.y = 0x4320;
  const __nv_bfloat162 d = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&u), __nv_bfloat162(k));
  return *reinterpret_cast<const uint32_t*>(&d);
}

__device__ __forceinline__ void expand_group(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t* out) {
  out[0] = code_pair_bf16(__byte_perm(w0, 0u, 0x3300));        // codes 0, 4   (offset 0)
  out[1] = code_pair_bf16(__byte_perm(w1, w2, 0x5522));        // codes 8, 12  (offset 0)
  out[2] = code_pair_bf16(__byte_perm(w0, w1, 0x5522) >> 2);   // codes 3, 7   (offset 2)
  out[3] = code_pair_bf16(__byte_perm(w2, 0u, 0x3300) >> 2);   // codes 11, 15 (offset 2)
  out[4] = code_pair_bf16(__byte_perm(w0, w1, 0x5421) >> 4);   // codes 2, 6   (offset 4)
  out[5] = code_pair_bf16(__byte_perm(w1, w2, 0x7643) >> 4);   // codes 10, 14 (offset 4)
  out[6] = code_pair_bf16(__byte_perm(w0, w1, 0x4310) >> 6);   // codes 1, 5   (offset 6)
  out[7] = code_pair_bf16(__byte_perm(w1, w2, 0x6532) >> 6);   // codes 9, 13  (offset 6)
}

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
  __shared__ uint64_t pk_full[kP], pk_empty[kP], act_full[kS], a_full[kS], st_empty[kS];
  __shared__ uint64_t tmem_full, drain;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ float srow[kWR];                 // row scales of the weight tile
  __shared__ int32_t mflags[kAR], mpos[kAR], mseq[kAR], mgen[kAR], mplen[kAR];  // per activation
  __shared__ unsigned long long vkey[kAR];    // VOCAB: this tile's first-maximum key per activation
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr bool kGlu = EPI == GEPI_GLU;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* packed = smem + (size_t)kS * kBT;
  const int C = (int)cl.num_blocks(), c = (int)cl.block_rank();
  const int nks = a.K / (64 * kG);
  const int wtiles = weight_tiles(EPI, a.ms);
  const int it = blockIdx.x / C;  // one item (weight tile, activation tile) per cluster
  const int wt = it % wtiles, at = it / wtiles;
  const int ks0 = c * (nks / C), nk = nks / C;  // this CTA's K steps

  if (warp == kDW + 1) {
    tc::tmem_alloc(&tmem_base, kTmemCols);
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
      mbar_init(st_empty + s, 1);
    }
    mbar_init(&tmem_full, 1);
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (EPI == GEPI_VOCAB && tid < kAR) vkey[tid] = 0ull;
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
        const int x = (ks0 + g) * 48 * kG;
        mbar_expect_tx(pk_full + p, kPT);
        if (kGlu) {
          tma_load_2d(dst, &maps.m[0], x, r0, pk_full + p);
          tma_load_2d(dst + (kWR / 2) * 48 * kG, &maps.m[1], x, r0, pk_full + p);
        } else {
          tma_load_2d(dst, &maps.m[mi], x, r0, pk_full + p);
        }
      }
    }
  } else if (warp == kDW + 2) {
    if (lane == 0) {
      // ---- activation loads: 3 bulk copies (one per part) per K step
      const int64_t arow = (int64_t)at * kAR;
      const uint8_t* isrc = a.img + (arow >> 7) * (3 * (int64_t)a.K * 256) + (arow & 127) * 128;
      for (int g = 0; g < nk && !abort_flag; ++g) {
        const int s = g % kS;
        if (g >= kS && !mbar_wait(st_empty + s, ((g / kS) - 1) & 1)) {
          abort_flag = 1;
          atomicOr(a.err, tc::kErrTimeout);
          break;
        }
        uint8_t* st = smem + (size_t)s * kBT;
        mbar_expect_tx(act_full + s, kBT);
#pragma unroll
        for (int h = 0; h < kG; ++h)
#pragma unroll
          for (int p = 0; p < 3; ++p)
            bulk_g2s(st + (h * 3 + p) * (kAR * 128),
                     isrc + (int64_t)p * a.K * 256 + (int64_t)((ks0 + g) * kG + h) * 16384, kAR * 128, act_full + s);
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
        const uint32_t b0 = smem_u32(smem + (size_t)s * kBT);
        const uint32_t a0 = taddr + kAcol + kAS * s;
#pragma unroll
        for (int kk = 0; kk < 4 * kG; ++kk)
          tc::umma_ts(taddr, a0 + 8 * kk, tc::sdesc(b0 + (kk >> 2) * (3 * kAR * 128) + (kk & 3) * 32), idesc,
                      (g | kk) != 0);
        tc::umma_commit(st_empty + s);  // frees the activation stage and the weight stage
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
    // the epilogue's row scales and per-activation state, fetched while the
    // first weight step is in flight (read after the cluster barriers below)
    if (tid < kWR) {
      int mi, r;
      weight_row(a.ms, kGlu, wt, tid, mi, r);
      // rows past the end of a partial GEPI_STORE tile have no scale
      srow[tid] = (EPI != GEPI_STORE || wt * kWR + tid < 2 * a.ms.n_pairs) ? __ldg(scale_ptr(a.ms, mi) + r) : 0.0f;
    } else if (tid < kWR + kAR) {
      const int al = tid - kWR, m = at * kAR + al;
      const EpiArgs& ep = a.ep;
      const bool in = m < a.n && (EPI == GEPI_QKV || EPI == GEPI_VOCAB);
      mflags[al] = in ? ep.flags[m] : SEQ_INVALID;
      mpos[al] = in && (EPI == GEPI_QKV || ep.step_logits) ? ep.pos[m] : 0;
      mseq[al] = in && EPI == GEPI_QKV && ep.seq ? ep.seq[m] : m;
      mgen[al] = in && EPI == GEPI_VOCAB && (ep.step_logits || ep.n_stop) ? ep.gen[m] : 0;
      mplen[al] = in && EPI == GEPI_VOCAB && ep.step_logits ? ep.plen[m] : 0;
    }
    // this thread's TMEM lane (row j), columns [16 kG half, 16 kG (half + 1)) of a stage:
    // K elements [32 kG half, 32 kG (half + 1)) of the step, bytes [24 kG half, +24 kG) of the row
    const uint32_t a_lane = taddr + ((uint32_t)((warp & 3) * 32) << 16) + kAcol + 16 * kG * half;
    for (int g = 0; g < nk; ++g) {
      const int p = g % kP, s = g % kS;
      bool got = !abort_flag && mbar_wait(pk_full + p, (g / kP) & 1);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform: the warp leaves together
      uint32_t w[6 * kG];
      {
        const uint2* pp = reinterpret_cast<const uint2*>(packed + (size_t)p * kPT + j * 48 * kG + half * 24 * kG);
#pragma unroll
        for (int i = 0; i < 3 * kG; ++i) {
          const uint2 v = pp[i];
          w[2 * i] = v.x;
          w[2 * i + 1] = v.y;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(pk_empty + p);  // the packed step is in registers
      // the MMAs of this stage's previous use have finished reading it
      got = g < kS || mbar_wait(st_empty + s, ((g / kS) - 1) & 1);
      if (!__all_sync(0xffffffffu, got)) break;
      tc::tc_fence_after();
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        uint32_t pk[16];  // two 16-column groups in expand_group's K order
#pragma unroll
        for (int uu = 0; uu < 2; ++uu) expand_group(w[6 * h + 3 * uu], w[6 * h + 3 * uu + 1], w[6 * h + 3 * uu + 2], pk + 8 * uu);
        tc::tmem_st16(a_lane + kAS * s + 16 * h, pk);
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full + s);
    }
  }

  // ---- partial tile -> the shared memory of the CTA that owns each activation
  // slice: CTA q receives, for activations [q SA, (q+1) SA), one [SA][128]
  // slot per rank (stage memory, free once this CTA's MMAs are done; a peer
  // writes into it only after its own K loop, and every CTA's MMAs finish
  // before the barrier).  A warp's 32 rows are 32 consecutive words.
  const int SA = kAR / C;
  float* recv = reinterpret_cast<float*>(smem);  // [C ranks][SA activations][128 rows]
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
    const int j = ((warp & 3) << 5) | lane;
    const int half = warp >> 2;
    const uint32_t lane_addr = taddr + ((uint32_t)((warp & 3) * 32) << 16);
    // parts summed in order (hi + mid) + lo, one part held at a time
    float d[32], e[32];
    tc::tmem_ld32(lane_addr + half * 32, d);
    tc::tmem_ld32(lane_addr + kAR + half * 32, e);
#pragma unroll
    for (int i = 0; i < 32; ++i) d[i] = __fadd_rn(d[i], e[i]);
    tc::tmem_ld32(lane_addr + 2 * kAR + half * 32, e);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int la = half * 32 + i;  // local activation
      const int q = la / SA;         // owner rank
      float* dst = C == 1 ? recv : cl.map_shared_rank(recv, q);
      dst[(c * SA + la - q * SA) * kWR + j] = __fadd_rn(d[i], e[i]);
    }
  }
  tc::tc_fence_before();
  cl.sync();  // every partial has landed in its owner

  // ---- epilogue of activations [c SA, (c+1) SA): thread t takes row pair
  // t % 64 ((2p, 2p+1), or (W1 row p, W3 row p) in GLU mode) of activations
  // t / 64, t / 64 + 4, ...; a warp works on one activation at a time and
  // its stores are contiguous.  The loop is kept rolled: straight-line code
  // run once per CTA is bound by instruction fetch.
  if (warp < kDW) {
    const EpiArgs& ep = a.ep;
    const int pp = tid & (kWR / 2 - 1), as = tid >> 6;
    const int r0 = kGlu ? pp : 2 * pp, r1 = kGlu ? pp + kWR / 2 : 2 * pp + 1;
    const float s0 = srow[r0], s1 = srow[r1];
    const int vrow = wt * kWR + 2 * pp;  // non-GLU: global row of the pair's first value
#pragma unroll 2
    for (int al = as; al < SA; al += kDW / 2) {
      float v0 = 0.f, v1 = 0.f;
      for (int q = 0; q < C; ++q) {  // rank order: one summation order everywhere
        const float* src = recv + (size_t)(q * SA + al) * kWR;
        const float p0 = src[r0], p1 = src[r1];
        v0 = q == 0 ? p0 : __fadd_rn(v0, p0);
        v1 = q == 0 ? p1 : __fadd_rn(v1, p1);
      }
      v0 = __fmul_rn(v0, s0);
      v1 = __fmul_rn(v1, s1);
      const int ml = c * SA + al, m = at * kAR + ml;
      if (EPI == GEPI_STORE) {
        // the plain linear: y[m, rows] as row pairs, 64 consecutive floats per warp
        if (m < a.n && vrow < 2 * a.ms.n_pairs)
          *reinterpret_cast<float2*>(ep.y + (int64_t)m * ep.ldy + vrow) = make_float2(v0, v1);
      } else if (EPI == GEPI_GLU) {
        if (m < a.n) ep.y[(int64_t)m * ep.ldy + wt * (kWR / 2) + pp] = swiglu(v0, v1);
      } else if (EPI == GEPI_RESID) {
        // the only writer of this element: one rounded add onto the residual
        if (m < a.n) atomicAdd(reinterpret_cast<float2*>(ep.y + (int64_t)m * ep.ldy + vrow), make_float2(v0, v1));
      } else if (EPI == GEPI_QKV) {
        // RoPE of torch_benchmark.py:84 (each product rounded before the add);
        // q to the query buffer, k and v to the cache row of the activation's sequence
        if (m < a.n && !(mflags[ml] & SEQ_INVALID)) {
          const int pos = mpos[ml];
          const int64_t crow = mseq[ml];
          float ra = v0, rb = v1;
          if (vrow < ep.q_rows + ep.kv_rows) {
            const int jr = (vrow % ep.hd) >> 1;
            const float cs = __ldg(ep.rope_cos + (int64_t)pos * (ep.hd >> 1) + jr);
            const float sn = __ldg(ep.rope_sin + (int64_t)pos * (ep.hd >> 1) + jr);
            ra = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
            rb = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
          }
          if (vrow < ep.q_rows) {
            *reinterpret_cast<float2*>(ep.qbuf + (int64_t)m * ep.ldq + vrow) = make_float2(ra, rb);
          } else {
            const bool kr = vrow < ep.q_rows + ep.kv_rows;
            const int64_t off = crow * ep.cache_stride + ep.layer_off + (int64_t)pos * ep.kv_rows +
                                (kr ? vrow - ep.q_rows : vrow - ep.q_rows - ep.kv_rows);
            store_kv2(kr ? ep.kc : ep.vc, off, ep.kv_half, ra, rb);
          }
        }
      } else {  // GEPI_VOCAB: logits, dumped step logits, stop masking, first-maximum key
        if (m < a.n) {  // warp-uniform: a warp holds one activation
          float va = v0, vb = v1;
          const int gen = mgen[ml];
          if (ep.y) *reinterpret_cast<float2*>(ep.y + (int64_t)m * ep.ldy + vrow) = make_float2(va, vb);
          if (ep.step_logits && !(mflags[ml] & (SEQ_DONE | SEQ_INVALID)) && mpos[ml] >= mplen[ml] - 1)
            *reinterpret_cast<float2*>(ep.step_logits + ((int64_t)m * ep.new_tokens + gen) * ep.vocab + vrow) =
                make_float2(va, vb);
          if (ep.n_stop && gen < ep.min_new) {
            for (int t = 0; t < ep.n_stop; ++t) {
              if (ep.stop_ids[t] == vrow) va = -INFINITY;
              if (ep.stop_ids[t] == vrow + 1) vb = -INFINITY;
            }
          }
          unsigned long long key = umax64(argmax_key(va, vrow), argmax_key(vb, vrow + 1));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, o));
          if (lane == 0) atomicMax(vkey + ml, key);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kDW + 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(taddr, kTmemCols);
  }
  // one global atomic per (tile, activation) instead of one per warp
  if (EPI == GEPI_VOCAB && tid < kAR && vkey[tid]) atomicMax(a.ep.keys + at * kAR + tid, vkey[tid]);
}

// Activation image (tc.cuh layout, K columns) of rows x[0..n): RMSNorm with
// weight g when g is given (torch_benchmark.py:22-24), else the rows as they
// are.  Inside every 16-column group the columns are stored in the order the
// weight expansion produces them (expand_group): image position p of a group
// holds column {0, 4, 8, 12, 3, 7, 11, 15, 2, 6, 10, 14, 1, 5, 9, 13}[p].  One CTA of 256 threads per row, each thread 16-column
// groups 16 (tid + 256 i) (K <= 8192: at most two per thread), all loaded
// before the reduction; rows beyond n are left as they are (never used).
constexpr int kImgThreads = 256;
constexpr int kImgGroups = 2;
constexpr int kImgMaxK = 16 * kImgThreads * kImgGroups;

// PERM = false writes the columns in natural order: the image tc.cuh's
// kernel reads (its weight expansion keeps the natural K order).
template <bool PERM = true>
__global__ void __launch_bounds__(kImgThreads) image_kernel(const float* __restrict__ x, int ldx, int n, int K,
                                                            const float* __restrict__ g, float eps,
                                                            uint8_t* __restrict__ img) {
  __shared__ float red[kImgThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  const float* xr = x + row * ldx;
  float v[kImgGroups][16], gw[kImgGroups][16];  // the norm weights load with x, before the reduction
#pragma unroll
  for (int c = 0; c < kImgGroups; ++c) {
    const int k0 = 16 * (tid + kImgThreads * c);
    if (k0 < K) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = *reinterpret_cast<const float4*>(xr + k0 + 4 * q);
        v[c][4 * q] = f.x; v[c][4 * q + 1] = f.y; v[c][4 * q + 2] = f.z; v[c][4 * q + 3] = f.w;
        const float4 w = g ? __ldg(reinterpret_cast<const float4*>(g + k0 + 4 * q)) : make_float4(0.f, 0.f, 0.f, 0.f);
        gw[c][4 * q] = w.x; gw[c][4 * q + 1] = w.y; gw[c][4 * q + 2] = w.z; gw[c][4 * q + 3] = w.w;
      }
    }
  }
  if (g) {
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < kImgGroups; ++c)
      if (16 * (tid + kImgThreads * c) < K)
#pragma unroll
        for (int i = 0; i < 16; ++i) ss = __fadd_rn(ss, __fmul_rn(v[c][i], v[c][i]));
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = lane < kImgThreads / 32 ? red[lane] : 0.0f;
    t = warp_sum(t);
    const float r = rms_scale(t, K, eps);
#pragma unroll
    for (int c = 0; c < kImgGroups; ++c) {
      const int k0 = 16 * (tid + kImgThreads * c);
      if (k0 < K)
#pragma unroll
        for (int i = 0; i < 16; ++i) v[c][i] = __fmul_rn(__fmul_rn(v[c][i], r), gw[c][i]);
    }
  }
#pragma unroll
  for (int c = 0; c < kImgGroups; ++c) {
    const int k0 = 16 * (tid + kImgThreads * c);
    if (k0 < K && PERM) {
      const float lo[8] = {v[c][0], v[c][4], v[c][8], v[c][12], v[c][3], v[c][7], v[c][11], v[c][15]};
      const float hi[8] = {v[c][2], v[c][6], v[c][10], v[c][14], v[c][1], v[c][5], v[c][9], v[c][13]};
      tc::img_store8(img, row, k0, K, lo);
      tc::img_store8(img, row, k0 + 8, K, hi);
    } else if (k0 < K) {
      const float lo[8] = {v[c][0], v[c][1], v[c][2], v[c][3], v[c][4], v[c][5], v[c][6], v[c][7]};
      const float hi[8] = {v[c][8], v[c][9], v[c][10], v[c][11], v[c][12], v[c][13], v[c][14], v[c][15]};
      tc::img_store8(img, row, k0, K, lo);
      tc::img_store8(img, row, k0 + 8, K, hi);
    }
  }
}

}  // namespace tcg
}  // namespace q6w
