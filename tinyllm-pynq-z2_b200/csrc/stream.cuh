// HBM-streaming Q6W GEMV for one activation row (B=1 decode of large models).
//
// At B=1 every weight byte is used once, so the kernel is a stream: weight
// tiles go HBM -> shared memory by bulk copies (cp.async.bulk, no multicast)
// issued by one producer warp into a ring of stages, and consumer warps
// decode them against a register-resident input slice.
//
// Work split.  A tile is TP row pairs (2 TP consecutive rows, or TP rows of
// W1 and the same TP rows of W3 in GLU mode) over the full row.  Consumer
// warps form WR row groups of WC warps; within a group, thread (warp wc,
// lane) owns 16-value unit u = 32 wc + lane of every row (U = K / 16 units,
// so WC = U / 32) and each group takes R = 8 rows of the tile.  A thread
// keeps its unit's 16 normalised inputs in registers for the whole launch.
//
// Decode (per 16-value unit, 3 words w0 w1 w2, values low-bit-first): field f
// at bit p of a source word becomes the float 1.5 * 2^23 + ((f ^ 32) << p) by
// one LOP3 ((w & (63 << p)) ^ (0x4B400000 | 32 << p)); subtracting the
// constant 1.5 * 2^23 + (32 << p) leaves exactly v * 2^p (v the signed code).
// The input of that column is pre-scaled by 2^-p (exact), so the FMA adds the
// same v * x.  Sources: w0 (fields 0-2 at p 0, 6, 12), funnel(w0, w1) >> 18
// (3-5), w1 (6-8 at p 4, 10, 16), funnel(w1, w2) >> 22 (9-11), w2 (12, 13 at
// p 8, 14), w2 >> 20 (14, 15): 3 shifts + 16 LOP3 + 8 FADD2 + 8 FFMA2 per 16
// weights.  The row scale multiplies the finished dot product
// (s * sum(v x) instead of sum((v s) x): equal up to FP32 rounding).
//
// Overlap across launches: the kernel allows its dependent launch at once and
// issues its first weight tiles before waiting on the previous grid
// (programmatic dependent launch); inputs and outputs are touched only after
// that wait.
#pragma once

#include "async.cuh"
#include "linear.cuh"

namespace q6w {
namespace stream {

constexpr int kR = 8;          // rows per row group per tile
constexpr int kStages = 2;  // per CTA; two CTAs per SM keep four tiles in flight

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Bit position of field i (0..15) of a unit in its decode source word.
__host__ __device__ constexpr int field_pos(int i) {
  return i < 3 ? 6 * i
         : i < 6 ? 6 * (i - 3)
         : i < 9 ? 4 + 6 * (i - 6)
         : i < 12 ? 6 * (i - 9)
         : i < 14 ? 8 + 6 * (i - 12)
                  : 6 * (i - 14);
}

// XOR constants 0x4B400000 | 32 << p, one per bit position p, handed to the
// kernel as parameters: opaque to the compiler, so each field costs one LOP3
// with the mask as its immediate (two folded immediates cost two ops).
struct FieldConsts {
  uint32_t x[17];
};

inline FieldConsts field_consts() {
  FieldConsts c;
  for (int p = 0; p < 17; ++p) c.x[p] = 0x4B400000u | (0x20u << p);
  return c;
}

__device__ __forceinline__ float fld(uint32_t src, int p, const FieldConsts& c) {
  return __uint_as_float((src & (0x3Fu << p)) ^ c.x[p]);
}

// acc += sum_i v_i * x_i over one unit; xs[i] = x_i * 2^-field_pos(i).
__device__ __forceinline__ void unit_fma(uint32_t w0, uint32_t w1, uint32_t w2, const float2 (&xs)[8], float2& acc,
                                         const FieldConsts& c) {
  const uint32_t s1 = __funnelshift_r(w0, w1, 18), s2 = __funnelshift_r(w1, w2, 22), s3 = w2 >> 20;
  const float f[16] = {fld(w0, 0, c), fld(w0, 6, c), fld(w0, 12, c), fld(s1, 0, c), fld(s1, 6, c), fld(s1, 12, c),
                       fld(w1, 4, c), fld(w1, 10, c), fld(w1, 16, c), fld(s2, 0, c), fld(s2, 6, c), fld(s2, 12, c),
                       fld(w2, 8, c), fld(w2, 14, c), fld(s3, 0, c), fld(s3, 6, c)};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 bias = make_float2(-(12582912.0f + (float)(32 << field_pos(2 * i))),
                                    -(12582912.0f + (float)(32 << field_pos(2 * i + 1))));
    const float2 v = __fadd2_rn(make_float2(f[2 * i], f[2 * i + 1]), bias);
    acc = __ffma2_rn(v, xs[i], acc);
  }
}

// Sums of 8 per-lane values over the warp: afterwards lane l holds the total
// of value l >> 2 (lanes with l % 4 == 0 hold the 8 distinct totals).
// Exchanges halve the values carried at each step: 4 + 2 + 1 + 1 + 1 shuffles.
__device__ __forceinline__ float reduce8(const float (&v)[8], int lane) {
  float w[4], z[2];
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = b4 ? v[4 + i] : v[i], send = b4 ? v[i] : v[4 + i];
    w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b3 ? w[2 + i] : w[i], send = b3 ? w[i] : w[2 + i];
    z[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float keep = b2 ? z[1] : z[0], send = b2 ? z[0] : z[1];
  float t = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return t;
}

// Compile-time layout for K = 512 WC: WR row groups of WC warps, tiles of
// 8 WR rows (4 WR pairs), a ring of 2 stages of about 25-34 KB.
template <int WC>
struct Shape {
  static constexpr int kWc = WC;
  static constexpr int kWr = WC >= 8 ? 1 : (8 / WC > 4 ? 4 : 8 / WC);
  static constexpr int kTp = kR * kWr / 2;
  static constexpr int kRows = 2 * kTp;
  static constexpr uint32_t kRbytes = 384u * WC;  // K * 3 / 4
  static constexpr uint32_t kStage = kRows * kRbytes + 8u * kTp;
  static constexpr int kNst = kStages;
  static constexpr size_t kSmem = 128 + (size_t)kNst * kStage + 4 * (2 * kR + 1) * (size_t)(kWr * WC);
  static constexpr int kThreads = 32 * (WC * kWr + 1);
};

// Per-launch values: tile count and the field constants.
struct Geometry {
  int wc;      // K / 512: selects the Shape instantiation
  int tiles;   // tiles of the matrix set
  size_t smem;
  int threads;
  FieldConsts fc;
};

template <int WC>
inline bool fill_geometry(const MatSet& ms, Geometry& g) {
  using S = Shape<WC>;
  if (ms.glu) {
    if (ms.n_pairs % S::kTp) return false;
  } else {
    const int total = 2 * ms.n_pairs;
    if (total % S::kRows || ms.end0 % S::kRows || ms.end1 % S::kRows) return false;
  }
  g.wc = WC;
  g.tiles = ms.n_pairs / S::kTp;
  g.smem = S::kSmem;
  g.threads = S::kThreads;
  g.fc = field_consts();
  return true;
}

// Shapes the stream kernel takes: K = 512 WC for WC in {1, 2, 4, 8, 11}
// (K 512, 1024, 2048, 4096, 5632), matrices whose row counts are multiples of
// the tile's rows.
inline bool geometry(const MatSet& ms, Geometry& g) {
  switch (ms.cols) {
    case 512: return fill_geometry<1>(ms, g);
    case 1024: return fill_geometry<2>(ms, g);
    case 2048: return fill_geometry<4>(ms, g);
    case 4096: return fill_geometry<8>(ms, g);
    case 5632: return fill_geometry<11>(ms, g);
    default: return false;
  }
}

// MINB: CTAs per SM the register allocation leaves room for (3 for matrices
// with at least three tiles per SM and no RMSNorm prologue: more warps hide
// the shared-memory latency of the decode; 1 otherwise, where the grid has at
// most two CTAs per SM).
template <bool RMS, int EPI, int WC, int MINB = 1>
__global__ void __launch_bounds__(Shape<WC>::kThreads, MINB)
    stream_gemv_kernel(const float* __restrict__ x, const float* __restrict__ gnorm, float eps, MatSet ms,
                       EpiArgs ep, Geometry geo, int32_t* err) {
  using S = Shape<WC>;
  constexpr bool kGlu = EPI == EPI_GLU;
  constexpr int kWr = S::kWr, kTp = S::kTp, rows = S::kRows, nst = S::kNst;
  constexpr uint32_t kRb = S::kRbytes, kSt = S::kStage;
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + 64);
  uint8_t* stages = sm + 128;
  float* part = reinterpret_cast<float*>(stages + (size_t)nst * kSt);  // [2][wr][wc][kR]
  float* sums = part + 2 * kR * kWr * WC;                                // [wr][wc]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nwc = WC * kWr;  // consumer warps; warp nwc is the producer

  pdl_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, nwc);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == nwc) {
    // ---- producer: one lane issues every copy (weights only: safe before the grid wait)
    if (lane == 0) {
      int i = 0;
      for (int t = blockIdx.x; t < geo.tiles; t += gridDim.x, ++i) {
        const int s = i % nst;
        if (*abort_flag) break;
        if (i >= nst && !mbar_wait(empty + s, ((i / nst) - 1) & 1)) {
          *abort_flag = 1;  // consumers stop waiting; a wait already running fails once
          if (err) atomicOr(err, 4);
          break;
        }
        uint8_t* dst = stages + (size_t)s * kSt;
        float* dsc = reinterpret_cast<float*>(dst + (size_t)rows * kRb);
        mbar_expect_tx(full + s, kSt);
        if (kGlu) {
          const int p0 = t * kTp;
          bulk_g2s(dst, ms.q0 + (size_t)p0 * kRb, kTp * kRb, full + s);
          bulk_g2s(dst + (size_t)kTp * kRb, ms.q1 + (size_t)p0 * kRb, kTp * kRb, full + s);
          bulk_g2s(dsc, ms.s0 + p0, 4 * kTp, full + s);
          bulk_g2s(dsc + kTp, ms.s1 + p0, 4 * kTp, full + s);
        } else {
          // rows [r0, r0 + rows) of the concatenation; tiles never straddle a matrix
          const int r0 = t * rows;
          const uint8_t* q;
          const float* sc;
          int r;
          if (r0 < ms.end0) {
            q = ms.q0; sc = ms.s0; r = r0;
          } else if (r0 < ms.end1) {
            q = ms.q1; sc = ms.s1; r = r0 - ms.end0;
          } else {
            q = ms.q2; sc = ms.s2; r = r0 - ms.end1;
          }
          bulk_g2s(dst, q + (size_t)r * kRb, rows * kRb, full + s);
          bulk_g2s(dsc, sc + r, 4 * rows, full + s);
        }
      }
    }
    return;
  }

  // ---- consumers
  const int g = warp / WC, wc = warp % WC;
  const int u = 32 * wc + lane;  // this thread's unit of every row
  constexpr int K = 512 * WC;
  pdl_wait();  // the previous grid's outputs (x) are complete from here on

  // normalised inputs of this unit, pre-scaled by 2^-field_pos
  float xv[16];
  {
    const float4* xp = reinterpret_cast<const float4*>(x + 16 * u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = __ldg(xp + j);
      xv[4 * j] = v.x; xv[4 * j + 1] = v.y; xv[4 * j + 2] = v.z; xv[4 * j + 3] = v.w;
    }
    if (RMS) {
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = __fadd_rn(ss, __fmul_rn(xv[i], xv[i]));
      ss = warp_sum(ss);
      // every row group covers all units once: reduce within group g
      if (lane == 0) sums[g * WC + wc] = ss;
      named_sync(1 + g, 32 * WC);
      float t = 0.0f;
      for (int w = 0; w < WC; ++w) t = __fadd_rn(t, sums[g * WC + w]);
      const float r = rms_scale(t, K, eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) xv[i] = __fmul_rn(__fmul_rn(xv[i], r), __ldg(gnorm + 16 * u + i));
    }
  }
  float2 xs[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    xs[i] = make_float2(xv[2 * i] * (1.0f / (float)(1 << field_pos(2 * i))),
                        xv[2 * i + 1] * (1.0f / (float)(1 << field_pos(2 * i + 1))));

  unsigned long long best = 0ull;
  int i = 0;
  for (int t = blockIdx.x; t < geo.tiles; t += gridDim.x, ++i) {
    const int s = i % nst;
    // after a failed wait the group keeps its barrier count but skips the work
    bool ok = !*abort_flag;
    if (ok && !mbar_wait(full + s, (i / nst) & 1)) {
      *abort_flag = 1;
      if (err) atomicOr(err, 4);
      ok = false;
    }
    const uint8_t* st = stages + (size_t)s * kSt;
    const float* ssc = reinterpret_cast<const float*>(st + (size_t)rows * kRb);
    const uint8_t* su = st + 12 * u;
    // local row r of group g: pair pr = g * kR/2 + r/2; GLU tiles hold W1 rows
    // then W3 rows, so the pair is (W1 row, W3 row); otherwise rows 2pr, 2pr+1
    float2 acc[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) acc[r] = make_float2(0.0f, 0.0f);
    // this lane's row after the reduction (lanes l % 4 == 0 write it)
    const int my_r = lane >> 2;
    const int my_pr = g * (kR / 2) + (my_r >> 1);
    float sc = 0.0f;
    if (ok) {
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        const int pr = g * (kR / 2) + (r >> 1);
        const int row = kGlu ? ((r & 1) * kTp + pr) : 2 * pr + (r & 1);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(su + row * kRb);
        unit_fma(w[0], w[1], w[2], xs, acc[r], geo.fc);
      }
      sc = ssc[kGlu ? ((my_r & 1) * kTp + my_pr) : 2 * my_pr + (my_r & 1)];
    }
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(empty + s);  // this warp is done with the stage
    float v[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) v[r] = acc[r].x + acc[r].y;
    const float tot = reduce8(v, lane);
    float* pb = part + ((i & 1) * kWr + g) * WC * kR;
    if ((lane & 3) == 0) pb[wc * kR + my_r] = tot * sc;
    named_sync(1 + g, 32 * WC);
    if (wc == 0 && lane < kR / 2) {
      float a = 0.0f, b = 0.0f;
      for (int w = 0; w < WC; ++w) {
        a = __fadd_rn(a, pb[w * kR + 2 * lane]);
        b = __fadd_rn(b, pb[w * kR + 2 * lane + 1]);
      }
      const int p = t * kTp + g * (kR / 2) + lane;
      if (ok) best = umax64(best, epilogue<EPI>(ep, 0, p, a, b));
    }
  }
  if (EPI == EPI_VOCAB && wc == 0) {
#pragma unroll
    for (int o = 2; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0 && best) atomicMax(ep.keys, best);
  }
}

}  // namespace stream
}  // namespace q6w
