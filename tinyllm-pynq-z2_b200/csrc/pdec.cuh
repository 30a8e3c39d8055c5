// Persistent B=1 decode step: one cooperative launch runs every layer and the
// vocab head of one model step for one sequence (CachedTransformer.step,
// benchmarks/torch_benchmark.py:96-125), for models whose widths suit the
// streaming GEMV (the 1.1B shape).
//
// Why.  At B=1 every weight byte is used once per token, so the step is an
// HBM stream, but as separate launches it is a chain of ~110 dependent kernels
// (five per layer) whose ramp-up and tail cost more than their bytes.  Here
// one CTA per SM stays resident for the whole step:
//  * a producer warp bulk-copies (cp.async.bulk, no multicast) the weight
//    tiles of every matrix of the step, in the order the consumers need them,
//    into a ring of 5 stages (~185 KB).  Weights do not depend on activations,
//    so it runs ahead across phase boundaries and HBM stays busy while the
//    consumers wait for a phase's input;
//  * twelve consumer warps walk the phases -- per layer QKV (RMSNorm prologue,
//    RoPE, K/V write), attention (one CTA per query head), wo + residual,
//    W1|W3 (RMSNorm prologue, SwiGLU), W2 + residual; then the vocab
//    (RMSNorm, logits, first-maximum argmax with stop masking) -- with a grid
//    barrier between dependent phases.
// Per tile the consumers do what stream_gemv_kernel does (stream.cuh): groups
// of WC = K/512 warps own the 16-value units of a row, each thread keeps its
// unit's normalised inputs in registers, decodes with one LOP3 per weight and
// reduces eight rows at once; the same summation orders, so the outputs equal
// the separate kernels'.  Activations written during the kernel are read
// through L2 (ld.global.cg), never the incoherent L1 / read-only paths.
//
// Every wait is bounded: a grid barrier gives up after kBarrierCycles, sets
// the timeout bit and a global abort word that every other waiter checks, so
// all CTAs leave promptly; the ring waits use mbar_wait (async.cuh).
#pragma once

#include "async.cuh"
#include "linear.cuh"
#include "stream.cuh"

namespace q6w {
namespace pdec {

constexpr int kCWarps = 12;                 // consumer warps
constexpr int kCT = 32 * kCWarps;           // consumer threads
constexpr int kThreads = kCT + 32;          // + the producer warp
constexpr int kStages = 5;
constexpr uint32_t kStage = 37376;          // >= the largest tile + its scales, 128-byte multiple
constexpr int kMaxLayers = 32;
constexpr int kMaxSeq = 4096;
constexpr uint64_t kBarrierCycles = 2000000000ull;  // ~1 s
constexpr int kErrTimeout = 4;
constexpr int kBarAll = 15;                 // named barrier over the consumer threads
constexpr int kBarAttn = 14;                // named barrier over the attention threads

struct QM {
  const uint8_t* q;
  const float* s;
};

struct Layer {
  QM wq, wk, wv, wo, w1, w2, w3;
  const float* attn_norm;
  const float* ffn_norm;
};

struct Args {
  int32_t dim, hidden, n_layers, n_heads, n_kv, hd, vocab, max_seq, kvr;
  float eps, denom;
  Layer layers[kMaxLayers];
  QM tok;
  const float* norm;
  const float* rope_cos;
  const float* rope_sin;
  float* x;    // residual stream [dim]
  float* qb;   // rotated q [dim]
  float* att;  // attention output [dim]
  float* hb;   // SwiGLU activations [hidden]
  float* kc;   // this sequence's caches (elements; FP16 when kv_half)
  float* vc;
  int32_t kv_half;
  const int32_t* pos;    // sequence state (row 0)
  const int32_t* flags;
  EpiArgs vep;           // vocab epilogue: keys, logits, dumped step logits, stop set, state
  uint32_t* sync;        // [0] arrivals, [1] abort; zero before the launch
  int32_t* err;
  stream::FieldConsts fc;
};

__host__ __device__ inline int n_phases(int n_layers) { return 5 * n_layers + 1; }

// A matrix phase: the weight set, K, and what its epilogue does.
enum { PH_QKV = 0, PH_ATTN = 1, PH_WO = 2, PH_W13 = 3, PH_W2 = 4, PH_VOCAB = 5 };

struct MPhase {
  MatSet ms;
  int kind;
  int K;
  const float* in;     // input vector
  const float* gnorm;  // RMSNorm weight or null
};

__host__ __device__ inline int phase_kind(const Args& a, int ph) { return ph == 5 * a.n_layers ? PH_VOCAB : ph % 5; }

__host__ __device__ inline MPhase matrix_phase(const Args& a, int ph) {
  MPhase m;
  m.kind = phase_kind(a, ph);
  const int l = ph / 5;
  MatSet ms = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, 0, 0, 0, 0};
  switch (m.kind) {
    case PH_QKV: {
      const Layer& L = a.layers[l];
      ms = {L.wq.q, L.wk.q, L.wv.q, L.wq.s, L.wk.s, L.wv.s, a.dim, a.dim + a.kvr, a.dim, 0, (a.dim + 2 * a.kvr) / 2};
      m.K = a.dim; m.in = a.x; m.gnorm = L.attn_norm;
      break;
    }
    case PH_WO: {
      const Layer& L = a.layers[l];
      ms = {L.wo.q, nullptr, nullptr, L.wo.s, nullptr, nullptr, a.dim, a.dim, a.dim, 0, a.dim / 2};
      m.K = a.dim; m.in = a.att; m.gnorm = nullptr;
      break;
    }
    case PH_W13: {
      const Layer& L = a.layers[l];
      ms = {L.w1.q, L.w3.q, nullptr, L.w1.s, L.w3.s, nullptr, a.hidden, a.hidden, a.dim, 1, a.hidden};
      m.K = a.dim; m.in = a.x; m.gnorm = L.ffn_norm;
      break;
    }
    case PH_W2: {
      const Layer& L = a.layers[l];
      ms = {L.w2.q, nullptr, nullptr, L.w2.s, nullptr, nullptr, a.dim, a.dim, a.hidden, 0, a.dim / 2};
      m.K = a.hidden; m.in = a.hb; m.gnorm = nullptr;
      break;
    }
    case PH_VOCAB:
      ms = {a.tok.q, nullptr, nullptr, a.tok.s, nullptr, nullptr, a.vocab, a.vocab, a.dim, 0, a.vocab / 2};
      m.K = a.dim; m.in = a.x; m.gnorm = a.norm;
      break;
    default:
      m.K = 0; m.in = nullptr; m.gnorm = nullptr;
  }
  m.ms = ms;
  return m;
}

// Tile geometry of a phase: G row groups of WC warps; non-GLU tiles are 8 G
// consecutive rows of the concatenated matrices, GLU tiles 4 G pairs.
__host__ __device__ inline int groups_of(int K) { return kCWarps / (K / 512); }
__host__ __device__ inline int tile_pairs(int K) { return 4 * groups_of(K); }
__host__ __device__ inline int n_tiles(const MPhase& m) {
  const int tp = tile_pairs(m.K);
  return (m.ms.n_pairs + tp - 1) / tp;
}

using stream::named_sync;

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---- producer: the copies of tile t of phase m into `dst` (returns the bytes)
__device__ __forceinline__ uint32_t load_tile(const MPhase& m, int t, uint8_t* dst, uint64_t* bar) {
  const uint32_t rb = (uint32_t)m.K * 3 / 4;
  const int tp = tile_pairs(m.K);
  const int p0 = t * tp;
  const int np = min(tp, m.ms.n_pairs - p0);
  if (m.ms.glu) {
    float* dsc = reinterpret_cast<float*>(dst + (size_t)2 * tp * rb);
    const uint32_t bytes = 2u * np * (rb + 4);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(dst, m.ms.q0 + (size_t)p0 * rb, np * rb, bar);
    bulk_g2s(dst + (size_t)tp * rb, m.ms.q1 + (size_t)p0 * rb, np * rb, bar);
    bulk_g2s(dsc, m.ms.s0 + p0, 4 * np, bar);
    bulk_g2s(dsc + tp, m.ms.s1 + p0, 4 * np, bar);
    return bytes;
  }
  // rows [r0, r1) of the concatenation m0 | m1 | m2, split where a matrix ends
  const int rows = 2 * tp, r0 = 2 * p0, r1 = r0 + 2 * np;
  float* dsc = reinterpret_cast<float*>(dst + (size_t)rows * rb);
  const uint32_t bytes = (uint32_t)(r1 - r0) * (rb + 4);
  mbar_expect_tx(bar, bytes);
  const int lo[3] = {0, m.ms.end0, m.ms.end1}, hi[3] = {m.ms.end0, m.ms.end1, 2 * m.ms.n_pairs};
  const uint8_t* qs[3] = {m.ms.q0, m.ms.q1, m.ms.q2};
  const float* ss[3] = {m.ms.s0, m.ms.s1, m.ms.s2};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int b0 = max(r0, lo[k]), b1 = min(r1, hi[k]);
    if (b1 <= b0) continue;
    bulk_g2s(dst + (size_t)(b0 - r0) * rb, qs[k] + (size_t)(b0 - lo[k]) * rb, (uint32_t)(b1 - b0) * rb, bar);
    bulk_g2s(dsc + (b0 - r0), ss[k] + (b0 - lo[k]), 4u * (b1 - b0), bar);
  }
  return bytes;
}

// ---- grid barrier over the consumer threads of every CTA (the producers never
// take part).  Returns false when the step is aborted.
__device__ __forceinline__ bool grid_barrier(const Args& a, uint32_t target, int* s_abort) {
  named_sync(kBarAll, kCT);
  if (threadIdx.x == 0) {
    if (*(volatile int*)s_abort) atomicExch(a.sync + 1, 1u);  // a local failure stops every CTA
    __threadfence();
    atomicAdd(a.sync, 1u);
    const uint64_t t0 = clock64();
    while (ld_acquire(a.sync) < target) {
      if (*(volatile uint32_t*)(a.sync + 1)) {
        *s_abort = 1;
        break;
      }
      if (clock64() - t0 > kBarrierCycles) {
        atomicOr(a.err, kErrTimeout);
        atomicExch(a.sync + 1, 1u);
        *s_abort = 1;
        break;
      }
      __nanosleep(32);
    }
  }
  named_sync(kBarAll, kCT);
  return !*(volatile int*)s_abort;
}

// ---- attention of query head h over positions 0..T-1 (threads 0..255), the
// arithmetic and orders of attn_head_kernel (model.cu), inputs through L2.
template <int HD, typename KT>
__device__ void attention_head(const Args& a, int h, const KT* kc, const KT* vc, float* sm) {
  constexpr int CQ = HD / 4, G = 256 / CQ;
  float* sq = sm;
  float* red = sq + HD;
  float4* part = reinterpret_cast<float4*>(red + 16);
  float* sp = reinterpret_cast<float*>(part + G * CQ);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = a.pos[0];
  int T = pos + 1;
  T = T > a.max_seq ? a.max_seq : T;
  float* o = a.att + h * HD;
  if ((a.flags[0] & SEQ_INVALID) || T <= 0) {
    if (tid < HD) __stcg(o + tid, 0.0f);
    return;
  }
  const int g = h / (a.n_heads / a.n_kv);
  const KT* kb = kc + g * HD;
  const KT* vb = vc + g * HD;
  if (tid < HD) sq[tid] = __ldcg(a.qb + h * HD + tid);
  named_sync(kBarAttn, 256);
  float mx = -INFINITY;
  for (int t = tid; t < T; t += 256) {
    const KT* kr = kb + (int64_t)t * a.kvr;
    float d = 0.0f;
#pragma unroll
    for (int j = 0; j < CQ; ++j) {
      float4 k4;
      if (sizeof(KT) == 4) {
        k4 = __ldcg(reinterpret_cast<const float4*>(kr) + j);
      } else {
        const uint2 u = __ldcg(reinterpret_cast<const uint2*>(kr) + j);
        const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        k4 = make_float4(p0.x, p0.y, p1.x, p1.y);
      }
      d = fmaf(sq[4 * j], k4.x, d);
      d = fmaf(sq[4 * j + 1], k4.y, d);
      d = fmaf(sq[4 * j + 2], k4.z, d);
      d = fmaf(sq[4 * j + 3], k4.w, d);
    }
    d = __fdiv_rn(d, a.denom);
    sp[t] = d;
    mx = fmaxf(mx, d);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  named_sync(kBarAttn, 256);
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  float sum = 0.0f;
  for (int t = tid; t < T; t += 256) {
    const float e = expf(sp[t] - mx);
    sp[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[8 + warp] = sum;
  named_sync(kBarAttn, 256);
  sum = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[8 + w];
  const int cq = tid % CQ, grp = tid / CQ;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = grp; t < T; t += G) {
    const float wt = __fdiv_rn(sp[t], sum);
    const KT* vr = vb + (int64_t)t * a.kvr + 4 * cq;
    float4 v4;
    if (sizeof(KT) == 4) {
      v4 = __ldcg(reinterpret_cast<const float4*>(vr));
    } else {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(vr));
      const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v4 = make_float4(p0.x, p0.y, p1.x, p1.y);
    }
    acc.x = fmaf(wt, v4.x, acc.x);
    acc.y = fmaf(wt, v4.y, acc.y);
    acc.z = fmaf(wt, v4.z, acc.z);
    acc.w = fmaf(wt, v4.w, acc.w);
  }
  part[grp * CQ + cq] = acc;
  named_sync(kBarAttn, 256);
  if (tid < CQ) {
    float4 r = part[tid];
    for (int k = 1; k < G; ++k) {
      const float4 p = part[k * CQ + tid];
      r.x += p.x; r.y += p.y; r.z += p.z; r.w += p.w;
    }
    __stcg(reinterpret_cast<float4*>(o) + tid, r);
  }
}

// QKV output pair p of the layer whose caches start at kc / vc: RoPE on q and
// k with each product rounded before the add (torch_benchmark.py:79-85), q to
// the query buffer, k and v to the cache row of this position -- the
// arithmetic of epilogue<EPI_QKV>.
__device__ __forceinline__ void qkv_store(const Args& a, float* kc, float* vc, int p, float va, float vb) {
  if (a.flags[0] & SEQ_INVALID) return;
  const int v = 2 * p, pos = a.pos[0];
  float ra = va, rb = vb;
  if (v < a.dim + a.kvr) {
    const int j = (v % a.hd) >> 1;
    const float c = __ldg(a.rope_cos + (int64_t)pos * (a.hd >> 1) + j);
    const float s = __ldg(a.rope_sin + (int64_t)pos * (a.hd >> 1) + j);
    ra = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
    rb = __fadd_rn(__fmul_rn(va, s), __fmul_rn(vb, c));
  }
  if (v < a.dim)
    __stcg(reinterpret_cast<float2*>(a.qb + v), make_float2(ra, rb));
  else if (v < a.dim + a.kvr)
    store_kv2(kc, (int64_t)pos * a.kvr + (v - a.dim), a.kv_half, ra, rb);
  else
    store_kv2(vc, (int64_t)pos * a.kvr + (v - a.dim - a.kvr), a.kv_half, ra, rb);
}

// ---- consumers: the tiles of one matrix phase owned by this CTA (kc / vc:
// the current layer's caches, for the QKV phase).
template <int WC>
__device__ void run_matrix(const Args& a, const MPhase& m, float* kc, float* vc, int& ring, uint8_t* stages,
                           uint64_t* full, uint64_t* empty, float* part, float* sums, int* s_abort,
                           unsigned long long& best) {
  constexpr int G = kCWarps / WC, TP = 4 * G, K = 512 * WC;
  constexpr uint32_t kRb = 384u * WC;
  constexpr int kR = stream::kR;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = warp / WC, wc = warp % WC;
  const bool active = g < G;
  const int u = 32 * wc + lane;
  const bool glu = m.ms.glu != 0;
  float2 xs[8];
  if (active) {
    float xv[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = ldcg4(m.in + 16 * u + 4 * j);
      xv[4 * j] = v.x; xv[4 * j + 1] = v.y; xv[4 * j + 2] = v.z; xv[4 * j + 3] = v.w;
    }
    if (m.gnorm) {
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = __fadd_rn(ss, __fmul_rn(xv[i], xv[i]));
      ss = warp_sum(ss);
      if (lane == 0) sums[g * WC + wc] = ss;
      stream::named_sync(1 + g, 32 * WC);
      float t = 0.0f;
      for (int w = 0; w < WC; ++w) t = __fadd_rn(t, sums[g * WC + w]);
      const float r = rms_scale(t, K, a.eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) xv[i] = __fmul_rn(__fmul_rn(xv[i], r), __ldg(m.gnorm + 16 * u + i));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      xs[i] = make_float2(xv[2 * i] * (1.0f / (float)(1 << stream::field_pos(2 * i))),
                          xv[2 * i + 1] * (1.0f / (float)(1 << stream::field_pos(2 * i + 1))));
  }
  const int tiles = n_tiles(m);
  for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++ring) {
    const int s = ring % kStages;
    bool ok = !*(volatile int*)s_abort;
    if (ok && !mbar_wait(full + s, (ring / kStages) & 1)) {
      *s_abort = 1;
      atomicOr(a.err, kErrTimeout);
      ok = false;
    }
    const uint8_t* st = stages + (size_t)s * kStage;
    const float* ssc = reinterpret_cast<const float*>(st + (size_t)2 * TP * kRb);
    float v[kR];
    const int my_r = lane >> 2;
    const int my_pr = g * (kR / 2) + (my_r >> 1);
    float sc = 0.0f;
    if (active) {
      float2 acc[kR];
#pragma unroll
      for (int r = 0; r < kR; ++r) acc[r] = make_float2(0.0f, 0.0f);
      if (ok) {
        const uint8_t* su = st + 12 * u;
#pragma unroll
        for (int r = 0; r < kR; ++r) {
          const int pr = g * (kR / 2) + (r >> 1);
          const int row = glu ? ((r & 1) * TP + pr) : 2 * pr + (r & 1);
          const uint32_t* w = reinterpret_cast<const uint32_t*>(su + row * kRb);
          stream::unit_fma(w[0], w[1], w[2], xs, acc[r], a.fc);
        }
        sc = ssc[glu ? ((my_r & 1) * TP + my_pr) : 2 * my_pr + (my_r & 1)];
      }
#pragma unroll
      for (int r = 0; r < kR; ++r) v[r] = acc[r].x + acc[r].y;
    }
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(empty + s);  // every consumer warp releases the stage
    if (!active) continue;
    const float tot = stream::reduce8(v, lane);
    float* pb = part + ((ring & 1) * G + g) * WC * kR;
    if ((lane & 3) == 0) pb[wc * kR + my_r] = tot * sc;
    stream::named_sync(1 + g, 32 * WC);
    if (wc == 0 && lane < kR / 2 && ok) {
      float va = 0.0f, vb = 0.0f;
      for (int w = 0; w < WC; ++w) {
        va = __fadd_rn(va, pb[w * kR + 2 * lane]);
        vb = __fadd_rn(vb, pb[w * kR + 2 * lane + 1]);
      }
      const int p = t * TP + g * (kR / 2) + lane;
      if (p < m.ms.n_pairs) {
        switch (m.kind) {
          case PH_QKV: qkv_store(a, kc, vc, p, va, vb); break;
          case PH_WO:
          case PH_W2: {
            float* y = a.x + 2 * p;
            const float2 old = __ldcg(reinterpret_cast<const float2*>(y));
            __stcg(reinterpret_cast<float2*>(y), make_float2(__fadd_rn(old.x, va), __fadd_rn(old.y, vb)));
            break;
          }
          case PH_W13: __stcg(a.hb + p, swiglu(va, vb)); break;
          default: best = umax64(best, epilogue<EPI_VOCAB>(a.vep, 0, p, va, vb)); break;
        }
      }
    }
  }
}

// 128 registers: the register file is four 16K sub-partitions, one per warp
// scheduler, so thirteen warps fit only at <= 4096 registers a warp.
__global__ void __maxnreg__(128) pdec_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + kStages;
  int* s_abort = reinterpret_cast<int*>(sm + 96);
  uint8_t* stages = sm + 128;
  float* part = reinterpret_cast<float*>(stages + (size_t)kStages * kStage);  // [2][G][WC][8] <= 2 * 96
  float* sums = part + 2 * kCWarps * stream::kR;                             // [12]
  float* attn = sums + 16;                                                   // attention scratch
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nph = n_phases(a.n_layers);
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kCWarps);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kCWarps) {
    // ---- producer: every weight tile of the step, in consumption order
    if (lane == 0) {
      int i = 0;
      for (int ph = 0; ph < nph && !*(volatile int*)s_abort; ++ph) {
        if (phase_kind(a, ph) == PH_ATTN) continue;
        const MPhase m = matrix_phase(a, ph);
        const int tiles = n_tiles(m);
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
          const int s = i % kStages;
          if (*(volatile int*)s_abort) break;
          if (i >= kStages && !mbar_wait(empty + s, ((i / kStages) - 1) & 1)) {
            *s_abort = 1;
            atomicOr(a.err, kErrTimeout);
            break;
          }
          load_tile(m, t, stages + (size_t)s * kStage, full + s);
        }
      }
    }
    return;
  }

  // ---- consumers
  int ring = 0;
  uint32_t target = 0;
  unsigned long long best = 0ull;
  for (int ph = 0; ph < nph; ++ph) {
    const int kind = phase_kind(a, ph);
    if (ph > 0) {
      target += gridDim.x;
      if (!grid_barrier(a, target, s_abort)) break;
    }
    // this layer's caches (element offsets; FP16 elements when kv_half)
    const int64_t off = (int64_t)(ph / 5) * a.max_seq * a.kvr;
    float* kcl = a.kv_half ? reinterpret_cast<float*>(reinterpret_cast<__half*>(a.kc) + off) : a.kc + off;
    float* vcl = a.kv_half ? reinterpret_cast<float*>(reinterpret_cast<__half*>(a.vc) + off) : a.vc + off;
    if (kind == PH_ATTN) {
      if (blockIdx.x < a.n_heads && tid < 256) {
        const __half* kh = reinterpret_cast<const __half*>(kcl);
        const __half* vh = reinterpret_cast<const __half*>(vcl);
        if (a.hd == 64) {
          if (a.kv_half) attention_head<64, __half>(a, blockIdx.x, kh, vh, attn);
          else attention_head<64, float>(a, blockIdx.x, kcl, vcl, attn);
        } else {
          if (a.kv_half) attention_head<128, __half>(a, blockIdx.x, kh, vh, attn);
          else attention_head<128, float>(a, blockIdx.x, kcl, vcl, attn);
        }
      }
      continue;
    }
    const MPhase m = matrix_phase(a, ph);
    switch (m.K / 512) {
      case 1: run_matrix<1>(a, m, kcl, vcl, ring, stages, full, empty, part, sums, s_abort, best); break;
      case 2: run_matrix<2>(a, m, kcl, vcl, ring, stages, full, empty, part, sums, s_abort, best); break;
      case 4: run_matrix<4>(a, m, kcl, vcl, ring, stages, full, empty, part, sums, s_abort, best); break;
      case 8: run_matrix<8>(a, m, kcl, vcl, ring, stages, full, empty, part, sums, s_abort, best); break;
      default: run_matrix<11>(a, m, kcl, vcl, ring, stages, full, empty, part, sums, s_abort, best); break;
    }
  }
  // vocab: one first-maximum key per warp-group leader lane, combined into the sequence's key
  if (best) atomicMax(a.vep.keys, best);
}

// Shared memory of a launch for max_seq positions.
__host__ __device__ inline size_t smem_bytes(int hd, int max_seq) {
  const int cq = hd / 4;
  return 128 + (size_t)kStages * kStage + 4 * (2 * kCWarps * stream::kR + 16) + 4 * (size_t)(hd + 16) +
         16 * (size_t)256 + 4 * (size_t)max_seq + 16 * (size_t)cq;
}

}  // namespace pdec
}  // namespace q6w
