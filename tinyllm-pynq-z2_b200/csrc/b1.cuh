// B=1 greedy request as one persistent kernel per launch: an 8-CTA thread-block
// cluster keeps every weight matrix resident in shared memory (each CTA its
// 1/8 share) and runs whole model steps -- embedding, the layers, vocab
// projection, argmax and the greedy stop contract -- with no host involvement,
// like the reference's autonomous FPGA top (rtl/autonomous/tinyllm_autonomous.cpp:955-1153).
//
// Work split (CTA c of 8):
//   attention half of a layer -- CTA c owns query head c: the q rows of head c
//     and the k, v rows of its kv head (so q, k, v of the current position are
//     computed locally, the first CTA of each kv group writes k, v to the
//     cache), attention of head c, and the head-c column block of wo, which
//     gives a partial of wo @ att over head c's columns;
//   FFN half -- CTA c owns a slice of hidden units: its W1 and W3 rows (so the
//     SwiGLU slice is local) and the matching column block of W2, which gives
//     a partial of W2 @ h over its hidden units;
//   vocab -- a slice of the (tied) embedding rows; the same slice serves the
//     embedding lookup of later steps through distributed shared memory.
// Exchange: each half's partial vector is pushed into every CTA's slot for
// this CTA through distributed shared memory, then one cluster barrier
// (release/acquire) publishes it and every CTA adds the slots in the same
// fixed order to its own copy of the residual stream: 2 barriers per layer
// + 1 for the argmax.  Slots are single-buffered: a slot is rewritten only in
// the next half of the same kind, which every CTA reaches after a barrier that
// follows its last read.  Every barrier sits in control flow that all CTAs
// evaluate identically, so barrier counts always match.
//
// Numerics: weights dequantised as float32(q) * scale, FP32 FMA dot products,
// RMSNorm with correctly rounded sqrt/divide, host-built RoPE tables, softmax
// with a per-thread running max rescaled to the CTA-wide max.  wo and W2
// outputs are sums of per-CTA partial dot products (fixed order), so the
// values match the batched step to FP32 rounding, not bit for bit.
#pragma once

#include <cooperative_groups.h>

#include "linear.cuh"

namespace q6w {
namespace b1 {

namespace cg = cooperative_groups;

constexpr int kCtas = 8;
constexpr int kThreads = 256;
constexpr int kMaxLayers = 8;
constexpr int kMaxHd = 32;
constexpr size_t kMaxSmem = 220 * 1024;  // dynamic shared memory cap of one CTA

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
  int dim, n_layers, n_heads, n_kv, hd, hidden, vocab, max_seq;
  float eps, denom;
  QM tok;
  const float* norm;
  const float* rope_cos;
  const float* rope_sin;
  Layer layers[kMaxLayers];
  // request
  const int32_t* prompt;
  const int32_t* prompt_len;  // device, one value
  int max_prompt_len, new_tokens, n_stop, min_new;
  int32_t stop_ids[kMaxStop];
  float* kc;
  float* vc;
  int32_t* sampled;
  int32_t* n_sampled;
  int32_t* stop_reason;
  float* step_logits;
  int32_t* state;  // [tok, pos, plen, gen, flags], carried between launches
  int32_t* err;
  int step_begin, step_end;  // model steps run by this launch
};

__host__ __device__ inline uint32_t up16(uint32_t v) { return (v + 15u) & ~15u; }

// Per-CTA slice bounds of a range split into kCtas parts (multiples of `m`).
__host__ __device__ inline void slice(int total, int m, int c, int& b, int& e) {
  const int units = total / m;
  const int per = units / kCtas, extra = units % kCtas;
  b = (c * per + (c < extra ? c : extra)) * m;
  e = b + (per + (c < extra ? 1 : 0)) * m;
}

// Widest hidden slice of any CTA, padded to whole 16-column units.
__host__ __device__ inline int hidden_cap(const Args& a) {
  const int units = a.hidden / 4;
  return (int)up16((uint32_t)(4 * (units / kCtas + (units % kCtas ? 1 : 0))));
}

// Vectors, at the same offsets in every CTA (peers address them with this
// CTA's offsets).  Bytes from the start of shared memory.
struct Vec {
  uint32_t cand;   // u64 [kCtas]: argmax candidate of each CTA
  uint32_t red;    // f32 [32]: reductions (16 u64 for the argmax)
  uint32_t x;      // f32 [dim]: residual stream
  uint32_t u;      // f32 [dim]: normalised input of the current matrix
  uint32_t att;    // f32 [kMaxHd]: attention output of this CTA's head
  uint32_t qkv;    // f32 [3 kMaxHd]: q | k | v of this CTA's head, current position
  uint32_t apart;  // f32 [8 kMaxHd]: per-warp attention partials
  uint32_t hl;     // f32 [hidden_cap]: SwiGLU slice (zero padded)
  uint32_t pa;     // f32 [kCtas][dim]: wo partials, slot per CTA
  uint32_t pb;     // f32 [kCtas][dim]: W2 partials, slot per CTA
  uint32_t rp;     // f32 [kMaxHd]: RoPE cos | sin of the current position
  uint32_t nw;     // f32 [(2 n_layers + 1) dim]: norm weights
  uint32_t tab;    // u32 [4][kCtas]: vocab slice begin, end, row offset, scale offset of each CTA
  uint32_t bytes;
};

__host__ __device__ inline Vec make_vec(const Args& a) {
  Vec v;
  uint32_t o = 0;
  auto take = [&](uint32_t bytes) { const uint32_t at = o; o = up16(o + bytes); return at; };
  v.cand = take(8 * kCtas);
  v.red = take(4 * 32);
  v.x = take(4 * a.dim);
  v.u = take(4 * a.dim);
  v.att = take(4 * kMaxHd);
  v.qkv = take(4 * 3 * kMaxHd);
  v.apart = take(4 * 8 * kMaxHd);
  v.hl = take(4 * hidden_cap(a));
  v.pa = take(4 * kCtas * a.dim);
  v.pb = take(4 * kCtas * a.dim);
  v.rp = take(4 * kMaxHd);
  v.nw = take(4 * (2 * a.n_layers + 1) * a.dim);
  v.tab = take(4 * 4 * kCtas);
  v.bytes = o;
  return v;
}

// Weights of CTA c, after the vectors.  Every layer block has the same
// layout; offsets within a block, then the vocab slice.
struct Plan {
  int head;                  // CTA c owns query head c
  int glu_b, glu_e, ngp;     // hidden units [glu_b, glu_e); ngp = width padded to 16
  int voc_b, voc_e;          // vocab rows
  int wo_stride, w2_stride;  // bytes per row of the wo / W2 column blocks
  uint32_t qkv, qkv_s, wo, wo_s, glu, glu_s, w2, w2_s;  // within a layer block
  uint32_t layers, layer_bytes;
  uint32_t voc, voc_s;
  uint32_t bytes;
};

__host__ __device__ inline void make_plan(const Args& a, int c, Plan& p) {
  const uint32_t rd = (uint32_t)a.dim * 3 / 4;
  p.head = c < a.n_heads;
  slice(a.hidden, 4, c, p.glu_b, p.glu_e);
  const int ng = p.glu_e - p.glu_b;
  p.ngp = (int)up16((uint32_t)ng);
  slice(a.vocab, 2, c, p.voc_b, p.voc_e);
  p.wo_stride = a.hd * 3 / 4;
  p.w2_stride = p.ngp * 3 / 4;
  const uint32_t nq = p.head ? 3u * a.hd : 0u, nd = p.head ? (uint32_t)a.dim : 0u;
  uint32_t o = 0;
  auto take = [&](uint32_t bytes) { const uint32_t at = o; o = up16(o + bytes); return at; };
  p.qkv = take(nq * rd);
  p.qkv_s = take(4 * nq);
  p.wo = take(nd * p.wo_stride);
  p.wo_s = take(4 * nd);
  p.glu = take(2u * ng * rd);
  p.glu_s = take(8u * ng);
  p.w2 = take((uint32_t)a.dim * p.w2_stride);
  p.w2_s = take(4u * a.dim);
  p.layer_bytes = o;
  p.layers = make_vec(a).bytes;
  o = p.layers + (uint32_t)a.n_layers * p.layer_bytes;
  p.voc = take((uint32_t)(p.voc_e - p.voc_b) * rd);
  p.voc_s = take(4u * (p.voc_e - p.voc_b));
  p.bytes = o;
}

// Dot products of N packed rows (K codes, K % 16 == 0; rows in shared memory)
// with x (shared memory) by a group of 8 lanes; every lane of the group
// returns the full sums.  The N rows share the x loads and run as independent
// FMA chains.  w = float32(q) * s then FMA, as the SIMT path.
template <int N>
__device__ __forceinline__ void group_dot(const uint8_t* const (&rows)[N], const float (&s)[N], const float* x,
                                          int K, int gl, float (&out)[N]) {
#pragma unroll
  for (int n = 0; n < N; ++n) out[n] = 0.0f;
  const int U = K >> 4;
  for (int u = gl; u < U; u += 8) {
    const float4* xv = reinterpret_cast<const float4*>(x + 16 * u);
    const float4 x0 = xv[0], x1 = xv[1], x2 = xv[2], x3 = xv[3];
#pragma unroll
    for (int n = 0; n < N; ++n) {
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(rows[n] + 12 * u);
      float w[16];
      dequant16(pw[0], pw[1], pw[2], s[n], w);
      float acc = out[n];
      acc = fmaf(w[0], x0.x, acc); acc = fmaf(w[1], x0.y, acc); acc = fmaf(w[2], x0.z, acc); acc = fmaf(w[3], x0.w, acc);
      acc = fmaf(w[4], x1.x, acc); acc = fmaf(w[5], x1.y, acc); acc = fmaf(w[6], x1.z, acc); acc = fmaf(w[7], x1.w, acc);
      acc = fmaf(w[8], x2.x, acc); acc = fmaf(w[9], x2.y, acc); acc = fmaf(w[10], x2.z, acc); acc = fmaf(w[11], x2.w, acc);
      acc = fmaf(w[12], x3.x, acc); acc = fmaf(w[13], x3.y, acc); acc = fmaf(w[14], x3.z, acc); acc = fmaf(w[15], x3.w, acc);
      out[n] = acc;
    }
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1)
#pragma unroll
    for (int n = 0; n < N; ++n) out[n] += __shfl_xor_sync(0xffffffffu, out[n], o);
}

// One thread's dot of a column block row (`units` 16-column units, packed at
// `row`, shared memory) with v (shared memory, read by every thread alike).
__device__ __forceinline__ float col_dot(const uint8_t* row, float s, const float* v, int units) {
  float acc = 0.0f;
  for (int u = 0; u < units; ++u) {
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 12 * u);
    float w[16];
    dequant16(pw[0], pw[1], pw[2], s, w);
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(w[k], v[16 * u + k], acc);
  }
  return acc;
}

// x (dim <= kThreads, shared) -> u = RMSNorm(x) * g (g in shared memory); whole
// CTA.  Thread k reads x[k] only, so a caller that just wrote x[k] from the
// same thread needs no barrier before.
__device__ __forceinline__ void rms_to(const float* x, const float* g, float* u, int dim, float eps, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float xv = tid < dim ? x[tid] : 0.0f;
  float ss = warp_sum(__fmul_rn(xv, xv));
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.0f;
  t = warp_sum(t);
  const float r = rms_scale(t, dim, eps);
  if (tid < dim) u[tid] = __fmul_rn(__fmul_rn(xv, r), g[tid]);
  __syncthreads();
}

// x[k] += sum of slots 0..n-1 of a partial buffer [kCtas][dim], fixed order.
__device__ __forceinline__ void add_partials(float* x, const float* part, int n, int dim) {
  const int k = threadIdx.x;
  if (k < dim) {
    float s = part[k];
    for (int i = 1; i < n; ++i) s = __fadd_rn(s, part[i * dim + k]);
    x[k] = __fadd_rn(x[k], s);
  }
}

__device__ __forceinline__ void copy_words(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
  // bytes and both addresses are multiples of 4
  const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
  uint32_t* d = reinterpret_cast<uint32_t*>(dst);
  for (uint32_t i = threadIdx.x; i < bytes / 4; i += kThreads) d[i] = __ldg(s + i);
}

// Column block [c0, c0 + n) of every row of a packed matrix (row_bytes per
// row; c0 % 4 == 0, n % 4 == 0) into rows of `stride` bytes, zero padded.
__device__ __forceinline__ void copy_cols(uint8_t* dst, const uint8_t* src, int rows, uint32_t row_bytes, int c0,
                                          int n, int stride) {
  const uint32_t b0 = (uint32_t)c0 * 3 / 4, nb = (uint32_t)n * 3 / 4;
  for (int i = threadIdx.x; i < rows * stride; i += kThreads) {
    const int r = i / stride, k = i % stride;
    dst[i] = k < (int)nb ? __ldg(src + (size_t)r * row_bytes + b0 + k) : (uint8_t)0;
  }
}

// One attention position held in registers: score q.k / denom, running max
// mt, running sum and weighted values rescaled when the max moves.
__device__ __forceinline__ void attn_visit(const float* q, const float4 (&k4)[kMaxHd / 4], const float4 (&v4)[kMaxHd / 4],
                                           int hd, float denom, float& mt, float& lsum, float (&acc)[kMaxHd]) {
  float d = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxHd / 4; ++i) {
    if (4 * i < hd) {
      d = fmaf(q[4 * i], k4[i].x, d);
      d = fmaf(q[4 * i + 1], k4[i].y, d);
      d = fmaf(q[4 * i + 2], k4[i].z, d);
      d = fmaf(q[4 * i + 3], k4[i].w, d);
    }
  }
  const float sc = __fdiv_rn(d, denom);
  const float mn = fmaxf(mt, sc);
  const float f = expf(mt - mn), pr = expf(sc - mn);
  mt = mn;
  lsum = fmaf(lsum, f, pr);
#pragma unroll
  for (int i = 0; i < kMaxHd / 4; ++i) {
    if (4 * i < hd) {
      acc[4 * i] = fmaf(acc[4 * i], f, pr * v4[i].x);
      acc[4 * i + 1] = fmaf(acc[4 * i + 1], f, pr * v4[i].y);
      acc[4 * i + 2] = fmaf(acc[4 * i + 2], f, pr * v4[i].z);
      acc[4 * i + 3] = fmaf(acc[4 * i + 3], f, pr * v4[i].w);
    }
  }
}

// K, V rows of one cached position (global memory, written by other CTAs of
// the cluster in earlier steps: read through L2).
__device__ __forceinline__ void load_kv(const float* k, const float* v, int hd, float4 (&k4)[kMaxHd / 4],
                                        float4 (&v4)[kMaxHd / 4]) {
#pragma unroll
  for (int i = 0; i < kMaxHd / 4; ++i) {
    if (4 * i < hd) {
      k4[i] = __ldcg(reinterpret_cast<const float4*>(k) + i);
      v4[i] = __ldcg(reinterpret_cast<const float4*>(v) + i);
    }
  }
}

__global__ void __cluster_dims__(kCtas, 1, 1) __launch_bounds__(kThreads, 1) b1_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t sm[];
  cg::cluster_group cl = cg::this_cluster();
  const int c = (int)cl.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane & 7, grp = tid >> 3;  // lane within its group of 8; group index (0..31)
  const int dim = a.dim, hd = a.hd, kvr = a.n_kv * hd, hid = a.hidden;
  const uint32_t rd = (uint32_t)dim * 3 / 4, rh = (uint32_t)hid * 3 / 4;
  const Vec V = make_vec(a);
  Plan P;
  make_plan(a, c, P);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(sm + V.cand);
  float* red = reinterpret_cast<float*>(sm + V.red);
  float* x = reinterpret_cast<float*>(sm + V.x);
  float* u = reinterpret_cast<float*>(sm + V.u);
  float* att = reinterpret_cast<float*>(sm + V.att);
  float* qkv = reinterpret_cast<float*>(sm + V.qkv);
  float* apart = reinterpret_cast<float*>(sm + V.apart);
  float* hl = reinterpret_cast<float*>(sm + V.hl);
  float* pa = reinterpret_cast<float*>(sm + V.pa);
  float* pb = reinterpret_cast<float*>(sm + V.pb);
  float* rp = reinterpret_cast<float*>(sm + V.rp);
  float* nw = reinterpret_cast<float*>(sm + V.nw);
  uint32_t* tab = reinterpret_cast<uint32_t*>(sm + V.tab);
  const int ng = P.glu_e - P.glu_b;
  const int rep = a.n_heads / a.n_kv;
  const int kvh = P.head ? c / rep : 0;
  const bool kv_writer = P.head && c % rep == 0;

  // ---- resident data (once per launch)
  for (int l = 0; l < a.n_layers; ++l) {
    const Layer& L = a.layers[l];
    uint8_t* blk = sm + P.layers + (uint32_t)l * P.layer_bytes;
    if (P.head) {
      copy_words(blk + P.qkv, L.wq.q + (size_t)c * hd * rd, hd * rd);
      copy_words(blk + P.qkv + hd * rd, L.wk.q + (size_t)kvh * hd * rd, hd * rd);
      copy_words(blk + P.qkv + 2 * hd * rd, L.wv.q + (size_t)kvh * hd * rd, hd * rd);
      copy_words(blk + P.qkv_s, reinterpret_cast<const uint8_t*>(L.wq.s + c * hd), 4 * hd);
      copy_words(blk + P.qkv_s + 4 * hd, reinterpret_cast<const uint8_t*>(L.wk.s + kvh * hd), 4 * hd);
      copy_words(blk + P.qkv_s + 8 * hd, reinterpret_cast<const uint8_t*>(L.wv.s + kvh * hd), 4 * hd);
      copy_cols(blk + P.wo, L.wo.q, dim, rd, c * hd, hd, P.wo_stride);
      copy_words(blk + P.wo_s, reinterpret_cast<const uint8_t*>(L.wo.s), 4 * dim);
    }
    copy_words(blk + P.glu, L.w1.q + (size_t)P.glu_b * rd, ng * rd);
    copy_words(blk + P.glu + ng * rd, L.w3.q + (size_t)P.glu_b * rd, ng * rd);
    copy_words(blk + P.glu_s, reinterpret_cast<const uint8_t*>(L.w1.s + P.glu_b), 4 * ng);
    copy_words(blk + P.glu_s + 4 * ng, reinterpret_cast<const uint8_t*>(L.w3.s + P.glu_b), 4 * ng);
    copy_cols(blk + P.w2, L.w2.q, dim, rh, P.glu_b, ng, P.w2_stride);
    copy_words(blk + P.w2_s, reinterpret_cast<const uint8_t*>(L.w2.s), 4 * dim);
    copy_words(reinterpret_cast<uint8_t*>(nw + 2 * l * dim), reinterpret_cast<const uint8_t*>(L.attn_norm), 4 * dim);
    copy_words(reinterpret_cast<uint8_t*>(nw + (2 * l + 1) * dim), reinterpret_cast<const uint8_t*>(L.ffn_norm),
               4 * dim);
  }
  copy_words(reinterpret_cast<uint8_t*>(nw + 2 * a.n_layers * dim), reinterpret_cast<const uint8_t*>(a.norm), 4 * dim);
  copy_words(sm + P.voc, a.tok.q + (size_t)P.voc_b * rd, (P.voc_e - P.voc_b) * rd);
  copy_words(sm + P.voc_s, reinterpret_cast<const uint8_t*>(a.tok.s + P.voc_b), 4 * (P.voc_e - P.voc_b));
  for (int j = tid; j < hidden_cap(a); j += kThreads) hl[j] = 0.0f;  // the padding stays zero
  if (tid < kCtas) {
    Plan q;
    make_plan(a, tid, q);
    tab[tid] = (uint32_t)q.voc_b;
    tab[kCtas + tid] = (uint32_t)q.voc_e;
    tab[2 * kCtas + tid] = q.voc;
    tab[3 * kCtas + tid] = q.voc_s;
  }
  __syncthreads();
  cl.sync();  // every CTA of the cluster is running and loaded before any remote access

  // greedy state (identical in every CTA)
  int tok = a.state[0], pos = a.state[1], plen = a.state[2], gen = a.state[3], flags = a.state[4];

  for (int step = a.step_begin; step < a.step_end && !(flags & SEQ_DONE); ++step) {
    // ---- step inputs: RoPE row of pos, next prompt token, embedding row of tok
    // (read from the shared memory of the CTA whose vocab slice holds it)
    if (tid < hd / 2) {
      rp[tid] = __ldg(a.rope_cos + (int64_t)pos * (hd / 2) + tid);
      rp[hd / 2 + tid] = __ldg(a.rope_sin + (int64_t)pos * (hd / 2) + tid);
    }
    const int next_prompt = pos + 1 < plen ? __ldg(a.prompt + pos + 1) : 0;
    {
      int o = 0;
      while (o < kCtas - 1 && (uint32_t)tok >= tab[kCtas + o]) ++o;
      const uint32_t rr = (uint32_t)tok - tab[o];
      const uint8_t* row = cl.map_shared_rank(sm + tab[2 * kCtas + o] + rr * rd, o);
      const float s = cl.map_shared_rank(reinterpret_cast<float*>(sm + tab[3 * kCtas + o]), o)[rr];
      if (tid < dim / 4) {
        const uint32_t v = (uint32_t)row[3 * tid] | ((uint32_t)row[3 * tid + 1] << 8) | ((uint32_t)row[3 * tid + 2] << 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) x[4 * tid + i] = __fmul_rn((float)group_code(v, i), s);
      }
      __syncthreads();
    }
    for (int l = 0; l < a.n_layers; ++l) {
      const uint8_t* blk = sm + P.layers + (uint32_t)l * P.layer_bytes;
      const int64_t layer_off = (int64_t)l * a.max_seq * kvr;
      const float* kb = a.kc + layer_off + kvh * hd;
      const float* vb = a.vc + layer_off + kvh * hd;
      // ---- attention half (no exchange until its end)
      if (l > 0) add_partials(x, pb, kCtas, dim);
      // cached k, v of this thread's first position: loads in flight during the norm and q, k, v
      float4 k4[kMaxHd / 4], v4[kMaxHd / 4];
      if (P.head && tid < pos) load_kv(kb + (int64_t)tid * kvr, vb + (int64_t)tid * kvr, hd, k4, v4);
      rms_to(x, nw + 2 * l * dim, u, dim, a.eps, red);
      if (P.head) {  // CTA-uniform
        // q of head c | k, v of its kv head; rows r, r ^ 1 sit on groups g, g ^ 1 (lanes ^ 8)
        const uint8_t* wq = blk + P.qkv;
        const float* sq = reinterpret_cast<const float*>(blk + P.qkv_s);
        for (int r0 = 0; r0 < 3 * hd; r0 += 64) {
          int r[2];
          const uint8_t* rows[2];
          float s[2], v[2];
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            r[n] = r0 + 32 * n + grp;
            const int rr = r[n] < 3 * hd ? r[n] : 0;
            rows[n] = wq + rr * rd;
            s[n] = sq[rr];
          }
          group_dot<2>(rows, s, u, dim, gl, v);
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            const float other = __shfl_xor_sync(0xffffffffu, v[n], 8);  // partner row r ^ 1
            if (r[n] < 3 * hd && gl == 0) {
              const int part = r[n] / hd, i = r[n] % hd, j = i >> 1;  // part 0: q, 1: k, 2: v
              float val = v[n];
              if (part < 2) {
                const float cs = rp[j], sn = rp[hd / 2 + j];
                val = (r[n] & 1) ? __fadd_rn(__fmul_rn(other, sn), __fmul_rn(v[n], cs))
                                 : __fsub_rn(__fmul_rn(v[n], cs), __fmul_rn(other, sn));
              }
              qkv[r[n]] = val;
              if (part > 0 && kv_writer) ((part == 1) ? a.kc : a.vc)[layer_off + (int64_t)pos * kvr + kvh * hd + i] = val;
            }
          }
        }
        __syncthreads();
        // attention of head c over positions 0..pos, one position per thread up to
        // 256; per-thread running max, then one rescale to the CTA-wide max
        float mt = -INFINITY, lsum = 0.0f, acc[kMaxHd];
#pragma unroll
        for (int i = 0; i < kMaxHd; ++i) acc[i] = 0.0f;
        if (tid < pos) attn_visit(qkv, k4, v4, hd, a.denom, mt, lsum, acc);
        for (int t = tid + kThreads; t < pos; t += kThreads) {
          load_kv(kb + (int64_t)t * kvr, vb + (int64_t)t * kvr, hd, k4, v4);
          attn_visit(qkv, k4, v4, hd, a.denom, mt, lsum, acc);
        }
        if (tid == pos % kThreads) {  // the current position, from shared memory
#pragma unroll
          for (int i = 0; i < kMaxHd / 4; ++i) {
            if (4 * i < hd) {
              k4[i] = reinterpret_cast<const float4*>(qkv + hd)[i];
              v4[i] = reinterpret_cast<const float4*>(qkv + 2 * hd)[i];
            }
          }
          attn_visit(qkv, k4, v4, hd, a.denom, mt, lsum, acc);
        }
        float mx = mt;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = red[0];
        for (int w = 1; w < kThreads / 32; ++w) mx = fmaxf(mx, red[w]);
        __syncthreads();
        const float g = expf(mt - mx);  // 0 for a thread without positions
        lsum = warp_sum(lsum * g);
#pragma unroll
        for (int i = 0; i < kMaxHd; ++i)
          if (i < hd) acc[i] = warp_sum(acc[i] * g);
        if (lane == 0) {
          red[warp] = lsum;
#pragma unroll
          for (int i = 0; i < kMaxHd; ++i)
            if (i < hd) apart[warp * hd + i] = acc[i];
        }
        __syncthreads();
        if (tid < hd) {
          float o = 0.0f, L = 0.0f;
          for (int w = 0; w < kThreads / 32; ++w) {
            o += apart[w * hd + tid];
            L += red[w];
          }
          att[tid] = __fdiv_rn(o, L);
        }
        __syncthreads();
        // wo columns of head c: partial of every output row, pushed to slot c
        if (tid < dim) {
          const float pv = col_dot(blk + P.wo + tid * P.wo_stride, reinterpret_cast<const float*>(blk + P.wo_s)[tid],
                                   att, hd / 16);
          for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(pa, d)[c * dim + tid] = pv;
        }
      }
      cl.sync();
      // ---- FFN half
      add_partials(x, pa, a.n_heads, dim);
      rms_to(x, nw + (2 * l + 1) * dim, u, dim, a.eps, red);
      {
        const uint8_t* w13 = blk + P.glu;
        const float* s13 = reinterpret_cast<const float*>(blk + P.glu_s);
        for (int j0 = 0; j0 < ng; j0 += 32) {  // warp-uniform: group g takes hidden unit j0 + g
          const int j = j0 + grp;
          const int jj = j < ng ? j : 0;
          const uint8_t* rows[2] = {w13 + jj * rd, w13 + (ng + jj) * rd};
          const float s[2] = {s13[jj], s13[ng + jj]};
          float v[2];
          group_dot<2>(rows, s, u, dim, gl, v);
          if (j < ng && gl == 0) hl[j] = swiglu(v[0], v[1]);
        }
      }
      __syncthreads();
      // W2 columns of this CTA's hidden units: partial of every output row, pushed to slot c
      if (tid < dim) {
        const float pv = col_dot(blk + P.w2 + tid * P.w2_stride, reinterpret_cast<const float*>(blk + P.w2_s)[tid],
                                 hl, P.ngp / 16);
        for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(pb, d)[c * dim + tid] = pv;
      }
      cl.sync();
    }
    // ---- vocab rows of this CTA, logits dump, masked argmax candidate
    add_partials(x, pb, kCtas, dim);
    rms_to(x, nw + 2 * a.n_layers * dim, u, dim, a.eps, red);
    {
      const bool sampling = pos >= plen - 1;
      const bool mask = a.n_stop && gen < a.min_new;
      const int nv = P.voc_e - P.voc_b;
      const float* vs = reinterpret_cast<const float*>(sm + P.voc_s);
      unsigned long long best = 0ull;
      for (int r0 = 0; r0 < nv; r0 += 128) {  // warp-uniform: group g takes rows r0 + g + 32 n
        const uint8_t* rows[4];
        float s[4], v[4];
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int r = r0 + 32 * n + grp;
          const int rr = r < nv ? r : 0;
          rows[n] = sm + P.voc + rr * rd;
          s[n] = vs[rr];
        }
        group_dot<4>(rows, s, u, dim, gl, v);
        if (gl == 0) {
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            const int r = r0 + 32 * n + grp;
            if (r < nv) {
              const int row = P.voc_b + r;
              float val = v[n];
              if (sampling && a.step_logits) a.step_logits[(int64_t)gen * a.vocab + row] = val;
              if (mask)
                for (int i = 0; i < a.n_stop; ++i)
                  if (a.stop_ids[i] == row) val = -INFINITY;
              best = umax64(best, argmax_key(val, row));
            }
          }
        }
      }
      for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
      if (lane == 0) reinterpret_cast<unsigned long long*>(red)[warp] = best;  // red: 16 u64
      __syncthreads();
      if (tid == 0) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kThreads / 32; ++w) k = umax64(k, reinterpret_cast<unsigned long long*>(red)[w]);
        for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(cand, d)[c] = k;
      }
    }
    cl.sync();
    // ---- greedy control (identical in every CTA; CTA 0 records)
    {
      unsigned long long k = 0ull;
      for (int i = 0; i < kCtas; ++i) k = umax64(k, cand[i]);
      const int t = argmax_index(k);
      if (pos < plen - 1) {
        tok = next_prompt;
        pos += 1;
      } else {
        if (c == 0 && tid == 0) {
          a.sampled[gen] = t;
          a.n_sampled[0] = gen + 1;
        }
        bool is_stop = false;
        for (int i = 0; i < a.n_stop; ++i) is_stop |= (a.stop_ids[i] == t);
        if (is_stop && gen >= a.min_new) {
          if (c == 0 && tid == 0) a.stop_reason[0] = t;
          flags |= SEQ_DONE;
        } else {
          gen += 1;
          if (gen >= a.new_tokens) {
            flags |= SEQ_DONE;
          } else {
            tok = t;
            pos += 1;
          }
        }
      }
      // every thread has read cand and red before the next step rewrites them
      // (cand only after the next vocab phase; red in the first norm)
      __syncthreads();
    }
  }
  if (c == 0 && tid == 0) {
    a.state[0] = tok;
    a.state[1] = pos;
    a.state[2] = plen;
    a.state[3] = gen;
    a.state[4] = flags;
  }
  cl.sync();  // no CTA leaves while a peer may still address its shared memory
}

// Prepare the state of a new request: token/position 0 and validation.
__global__ void b1_init_kernel(const int32_t* prompt, const int32_t* lens, int max_len, int vocab,
                               int32_t* state, int32_t* n_sampled, int32_t* stop_reason, int32_t* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int L = lens[0];
  bool ok = L >= 1 && L <= max_len;
  for (int i = 0; ok && i < L; ++i) ok = prompt[i] >= 0 && prompt[i] < vocab;
  state[0] = ok ? prompt[0] : 0;
  state[1] = 0;
  state[2] = ok ? L : 1;
  state[3] = 0;
  state[4] = ok ? 0 : (SEQ_DONE | SEQ_INVALID);
  n_sampled[0] = 0;
  stop_reason[0] = -1;
  if (!ok) atomicOr(err, 1);
}

}  // namespace b1
}  // namespace q6w
