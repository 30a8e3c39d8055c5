// B=1 greedy request as one persistent kernel per launch: an 8-CTA thread-block
// cluster keeps every weight matrix resident in shared memory (each CTA its
// 1/8 slice) and runs whole model steps -- embedding, the 5-phase layers,
// vocab projection, argmax and the greedy stop contract -- with no host
// involvement, like the reference's autonomous FPGA top
// (rtl/autonomous/tinyllm_autonomous.cpp:955-1153).
//
// Exchange: each phase's output slice is pushed into every CTA's copy of the
// vector through distributed shared memory, then one cluster barrier
// (release/acquire) publishes it; 5 barriers per layer + 1 for the argmax.
// A phase writes only its own slice of a vector that peers read no earlier
// than after the next barrier, so single buffering is race-free.  Every
// barrier sits in control flow that all CTAs evaluate identically (the same
// data drives the same branches), so barrier counts always match.
//
// Numerics are those of the SIMT step: weights dequantised as
// float32(q) * scale, FP32 FMA dot products, RMSNorm with correctly rounded
// sqrt/divide, host-built RoPE tables, online-softmax attention.
#pragma once

#include <cooperative_groups.h>

#include "linear.cuh"

namespace q6w {
namespace b1 {

namespace cg = cooperative_groups;

constexpr int kCtas = 8;
constexpr int kThreads = 256;
constexpr int kMaxLayers = 8;
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

// Per-CTA slice bounds of a row range split into kCtas parts (multiples of `m`).
__host__ __device__ inline void slice(int total, int m, int c, int& b, int& e) {
  const int units = total / m;
  const int per = units / kCtas, extra = units % kCtas;
  b = (c * per + (c < extra ? c : extra)) * m;
  e = b + (per + (c < extra ? 1 : 0)) * m;
}

// Dot product of one packed row (K codes, K % 16 == 0; `row` in shared
// memory) with x (shared memory) by a group of 8 lanes; every lane of the
// group returns the full sum.  w = float32(q) * s then FMA, as the SIMT path.
__device__ __forceinline__ float group_dot(const uint8_t* row, float s, const float* x, int K, int gl) {
  float acc = 0.0f;
  const int U = K >> 4;
  for (int u = gl; u < U; u += 8) {
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 12 * u);
    float w[16];
    dequant16(pw[0], pw[1], pw[2], s, w);
    const float4* xv = reinterpret_cast<const float4*>(x + 16 * u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = xv[j];
      acc = fmaf(w[4 * j], v.x, acc);
      acc = fmaf(w[4 * j + 1], v.y, acc);
      acc = fmaf(w[4 * j + 2], v.z, acc);
      acc = fmaf(w[4 * j + 3], v.w, acc);
    }
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

// x (dim, shared) -> u = RMSNorm(x) * g into shared memory; whole CTA.
__device__ __forceinline__ void rms_to(const float* x, const float* __restrict__ g, float* u, int dim, float eps,
                                       float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float ss = 0.0f;
  for (int k = tid; k < dim; k += kThreads) ss = __fadd_rn(ss, __fmul_rn(x[k], x[k]));
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.0f;
  t = warp_sum(t);
  const float r = rms_scale(t, dim, eps);
  for (int k = tid; k < dim; k += kThreads) u[k] = __fmul_rn(__fmul_rn(x[k], r), __ldg(g + k));
  __syncthreads();
}

// Shared-memory plan (bytes, 16-aligned), computed identically on host and device.
struct Plan {
  int qkv_b, qkv_e, wo_b, wo_e, glu_b, glu_e, w2_b, w2_e, voc_b, voc_e;  // row/pair ranges of CTA c
  size_t off_w[kMaxLayers][4];  // per layer: qkv rows, wo rows, w1|w3 pairs, w2 rows (packed bytes)
  size_t off_s[kMaxLayers][4];  // their scales
  size_t off_voc, off_voc_s;
  size_t off_vec;               // vectors
  size_t bytes;
};

__host__ __device__ inline size_t up16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ inline void make_plan(const Args& a, int c, Plan& p) {
  p.qkv_b = 0;
  p.qkv_e = c < a.n_heads ? 3 * a.hd : 0;  // rows: q of head c | k, v of its kv head
  slice(a.dim, 2, c, p.wo_b, p.wo_e);
  slice(a.hidden, 1, c, p.glu_b, p.glu_e);
  slice(a.dim, 2, c, p.w2_b, p.w2_e);
  slice(a.vocab, 2, c, p.voc_b, p.voc_e);
  const size_t rd = (size_t)a.dim * 3 / 4, rh = (size_t)a.hidden * 3 / 4;
  // vectors first: peers address them with this CTA's own offsets (DSMEM
  // pushes), so they sit at the same place in every CTA whatever its slices.
  // cand [kCtas] u64; red [32]; x, u, att [dim]; qkv [3 hd]; h [hidden]
  p.off_vec = 0;
  size_t o = up16(8 * kCtas + 4 * (size_t)(32 + 3 * a.dim + 3 * a.hd + a.hidden));
  for (int l = 0; l < a.n_layers; ++l) {
    p.off_w[l][0] = o; o = up16(o + (p.qkv_e - p.qkv_b) * rd);
    p.off_w[l][1] = o; o = up16(o + (p.wo_e - p.wo_b) * rd);
    p.off_w[l][2] = o; o = up16(o + 2 * (p.glu_e - p.glu_b) * rd);
    p.off_w[l][3] = o; o = up16(o + (p.w2_e - p.w2_b) * rh);
    p.off_s[l][0] = o; o = up16(o + 4 * (p.qkv_e - p.qkv_b));
    p.off_s[l][1] = o; o = up16(o + 4 * (p.wo_e - p.wo_b));
    p.off_s[l][2] = o; o = up16(o + 8 * (p.glu_e - p.glu_b));
    p.off_s[l][3] = o; o = up16(o + 4 * (p.w2_e - p.w2_b));
  }
  p.off_voc = o; o = up16(o + (p.voc_e - p.voc_b) * rd);
  p.off_voc_s = o; o = up16(o + 4 * (p.voc_e - p.voc_b));
  p.bytes = o;
}

// One attention position: score q.k / denom, running max mt, running sum and
// weighted values rescaled when the max moves.  kGlobal: k, v rows are in
// global memory (read through L2, written by other CTAs of the cluster);
// otherwise in this CTA's shared memory.
template <bool kGlobal>
__device__ __forceinline__ void attn_visit(const float* q, const float* k, const float* v, int hd, float denom,
                                           float& mt, float& lsum, float (&acc)[32]) {
  float d = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (4 * i < hd) {
      const float4 k4 = kGlobal ? __ldcg(reinterpret_cast<const float4*>(k) + i) : reinterpret_cast<const float4*>(k)[i];
      d = fmaf(q[4 * i], k4.x, d);
      d = fmaf(q[4 * i + 1], k4.y, d);
      d = fmaf(q[4 * i + 2], k4.z, d);
      d = fmaf(q[4 * i + 3], k4.w, d);
    }
  }
  const float sc = __fdiv_rn(d, denom);
  const float mn = fmaxf(mt, sc);
  const float f = expf(mt - mn), pr = expf(sc - mn);
  mt = mn;
  lsum = fmaf(lsum, f, pr);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (4 * i < hd) {
      const float4 v4 = kGlobal ? __ldcg(reinterpret_cast<const float4*>(v) + i) : reinterpret_cast<const float4*>(v)[i];
      acc[4 * i] = fmaf(acc[4 * i], f, pr * v4.x);
      acc[4 * i + 1] = fmaf(acc[4 * i + 1], f, pr * v4.y);
      acc[4 * i + 2] = fmaf(acc[4 * i + 2], f, pr * v4.z);
      acc[4 * i + 3] = fmaf(acc[4 * i + 3], f, pr * v4.w);
    }
  }
}

__device__ __forceinline__ void copy_rows(uint8_t* dst, const uint8_t* src, size_t bytes) {
  // bytes and both addresses are multiples of 4
  const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
  uint32_t* d = reinterpret_cast<uint32_t*>(dst);
  for (size_t i = threadIdx.x; i < bytes / 4; i += kThreads) d[i] = __ldg(s + i);
}

__global__ void __cluster_dims__(kCtas, 1, 1) __launch_bounds__(kThreads, 1) b1_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t sm[];
  cg::cluster_group cl = cg::this_cluster();
  const int c = (int)cl.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane & 7;  // lane within its group of 8 (one row per group)
  const int dim = a.dim, kvr = a.n_kv * a.hd, hid = a.hidden;
  const size_t rd = (size_t)dim * 3 / 4, rh = (size_t)hid * 3 / 4;
  Plan P;
  make_plan(a, c, P);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(sm + P.off_vec);  // [kCtas]
  float* red = reinterpret_cast<float*>(sm + P.off_vec + 8 * kCtas);                  // [32] (16 u64 for the argmax)
  float* x = red + 32;
  float* u = x + dim;
  float* att = u + dim;
  float* qkv = att + dim;  // q | k | v of this CTA's head (current position)
  float* h = qkv + 3 * a.hd;

  // ---- weight slices into shared memory (once per launch)
  for (int l = 0; l < a.n_layers; ++l) {
    const Layer& L = a.layers[l];
    // q rows of head c, k and v rows of its kv head
    if (c < a.n_heads) {
      const int kvh = c / (a.n_heads / a.n_kv), hd = a.hd;
      const QM* src[3] = {&L.wq, &L.wk, &L.wv};
      const int r0[3] = {c * hd, kvh * hd, kvh * hd};
      for (int m = 0; m < 3; ++m) {
        copy_rows(sm + P.off_w[l][0] + m * hd * rd, src[m]->q + r0[m] * rd, hd * rd);
        copy_rows(sm + P.off_s[l][0] + 4 * m * hd, reinterpret_cast<const uint8_t*>(src[m]->s + r0[m]), 4 * hd);
      }
    }
    copy_rows(sm + P.off_w[l][1], L.wo.q + P.wo_b * rd, (P.wo_e - P.wo_b) * rd);
    copy_rows(sm + P.off_s[l][1], reinterpret_cast<const uint8_t*>(L.wo.s + P.wo_b), 4 * (P.wo_e - P.wo_b));
    const int ng = P.glu_e - P.glu_b;
    copy_rows(sm + P.off_w[l][2], L.w1.q + P.glu_b * rd, ng * rd);
    copy_rows(sm + P.off_w[l][2] + ng * rd, L.w3.q + P.glu_b * rd, ng * rd);
    copy_rows(sm + P.off_s[l][2], reinterpret_cast<const uint8_t*>(L.w1.s + P.glu_b), 4 * ng);
    copy_rows(sm + P.off_s[l][2] + 4 * ng, reinterpret_cast<const uint8_t*>(L.w3.s + P.glu_b), 4 * ng);
    copy_rows(sm + P.off_w[l][3], L.w2.q + P.w2_b * rh, (P.w2_e - P.w2_b) * rh);
    copy_rows(sm + P.off_s[l][3], reinterpret_cast<const uint8_t*>(L.w2.s + P.w2_b), 4 * (P.w2_e - P.w2_b));
  }
  copy_rows(sm + P.off_voc, a.tok.q + P.voc_b * rd, (P.voc_e - P.voc_b) * rd);
  copy_rows(sm + P.off_voc_s, reinterpret_cast<const uint8_t*>(a.tok.s + P.voc_b), 4 * (P.voc_e - P.voc_b));
  __syncthreads();
  cl.sync();  // every CTA of the cluster is running before any remote access

  // greedy state (identical in every CTA)
  int tok = a.state[0], pos = a.state[1], plen = a.state[2], gen = a.state[3], flags = a.state[4];
  const int rep = a.n_heads / a.n_kv;

  for (int step = a.step_begin; step < a.step_end && !(flags & SEQ_DONE); ++step) {
    // ---- embedding row (every CTA, full vector)
    {
      const int groups = dim >> 2;
      const uint8_t* row = a.tok.q + (size_t)tok * rd;
      const float s = __ldg(a.tok.s + tok);
      for (int g = tid; g < groups; g += kThreads) {
        const uint32_t v = load_group(row + 3 * g);
#pragma unroll
        for (int i = 0; i < 4; ++i) x[4 * g + i] = __fmul_rn((float)group_code(v, i), s);
      }
      __syncthreads();
    }
    for (int l = 0; l < a.n_layers; ++l) {
      const Layer& L = a.layers[l];
      const int64_t layer_off = (int64_t)l * a.max_seq * kvr;
      // ---- phase 1: RMSNorm; q of head c and k, v of its kv head (RoPE on q, k);
      // the first CTA of each kv group writes k, v to the cache
      rms_to(x, L.attn_norm, u, dim, a.eps, red);
      const int rep_c = c < a.n_heads ? c % rep : 0;
      const int kvh = c < a.n_heads ? c / rep : 0;
      for (int r0 = warp * 4; r0 < P.qkv_e; r0 += 32) {  // warp-uniform (qkv_e is CTA-uniform); pairs on adjacent groups
        const int r = r0 + (lane >> 3);
        const bool live = r < P.qkv_e;
        const int rr = live ? r : r0;
        const uint8_t* row = sm + P.off_w[l][0] + rr * rd;
        const float s = reinterpret_cast<const float*>(sm + P.off_s[l][0])[rr];
        float v = group_dot(row, s, u, dim, gl);
        const float other = __shfl_xor_sync(0xffffffffu, v, 8);  // partner row (r ^ 1)
        if (live && gl == 0) {
          const int part = r / a.hd, j = (r % a.hd) >> 1;  // part 0: q, 1: k, 2: v
          if (part < 2) {
            const float cs = __ldg(a.rope_cos + (int64_t)pos * (a.hd >> 1) + j);
            const float sn = __ldg(a.rope_sin + (int64_t)pos * (a.hd >> 1) + j);
            v = (r & 1) ? __fadd_rn(__fmul_rn(other, sn), __fmul_rn(v, cs))
                        : __fsub_rn(__fmul_rn(v, cs), __fmul_rn(other, sn));
          }
          qkv[r] = v;
          if (part > 0 && rep_c == 0) {
            float* dst = (part == 1 ? a.kc : a.vc) + layer_off + (int64_t)pos * kvr + kvh * a.hd + (r % a.hd);
            *dst = v;
          }
        }
      }
      __syncthreads();
      // ---- phase 2: attention of head c over positions 0..pos, positions spread over
      // the threads (one each up to 256); per-thread running max, then one rescale to
      // the CTA-wide max, so a thread holding a single position computes exp(s - max)
      if (c < a.n_heads) {  // CTA-uniform
        const int hd = a.hd;
        const float* q = qkv;
        float mt = -INFINITY, lsum = 0.0f, acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        // earlier positions from the cache (global memory only), the current one
        // from shared memory: no pointer here may be of either space
        const float* kb = a.kc + layer_off + kvh * hd;
        const float* vb = a.vc + layer_off + kvh * hd;
        for (int t = tid; t < pos; t += kThreads)
          attn_visit<true>(q, kb + (int64_t)t * kvr, vb + (int64_t)t * kvr, hd, a.denom, mt, lsum, acc);
        if (tid == pos % kThreads) attn_visit<false>(q, qkv + hd, qkv + 2 * hd, hd, a.denom, mt, lsum, acc);
        float mx = mt;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = red[0];
        for (int w = 1; w < kThreads / 32; ++w) mx = fmaxf(mx, red[w]);
        __syncthreads();
        const float g = expf(mt - mx);  // 0 for a thread without positions
        lsum *= g;
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] *= g;
        lsum = warp_sum(lsum);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = warp_sum(acc[i]);
        // h is free during this phase (its next writer is phase 4): per-warp partials
        if (lane == 0) {
          red[warp] = lsum;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < hd) h[warp * hd + i] = acc[i];
        }
        __syncthreads();
        if (tid < hd) {
          float o = 0.0f, L = 0.0f;
          for (int w = 0; w < kThreads / 32; ++w) {
            o += h[w * hd + tid];
            L += red[w];
          }
          const float val = __fdiv_rn(o, L);
          for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(att, d)[c * hd + tid] = val;
        }
      }
      cl.sync();
      // ---- phase 3: wo rows of this CTA + residual, push x slice
      for (int r0 = P.wo_b + warp * 4; r0 < P.wo_e; r0 += 32) {
        const int r = r0 + (lane >> 3);
        const bool live = r < P.wo_e;
        const int rr = live ? r : r0;
        const uint8_t* row = sm + P.off_w[l][1] + (rr - P.wo_b) * rd;
        const float s = reinterpret_cast<const float*>(sm + P.off_s[l][1])[rr - P.wo_b];
        const float v = group_dot(row, s, att, dim, gl);
        if (live && gl == 0) {
          const float nx = __fadd_rn(x[r], v);
          for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(x, d)[r] = nx;
        }
      }
      cl.sync();
      // ---- phase 4: RMSNorm, W1/W3 pairs of this CTA, SwiGLU, push h slice
      rms_to(x, L.ffn_norm, u, dim, a.eps, red);
      {
        const int ng = P.glu_e - P.glu_b;
        const float* s1 = reinterpret_cast<const float*>(sm + P.off_s[l][2]);
        for (int j0 = warp * 2; j0 < ng; j0 += 16) {  // warp-uniform; groups (2q, 2q+1): W1 and W3 row j
          const int j = j0 + (lane >> 4);
          const bool live = j < ng;
          const int jj = live ? j : j0;
          const int which = (lane >> 3) & 1;
          const uint8_t* row = sm + P.off_w[l][2] + (which * ng + jj) * rd;
          const float s = s1[which * ng + jj];
          const float v = group_dot(row, s, u, dim, gl);
          const float other = __shfl_xor_sync(0xffffffffu, v, 8);
          if (live && gl == 0 && which == 0) {
            const float hv = swiglu(v, other);
            for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(h, d)[P.glu_b + j] = hv;
          }
        }
      }
      cl.sync();
      // ---- phase 5: w2 rows of this CTA + residual, push x slice
      for (int r0 = P.w2_b + warp * 4; r0 < P.w2_e; r0 += 32) {
        const int r = r0 + (lane >> 3);
        const bool live = r < P.w2_e;
        const int rr = live ? r : r0;
        const uint8_t* row = sm + P.off_w[l][3] + (rr - P.w2_b) * rh;
        const float s = reinterpret_cast<const float*>(sm + P.off_s[l][3])[rr - P.w2_b];
        const float v = group_dot(row, s, h, hid, gl);
        if (live && gl == 0) {
          const float nx = __fadd_rn(x[r], v);
          for (int d = 0; d < kCtas; ++d) cl.map_shared_rank(x, d)[r] = nx;
        }
      }
      cl.sync();
    }
    // ---- vocab rows of this CTA, logits dump, masked argmax candidate
    rms_to(x, a.norm, u, dim, a.eps, red);
    {
      const bool sampling = pos >= plen - 1;
      const bool mask = a.n_stop && gen < a.min_new;
      float bv = -INFINITY;
      int bi = -1;
      for (int r0 = P.voc_b + warp * 4; r0 < P.voc_e; r0 += 32) {
        const int r = r0 + (lane >> 3);
        const bool live = r < P.voc_e;
        const int rr = live ? r : r0;
        const uint8_t* row = sm + P.off_voc + (rr - P.voc_b) * rd;
        const float s = reinterpret_cast<const float*>(sm + P.off_voc_s)[rr - P.voc_b];
        float v = group_dot(row, s, u, dim, gl);
        if (!live) continue;
        if (gl == 0 && sampling && a.step_logits) a.step_logits[(int64_t)gen * a.vocab + r] = v;
        if (mask)
          for (int i = 0; i < a.n_stop; ++i)
            if (a.stop_ids[i] == r) v = -INFINITY;
        if (v > bv || bi < 0) {
          bv = v;
          bi = r;
        }
      }
      unsigned long long key = bi >= 0 && gl == 0 ? argmax_key(bv, bi) : 0ull;
      for (int o = 16; o > 0; o >>= 1) key = umax64(key, __shfl_xor_sync(0xffffffffu, key, o));
      if (lane == 0) reinterpret_cast<unsigned long long*>(red)[warp] = key;  // red: 8 u64 = 16 floats
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
        tok = __ldg(a.prompt + pos + 1);
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
      // next step's embedding overwrites x: every CTA must be past the
      // candidates read above before a peer could push again (next phase 1),
      // which happens only after the next step's first cl.sync -- fine.
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
