// Cached decode step of the Q6W transformer on sm_100a, and the device-resident
// greedy generation loop.
//
// One step for n sequences (each at its own position) is:
//   embed  -> x = dequant(E[token])                              (a4)
//   per layer l:
//     qkv    RMSNorm prologue, [wq|wk|wv] linear, RoPE, K/V cache write   (a5, a3, a6, a7)
//     attn   softmax(q K^T / sqrt(hd)) V over positions 0..pos, GQA       (a7)
//     wo     linear + residual add                                       (a3, a9)
//     ffn1   RMSNorm prologue, W1 and W3 together, silu(a) * b            (a5, a8)
//     w2     linear + residual add                                       (a8, a9)
//   vocab  RMSNorm prologue, tied-embedding linear, logits and
//          first-maximum argmax (with stop-id masking)               (a10)
// mirroring CachedTransformer.step (benchmarks/torch_benchmark.py:96-125).
// The greedy loop appends an `advance` kernel that applies the stop contract
// of torch_benchmark.py:272-293 / scripts/prepare_e2e.py:129-143 per
// sequence and feeds the next token; the whole step is captured once into a
// CUDA graph and replayed, so the host never synchronises inside a request.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <new>
#include <utility>
#include <vector>

#include "b1.cuh"
#include "launch.cuh"
#include "pdec.cuh"
#include "sample.cuh"
#include "tc.cuh"
#include "tcg.cuh"

#include <cudaTypedefs.h>

namespace q6w {

struct Work {
  float* x;
  float* qb;
  float* att;
  float* hb;
  unsigned long long* keys;
  int32_t* tok;
  int32_t* pos;
  int32_t* plen;
  int32_t* gen;
  int32_t* flags;
  int32_t* err;
  uint8_t* xs_img;   // tensor-core path: activation images (see tc.cuh)
  uint8_t* att_img;
  uint8_t* hs_img;
  const int32_t* seq;  // cache row of each activation row (prefill: rows are tokens); null: row i
  float* logits;       // sampling: the step's logits [N, vocab] (null unless laid out for sampling)
  unsigned long long* rng;  // sampling: XorShift64 state per sequence
  uint32_t* sync;      // persistent B=1 step: grid-barrier arrivals and the abort word
  const int32_t* poff;   // prefill: row offset and length of every prompt (null otherwise)
  const int32_t* plens;
  int32_t n_prompts, max_len;
  int32_t pdl;           // launch the tensor-core step's kernels with programmatic dependencies
};

struct GraphKey {
  q6w_greedy_args a;
  int32_t stop[kMaxStop];
  void* ws;
  int32_t sampler;          // the step graph runs the sampler kernel
  smp::Params sp;
};

}  // namespace q6w

struct q6w_model {
  q6w_model_desc d;
  std::vector<q6w_layer_weights> layers;
  int32_t hd, kv_rows;
  float denom;
  int device;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t exec = nullptr;
  q6w::GraphKey key;
  bool have_key = false;
  bool use_tc = false;  // shapes qualify for the tensor-core batched path (dim 128)
  bool use_tcg = false; // shapes qualify for the general tensor-core linears (any width)
  int sm_count = 148;
  bool use_b1 = false;  // shapes qualify for the single-request cluster kernel
  bool kv_half = false; // the KV cache holds FP16 (q6w_model_set_kv_dtype)
  bool use_pdec = false;  // shapes qualify for the persistent B=1 step (pdec.cuh)
  int pdl_mode = -1;      // programmatic dependent launch in the tensor-core step: 1 on, 0 off (Q6W_PDL), -1 by batch
  int attn_deep_mode = -1;  // decode attention with two passes of K/V in flight: 1 on, 0 off (Q6W_ATTN_DEEP), -1 by batch
  int pdec_grid = 0;
  size_t pdec_smem = 0;
  size_t b1_smem = 0;
};

namespace q6w {

static size_t carve(char*& p, size_t bytes) {
  size_t off = (size_t)p;
  p += (bytes + 255) & ~(size_t)255;
  return off;
}

// Launch with an optional programmatic dependency on the stream's preceding
// kernel (the kernel itself calls grid_dep_wait before reading its inputs).
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Workspace of N sequences.  With `sample`, the sampler's regions (the step
// logits and the generator states) follow the rest, so every other offset is
// the same with or without them.
static size_t layout(const q6w_model* M, int N, char* base, Work* w, bool sample = false) {
  const auto& d = M->d;
  char* p = base;
  Work t;
  t.err = (int32_t*)carve(p, 4);  // first: q6w_workspace_status reads offset 0
  t.x = (float*)carve(p, sizeof(float) * (size_t)N * d.dim);
  t.qb = (float*)carve(p, sizeof(float) * (size_t)N * d.dim);
  t.att = (float*)carve(p, sizeof(float) * (size_t)N * d.dim);
  t.hb = (float*)carve(p, sizeof(float) * (size_t)N * d.hidden_dim);
  t.keys = (unsigned long long*)carve(p, sizeof(unsigned long long) * (size_t)N);
  t.tok = (int32_t*)carve(p, 4 * (size_t)N);
  t.pos = (int32_t*)carve(p, 4 * (size_t)N);
  t.plen = (int32_t*)carve(p, 4 * (size_t)N);
  t.gen = (int32_t*)carve(p, 4 * (size_t)N);
  t.flags = (int32_t*)carve(p, 4 * (size_t)N);
  t.sync = (uint32_t*)carve(p, 8);
  if (M->use_tc || M->use_tcg) {
    t.xs_img = (uint8_t*)carve(p, tc::img_bytes(N, d.dim));
    t.att_img = (uint8_t*)carve(p, tc::img_bytes(N, d.dim));
    t.hs_img = (uint8_t*)carve(p, tc::img_bytes(N, d.hidden_dim));
  } else {
    t.xs_img = t.att_img = t.hs_img = nullptr;
  }
  t.seq = nullptr;
  t.poff = t.plens = nullptr;
  t.n_prompts = t.max_len = 0;
  t.pdl = 0;
  t.logits = nullptr;
  t.rng = nullptr;
  if (sample) {
    t.logits = (float*)carve(p, sizeof(float) * (size_t)N * d.vocab_size);
    t.rng = (unsigned long long*)carve(p, 8 * (size_t)N);
  }
  if (w) *w = t;
  return (size_t)(p - base);
}

// ---- small kernels -----------------------------------------------------------

__global__ void init_batch_kernel(int n, const int32_t* __restrict__ tokens,
                                  const int32_t* __restrict__ positions, int32_t tok_scalar,
                                  int32_t pos_scalar, Work w) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n; b += gridDim.x * blockDim.x) {
    w.tok[b] = tokens ? tokens[b] : tok_scalar;
    w.pos[b] = positions ? positions[b] : pos_scalar;
    w.plen[b] = 0;
    w.gen[b] = 0;
    w.flags[b] = 0;
    w.keys[b] = 0ull;
  }
}

__global__ void init_greedy_kernel(int n, const int32_t* __restrict__ prompts,
                                   const int32_t* __restrict__ lens, int32_t stride,
                                   int32_t max_len, Work w, int32_t* n_sampled,
                                   int32_t* stop_reason, const unsigned long long* __restrict__ seeds) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n; b += gridDim.x * blockDim.x) {
    if (w.rng) w.rng[b] = seeds ? seeds[b] : 0ull;  // XorShift64(seed): the state is the seed
    const int32_t L = lens[b];
    const bool ok = L >= 1 && L <= max_len;
    w.tok[b] = ok ? prompts[(int64_t)b * stride] : 0;
    w.pos[b] = 0;
    w.plen[b] = ok ? L : 1;
    w.gen[b] = 0;
    w.flags[b] = ok ? 0 : (SEQ_DONE | SEQ_INVALID);
    w.keys[b] = 0ull;
    n_sampled[b] = 0;
    stop_reason[b] = -1;
    if (!ok) atomicOr(w.err, 1);
  }
}

// x[b] = float(E[token]) * scale[token]; also validates token/position.
__global__ void embed_kernel(const uint8_t* __restrict__ E, const float* __restrict__ Es, int dim,
                             int vocab, int max_seq, int n, Work w) {
  const int groups = dim >> 2;
  for (int b = blockIdx.x; b < n; b += gridDim.x) {
    const int t = w.tok[b], p = w.pos[b];
    const bool ok = t >= 0 && t < vocab && p >= 0 && p < max_seq;
    if (threadIdx.x == 0) {
      const int f = w.flags[b];
      w.flags[b] = ok ? (f & ~SEQ_INVALID) : (f | SEQ_INVALID);
      if (!ok && !(f & SEQ_DONE)) atomicOr(w.err, 1);
    }
    float* xr = w.x + (int64_t)b * dim;
    if (!ok) {
      for (int c = threadIdx.x; c < dim; c += blockDim.x) xr[c] = 0.0f;
      continue;
    }
    const uint8_t* row = E + (int64_t)t * groups * 3;
    const float s = __ldg(Es + t);
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
      const uint32_t v = load_group(row + 3 * g);
      reinterpret_cast<float4*>(xr)[g] =
          make_float4(__fmul_rn((float)group_code(v, 0), s), __fmul_rn((float)group_code(v, 1), s),
                      __fmul_rn((float)group_code(v, 2), s), __fmul_rn((float)group_code(v, 3), s));
    }
  }
}

// Decode attention over the FP32 cache (torch_benchmark.py:113-119).
// One warp per (sequence, query head); G lanes share one cached position
// (16 head dims per lane), 32/G positions per pass.  Pass 1 writes the
// scaled scores to shared memory, pass 2 the max-subtracted exponentials,
// pass 3 accumulates the normalised weights times V.
template <int G>
__global__ void __launch_bounds__(256) attn_kernel(const float* __restrict__ qb, int ldq,
                                                   const float* __restrict__ kc,
                                                   const float* __restrict__ vc, int64_t cstride,
                                                   int64_t layer_off, const int32_t* __restrict__ len,
                                                   int len_add, const int32_t* __restrict__ flags,
                                                   float* __restrict__ out, int ldo, int H, int KV,
                                                   int S, float denom, const int32_t* __restrict__ seq) {
  extern __shared__ float sc[];
  constexpr int P = 32 / G;
  constexpr int HD = 16 * G;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x, h = blockIdx.y * (blockDim.x >> 5) + warp;
  if (h >= H) return;
  const int slot = lane / G, part = lane % G;
  float* o = out + (int64_t)b * ldo + h * HD + 16 * part;
  int T = len[b] + len_add;
  T = T > S ? S : T;
  if ((flags && (flags[b] & SEQ_INVALID)) || T <= 0) {
    if (slot == 0)
      for (int i = 0; i < 16; ++i) o[i] = 0.0f;
    return;
  }
  const int g = h / (H / KV);
  const int kvr = KV * HD;
  const int64_t crow = seq ? seq[b] : b;
  const float* kb = kc + crow * cstride + layer_off + g * HD + 16 * part;
  const float* vb = vc + crow * cstride + layer_off + g * HD + 16 * part;
  float q[16];
  {
    const float4* qp = reinterpret_cast<const float4*>(qb + (int64_t)b * ldq + h * HD + 16 * part);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = qp[j];
      q[4 * j] = v.x; q[4 * j + 1] = v.y; q[4 * j + 2] = v.z; q[4 * j + 3] = v.w;
    }
  }
  float* s = sc + warp * S;
  float mx = -INFINITY;
  for (int t0 = 0; t0 < T; t0 += P) {
    const int t = t0 + slot;
    float d = 0.0f;
    if (t < T) {
      const float4* kp = reinterpret_cast<const float4*>(kb + (int64_t)t * kvr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 k4 = kp[j];
        d = fmaf(q[4 * j], k4.x, d);
        d = fmaf(q[4 * j + 1], k4.y, d);
        d = fmaf(q[4 * j + 2], k4.z, d);
        d = fmaf(q[4 * j + 3], k4.w, d);
      }
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    d = __fdiv_rn(d, denom);
    if (t < T) {
      if (part == 0) s[t] = d;
      mx = fmaxf(mx, d);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  __syncwarp();
  float sum = 0.0f;
  for (int t = lane; t < T; t += 32) {
    const float e = expf(s[t] - mx);
    s[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  __syncwarp();
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
  for (int t0 = 0; t0 < T; t0 += P) {
    const int t = t0 + slot;
    if (t < T) {
      const float wt = __fdiv_rn(s[t], sum);
      const float4* vp = reinterpret_cast<const float4*>(vb + (int64_t)t * kvr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v4 = vp[j];
        acc[4 * j] = fmaf(wt, v4.x, acc[4 * j]);
        acc[4 * j + 1] = fmaf(wt, v4.y, acc[4 * j + 1]);
        acc[4 * j + 2] = fmaf(wt, v4.z, acc[4 * j + 2]);
        acc[4 * j + 3] = fmaf(wt, v4.w, acc[4 * j + 3]);
      }
    }
  }
#pragma unroll
  for (int off = G; off < 32; off <<= 1)
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
  if (slot == 0) {
    float4* op = reinterpret_cast<float4*>(o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      op[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
  }
}

// Decode attention, one CTA per (sequence, query head), for head dims the
// warp-per-sequence kernel does not cover (64, 128) and few sequences (B=1
// decode of large models): every thread scores its own positions (all K rows
// in flight at once), the CTA reduces max and sum, then threads regroup as
// (4-dim column, position stride) to accumulate probability * V, merged in a
// fixed order.  Softmax as torch: exp(s - max), divide by the sum, then the
// weighted sum of V rows (torch_benchmark.py:114-119).
template <int HD, typename KT = float>
__global__ void __launch_bounds__(256) attn_head_kernel(
    const float* __restrict__ qb, int ldq, const KT* __restrict__ kc, const KT* __restrict__ vc,
    int64_t cstride, int64_t layer_off, const int32_t* __restrict__ len, int len_add,
    const int32_t* __restrict__ flags, float* __restrict__ out, int ldo, int H, int KV, int S, float denom,
    const int32_t* __restrict__ seq) {
  constexpr int CQ = HD / 4;        // float4 columns of a row
  constexpr int G = 256 / CQ;       // position groups in the V pass
  extern __shared__ __align__(16) float sa[];
  float* sq = sa;                   // [HD]
  float* red = sq + HD;             // [16]
  float4* part = reinterpret_cast<float4*>(red + 16);  // [G][CQ]
  float* sp = reinterpret_cast<float*>(part + G * CQ);  // [S] scores, then exp
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x, h = blockIdx.y;
  float* o = out + (int64_t)b * ldo + h * HD;
  int T = len[b] + len_add;
  T = T > S ? S : T;
  if ((flags && (flags[b] & SEQ_INVALID)) || T <= 0) {
    if (tid < HD) o[tid] = 0.0f;
    return;
  }
  const int kvr = KV * HD;
  const int g = h / (H / KV);
  const int64_t crow = seq ? seq[b] : b;
  const KT* kb = kc + crow * cstride + layer_off + g * HD;
  const KT* vb = vc + crow * cstride + layer_off + g * HD;
  if (tid < HD) sq[tid] = qb[(int64_t)b * ldq + h * HD + tid];
  // this thread's first V rows of the V pass, requested now so their latency
  // hides behind the score phase
  const int cq = tid % CQ, grp = tid / CQ;
  constexpr int kVP = 4;
  float4 vpre[kVP];
#pragma unroll
  for (int i = 0; i < kVP; ++i) {
    const int t = grp + i * G;
    vpre[i] = t < T ? load_kv4(vb + (int64_t)t * kvr + 4 * cq) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int t = tid; t < T; t += 256) {
    const KT* kr = kb + (int64_t)t * kvr;
    float d = 0.0f;
#pragma unroll
    for (int j = 0; j < CQ; ++j) {
      const float4 k4 = load_kv4(kr + 4 * j);
      d = fmaf(sq[4 * j], k4.x, d);
      d = fmaf(sq[4 * j + 1], k4.y, d);
      d = fmaf(sq[4 * j + 2], k4.z, d);
      d = fmaf(sq[4 * j + 3], k4.w, d);
    }
    d = __fdiv_rn(d, denom);
    sp[t] = d;
    mx = fmaxf(mx, d);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
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
  __syncthreads();
  sum = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[8 + w];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kVP; ++i) {  // the prefetched rows, in position order
    const int t = grp + i * G;
    if (t < T) {
      const float wt = __fdiv_rn(sp[t], sum);
      acc.x = fmaf(wt, vpre[i].x, acc.x);
      acc.y = fmaf(wt, vpre[i].y, acc.y);
      acc.z = fmaf(wt, vpre[i].z, acc.z);
      acc.w = fmaf(wt, vpre[i].w, acc.w);
    }
  }
  for (int t = grp + kVP * G; t < T; t += G) {
    const float wt = __fdiv_rn(sp[t], sum);
    const float4 v4 = load_kv4(vb + (int64_t)t * kvr + 4 * cq);
    acc.x = fmaf(wt, v4.x, acc.x);
    acc.y = fmaf(wt, v4.y, acc.y);
    acc.z = fmaf(wt, v4.z, acc.z);
    acc.w = fmaf(wt, v4.w, acc.w);
  }
  part[grp * CQ + cq] = acc;
  __syncthreads();
  if (tid < CQ) {
    float4 r = part[tid];
    for (int k = 1; k < G; ++k) {
      const float4 p = part[k * CQ + tid];
      r.x += p.x; r.y += p.y; r.z += p.z; r.w += p.w;
    }
    reinterpret_cast<float4*>(o)[tid] = r;
  }
}

// Decode attention for one (sequence, kv head): the REP query heads of the
// group share every K and V row load (attn_head_kernel reads each row once per
// query head).  Per head, the scores, the maximum, the sum of exponentials and
// the V accumulation keep attn_head_kernel's thread mapping and order, so the
// outputs are bit-identical to it.
// STAGE_V: the group's V rows [0, T) are copied into shared memory (cp.async)
// at the start, so their latency hides behind the score phase.
template <int HD, int REP, bool STAGE_V, typename KT = float>
__global__ void __launch_bounds__(256) attn_group_kernel(
    const float* __restrict__ qb, int ldq, const KT* __restrict__ kc, const KT* __restrict__ vc,
    int64_t cstride, int64_t layer_off, const int32_t* __restrict__ len, int len_add,
    const int32_t* __restrict__ flags, float* __restrict__ out, int ldo, int KV, int S, float denom,
    const int32_t* __restrict__ seq) {
  constexpr int CQ = HD / 4;  // float4 columns of a row
  constexpr int G = 256 / CQ; // position groups in the V pass
  extern __shared__ __align__(16) float sa[];
  float* sq = sa;                                              // [REP][HD]
  float* red = sq + REP * HD;                                  // [REP][16]
  float4* part = reinterpret_cast<float4*>(red + REP * 16);    // [REP][G][CQ]
  float* sp = reinterpret_cast<float*>(part + REP * G * CQ);   // [REP][S] scores, then exp
  float4* sv = reinterpret_cast<float4*>(sp + ((REP * S + 3) & ~3));  // STAGE_V: [S][CQ] V rows, 16-B aligned
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x, g = blockIdx.y;
  float* o = out + (int64_t)b * ldo + g * REP * HD;
  int T = len[b] + len_add;
  T = T > S ? S : T;
  if ((flags && (flags[b] & SEQ_INVALID)) || T <= 0) {
    for (int i = tid; i < REP * HD; i += 256) o[i] = 0.0f;
    return;
  }
  const int kvr = KV * HD;
  const int64_t crow = seq ? seq[b] : b;
  const KT* kb = kc + crow * cstride + layer_off + g * HD;
  const KT* vb = vc + crow * cstride + layer_off + g * HD;
  static_assert(!STAGE_V || sizeof(KT) == 4, "V staging copies FP32 rows");
  if (STAGE_V) {
    for (int i = tid; i < T * CQ; i += 256) {
      const int t = i / CQ, c = i % CQ;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sv + i)),
                   "l"(vb + (int64_t)t * kvr + 4 * c)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int i = tid; i < REP * HD; i += 256) sq[i] = qb[(int64_t)b * ldq + g * REP * HD + i];
  __syncthreads();
  float mx[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) mx[r] = -INFINITY;
  for (int t = tid; t < T; t += 256) {
    const KT* kr = kb + (int64_t)t * kvr;
    float d[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) d[r] = 0.0f;
#pragma unroll
    for (int j = 0; j < CQ; ++j) {
      const float4 k4 = load_kv4(kr + 4 * j);
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        const float4 q4 = reinterpret_cast<const float4*>(sq + r * HD)[j];
        d[r] = fmaf(q4.x, k4.x, d[r]);
        d[r] = fmaf(q4.y, k4.y, d[r]);
        d[r] = fmaf(q4.z, k4.z, d[r]);
        d[r] = fmaf(q4.w, k4.w, d[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float sc = __fdiv_rn(d[r], denom);
      sp[r * S + t] = sc;
      mx[r] = fmaxf(mx[r], sc);
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], off));
    if (lane == 0) red[r * 16 + warp] = mx[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float m = red[r * 16];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[r * 16 + w]);
    mx[r] = m;
  }
  float sum[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) sum[r] = 0.0f;
  for (int t = tid; t < T; t += 256) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float e = expf(sp[r * S + t] - mx[r]);
      sp[r * S + t] = e;
      sum[r] += e;
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    sum[r] = warp_sum(sum[r]);
    if (lane == 0) red[r * 16 + 8 + warp] = sum[r];
  }
  if (STAGE_V) asm volatile("cp.async.wait_group 0;" ::: "memory");  // this thread's V copies landed
  __syncthreads();
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    float sm = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sm += red[r * 16 + 8 + w];
    sum[r] = sm;
  }
  const int cq = tid % CQ, grp = tid / CQ;
  float4 acc[REP];
#pragma unroll
  for (int r = 0; r < REP; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = grp; t < T; t += G) {
    const float4 v4 = STAGE_V ? sv[t * CQ + cq] : load_kv4(vb + (int64_t)t * kvr + 4 * cq);
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float wt = __fdiv_rn(sp[r * S + t], sum[r]);
      acc[r].x = fmaf(wt, v4.x, acc[r].x);
      acc[r].y = fmaf(wt, v4.y, acc[r].y);
      acc[r].z = fmaf(wt, v4.z, acc[r].z);
      acc[r].w = fmaf(wt, v4.w, acc[r].w);
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) part[(r * G + grp) * CQ + cq] = acc[r];
  __syncthreads();
  for (int i = tid; i < REP * CQ; i += 256) {
    const int r = i / CQ, c = i % CQ;
    float4 x = part[r * G * CQ + c];
    for (int k = 1; k < G; ++k) {
      const float4 p = part[(r * G + k) * CQ + c];
      x.x += p.x; x.y += p.y; x.z += p.z; x.w += p.w;
    }
    reinterpret_cast<float4*>(o + r * HD)[c] = x;
  }
}

// Shared memory of attn_group_kernel for S positions (+ the staged V rows).
static size_t attn_group_smem(int hd, int rep, int S, bool stage_v) {
  return (size_t)rep * ((size_t)hd * 4 + 64 + 256 * 16 + (size_t)S * 4) + (stage_v ? (size_t)S * hd * 4 + 16 : 0);
}

// The V-staging kernels need more than the default 48 KB of dynamic shared
// memory: allowed once per process (model creation and the attention op call
// this before any launch); two CTAs still fit on an SM.
constexpr size_t kAttnStageMax = 110 * 1024;
static bool g_attn_stage_ok = false;
static void attn_group_setup() {
  static std::once_flag once;
  std::call_once(once, [] {
    bool ok = true;
#define Q6W_GROUP_ATTR(HDV, REPV)                                                                          \
  ok = ok && cudaFuncSetAttribute(attn_group_kernel<HDV, REPV, true>,                                      \
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnStageMax) == cudaSuccess;
    Q6W_GROUP_ATTR(64, 2) Q6W_GROUP_ATTR(64, 4) Q6W_GROUP_ATTR(64, 8)
    Q6W_GROUP_ATTR(128, 2) Q6W_GROUP_ATTR(128, 4) Q6W_GROUP_ATTR(128, 8)
#undef Q6W_GROUP_ATTR
    if (!ok) cudaGetLastError();
    g_attn_stage_ok = ok;
  });
}

// Shared memory of attn_head_kernel for S positions.
static size_t attn_head_smem(int hd, int S) { return (size_t)(hd + 16) * 4 + 256 * 16 + (size_t)S * 4; }

static bool launch_attn_head(int hd, int n, int H, int KV, cudaStream_t st, const float* qb, int ldq,
                             const void* kc, const void* vc, int64_t cstride, int64_t layer_off,
                             const int32_t* len, int len_add, const int32_t* flags, float* out, int ldo, int S,
                             float denom, const int32_t* seq = nullptr, bool kv_half = false) {
  const float* kf = static_cast<const float*>(kc);
  const float* vf = static_cast<const float*>(vc);
  const __half* kh = static_cast<const __half*>(kc);
  const __half* vh = static_cast<const __half*>(vc);
  // many (sequence, kv head) pairs: one CTA per pair serves the group's query heads
  const int rep = KV > 0 ? H / KV : 0;
  const bool stage = !kv_half && g_attn_stage_ok && attn_group_smem(hd, rep, S, true) <= kAttnStageMax;
  if (n * KV >= 128 && KV * rep == H && KV <= 65535 && (rep == 2 || rep == 4 || rep == 8) &&
      (hd == 64 || hd == 128) && (stage || attn_group_smem(hd, rep, S, false) <= 48 * 1024)) {
    const dim3 ggrid(n, KV);
    const size_t gsm = attn_group_smem(hd, rep, S, stage);
#define Q6W_GROUP(HDV, REPV)                                                                                     \
  if (hd == HDV && rep == REPV) {                                                                                \
    if (kv_half)                                                                                                 \
      attn_group_kernel<HDV, REPV, false, __half><<<ggrid, 256, gsm, st>>>(qb, ldq, kh, vh, cstride, layer_off, \
                                                                           len, len_add, flags, out, ldo, KV, S, \
                                                                           denom, seq);                          \
    else if (stage)                                                                                              \
      attn_group_kernel<HDV, REPV, true><<<ggrid, 256, gsm, st>>>(qb, ldq, kf, vf, cstride, layer_off, len,      \
                                                                  len_add, flags, out, ldo, KV, S, denom, seq);  \
    else                                                                                                         \
      attn_group_kernel<HDV, REPV, false><<<ggrid, 256, gsm, st>>>(qb, ldq, kf, vf, cstride, layer_off, len,     \
                                                                   len_add, flags, out, ldo, KV, S, denom, seq); \
  }
    Q6W_GROUP(64, 2) Q6W_GROUP(64, 4) Q6W_GROUP(64, 8) Q6W_GROUP(128, 2) Q6W_GROUP(128, 4) Q6W_GROUP(128, 8)
#undef Q6W_GROUP
    return true;
  }
  const size_t smem = attn_head_smem(hd, S);
  if (smem > 48 * 1024 || H > 65535 || (hd != 64 && hd != 128)) return false;
  const dim3 grid(n, H);
  if (hd == 64 && kv_half)
    attn_head_kernel<64, __half><<<grid, 256, smem, st>>>(qb, ldq, kh, vh, cstride, layer_off, len, len_add, flags,
                                                          out, ldo, H, KV, S, denom, seq);
  else if (hd == 64)
    attn_head_kernel<64><<<grid, 256, smem, st>>>(qb, ldq, kf, vf, cstride, layer_off, len, len_add, flags, out,
                                                  ldo, H, KV, S, denom, seq);
  else if (kv_half)
    attn_head_kernel<128, __half><<<grid, 256, smem, st>>>(qb, ldq, kh, vh, cstride, layer_off, len, len_add,
                                                           flags, out, ldo, H, KV, S, denom, seq);
  else
    attn_head_kernel<128><<<grid, 256, smem, st>>>(qb, ldq, kf, vf, cstride, layer_off, len, len_add, flags, out,
                                                   ldo, H, KV, S, denom, seq);
  return true;
}

// Whether FP16 KV storage is served for this head layout: the warp kernel
// (head dims 16 / 32 with an instantiated kv-head count and group size) or
// the group / per-head kernels (head dims 64 / 128).
static bool attn_rows_instantiated(int hd, int KV, int rep) {
  const bool k16 = hd == 16 && (KV == 1 || KV == 2 || KV == 4 || KV == 8) && (rep == 1 || rep == 2 || rep == 4);
  const bool k32 = hd == 32 && (KV == 1 || KV == 2 || KV == 4) && (rep == 1 || rep == 2 || rep == 4);
  return k16 || k32;
}

// Decode attention, one warp per sequence: the warp streams the sequence's
// K and V rows 0..T-1 once (32/R rows per pass, R = KV*HD/16 lanes per row,
// 16 dims per lane), prefetching the next pass's rows (or the next two
// passes', at small batches) while it computes the current one, with an
// online softmax per lane for the REP query heads of its kv head; lanes
// holding the same (kv head, dims) merge by shuffles.

// One pass of a lane: position t's K and V rows (kv, vv; act: t < T) into
// the lane's online softmax (m, l, acc) of its REP query heads.
template <int C, int REP>
__device__ __forceinline__ void attn_pass(const float (&q)[REP][16], const float (&kv)[16], const float (&vv)[16],
                                          bool act, float denom, float (&m)[REP], float (&l)[REP],
                                          float (&acc)[REP][16]) {
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) d = fmaf(q[j][i], kv[i], d);
#pragma unroll
    for (int o = 1; o < C; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (act) {
      const float sc = __fdiv_rn(d, denom);
      if (sc > m[j]) {
        const float c = expf(m[j] - sc);
        l[j] *= c;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[j][i] *= c;
        m[j] = sc;
      }
      const float p = expf(sc - m[j]);
      l[j] += p;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[j][i] = fmaf(p, vv[i], acc[j][i]);
    }
  }
}

__device__ __forceinline__ void unpack16(const float4 (&a)[4], float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[4 * i] = a[i].x; v[4 * i + 1] = a[i].y; v[4 * i + 2] = a[i].z; v[4 * i + 3] = a[i].w;
  }
}

// The lane groups' softmax states merged by shuffles (lanes holding the same
// kv head and dims: lane % R) and the REP output rows written by the first R
// lanes (as FP32 rows, or as three-part image units when SPLIT).
template <int HD, int KV, int REP, bool SPLIT>
__device__ __forceinline__ void attn_rows_finish(float (&m)[REP], float (&l)[REP], float (&acc)[REP][16], int b,
                                                 int lane, float* __restrict__ out, int ldo,
                                                 uint8_t* __restrict__ out_img) {
  constexpr int C = HD / 16;
  constexpr int R = KV * C;
  const int r = lane % R, kvh = r / C, chunk = r % C;
#pragma unroll
  for (int o = R; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < REP; ++j) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[j], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[j], o);
      const float mt = fmaxf(m[j], mo);
      const float ca = m[j] == -INFINITY ? 0.0f : expf(m[j] - mt);
      const float cb = mo == -INFINITY ? 0.0f : expf(mo - mt);
      l[j] = l[j] * ca + lo * cb;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[j][i], o);
        acc[j][i] = acc[j][i] * ca + ao * cb;
      }
      m[j] = mt;
    }
  }
  if (lane < R) {
#pragma unroll
    for (int j = 0; j < REP; ++j) {
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = __fdiv_rn(acc[j][i], l[j]);
      const int k0 = (kvh * REP + j) * HD + chunk * 16;
      if (SPLIT) {
        const float o0[8] = {o[0], o[1], o[2], o[3], o[4], o[5], o[6], o[7]};
        const float o1[8] = {o[8], o[9], o[10], o[11], o[12], o[13], o[14], o[15]};
        tc::img_store8(out_img, b, k0, KV * REP * HD, o0);
        tc::img_store8(out_img, b, k0 + 8, KV * REP * HD, o1);
      } else {
        float4* op = reinterpret_cast<float4*>(out + (int64_t)b * ldo + k0);
#pragma unroll
        for (int i = 0; i < 4; ++i) op[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      }
    }
  }
}

// One sequence's attention from its query rows (q) and the K/V rows of the
// first pass (kn, vn: row t_lane); kb / vb are this lane's cache columns at
// row 0.  Each pass requests the next pass's rows before it computes.
template <int HD, int KV, int REP, bool SPLIT, typename KT>
__device__ __forceinline__ void attn_rows_body(const float (&q)[REP][16], float4 (&kn)[4], float4 (&vn)[4],
                                               const KT* __restrict__ kb, const KT* __restrict__ vb, int T, int b,
                                               int lane, float denom, float* __restrict__ out, int ldo,
                                               uint8_t* __restrict__ out_img) {
  constexpr int C = HD / 16;
  constexpr int R = KV * C;
  constexpr int PPW = 32 / R;
  constexpr int ROW = KV * HD;
  const int t_lane = lane / R;
  float m[REP], l[REP], acc[REP][16];
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[j][i] = 0.0f;
  }
  for (int t0 = 0; t0 < T; t0 += PPW) {
    const int t = t0 + t_lane;
    float kv[16], vv[16];
    unpack16(kn, kv);
    unpack16(vn, vv);
    const int tn = t + PPW;
    if (tn < T) {
      load_kv16(kb + (int64_t)tn * ROW, kn);
      load_kv16(vb + (int64_t)tn * ROW, vn);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) kn[i] = vn[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    attn_pass<C, REP>(q, kv, vv, t < T, denom, m, l, acc);
  }
  attn_rows_finish<HD, KV, REP, SPLIT>(m, l, acc, b, lane, out, ldo, out_img);
}

// The same with the rows of two passes in flight: buffers A (even passes)
// and B (odd passes, first rows kn2 / vn2) alternate, each refilled with the
// rows two passes ahead when it is consumed.  Same positions per lane in the
// same order as attn_rows_body, so the same bits; more registers, so it is
// used when the batch leaves room on the SMs.
template <int HD, int KV, int REP, bool SPLIT, typename KT>
__device__ __forceinline__ void attn_rows_body2(const float (&q)[REP][16], float4 (&kn)[4], float4 (&vn)[4],
                                                float4 (&kn2)[4], float4 (&vn2)[4], const KT* __restrict__ kb,
                                                const KT* __restrict__ vb, int T, int b, int lane, float denom,
                                                float* __restrict__ out, int ldo, uint8_t* __restrict__ out_img) {
  constexpr int C = HD / 16;
  constexpr int R = KV * C;
  constexpr int PPW = 32 / R;
  constexpr int ROW = KV * HD;
  const int t_lane = lane / R;
  float m[REP], l[REP], acc[REP][16];
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[j][i] = 0.0f;
  }
  for (int t0 = 0; t0 < T; t0 += 2 * PPW) {
    {
      const int t = t0 + t_lane;
      float kv[16], vv[16];
      unpack16(kn, kv);
      unpack16(vn, vv);
      const int tn = t + 2 * PPW;
      if (tn < T) {
        load_kv16(kb + (int64_t)tn * ROW, kn);
        load_kv16(vb + (int64_t)tn * ROW, vn);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) kn[i] = vn[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      attn_pass<C, REP>(q, kv, vv, t < T, denom, m, l, acc);
    }
    if (t0 + PPW < T) {
      const int t = t0 + PPW + t_lane;
      float kv[16], vv[16];
      unpack16(kn2, kv);
      unpack16(vn2, vv);
      const int tn = t + 2 * PPW;
      if (tn < T) {
        load_kv16(kb + (int64_t)tn * ROW, kn2);
        load_kv16(vb + (int64_t)tn * ROW, vn2);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) kn2[i] = vn2[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      attn_pass<C, REP>(q, kv, vv, t < T, denom, m, l, acc);
    }
  }
  attn_rows_finish<HD, KV, REP, SPLIT>(m, l, acc, b, lane, out, ldo, out_img);
}

// Zeros for a sequence with nothing to attend (invalid, or no positions).
template <int HD, int KV, int REP, bool SPLIT>
__device__ __forceinline__ void attn_rows_zero(int b, int lane, float* __restrict__ out, int ldo,
                                               uint8_t* __restrict__ out_img) {
  if (SPLIT) {
    const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = lane * 8; k < KV * REP * HD; k += 256) tc::img_store8(out_img, b, k, KV * REP * HD, z);
  } else {
    for (int i = lane; i < KV * REP * HD; i += 32) out[(int64_t)b * ldo + i] = 0.0f;
  }
}

// DEEP: two passes of K/V rows in flight (attn_rows_body2) instead of one.
template <int HD, int KV, int REP, bool SPLIT, typename KT = float, bool DEEP = false>
__global__ void __launch_bounds__(128) attn_warp_kernel(
    const float* __restrict__ qb, int ldq, const KT* __restrict__ kc, const KT* __restrict__ vc,
    int64_t cstride, int64_t layer_off, const int32_t* __restrict__ len, int len_add,
    const int32_t* __restrict__ flags, float* __restrict__ out, int ldo, int S, float denom, int n,
    uint8_t* __restrict__ out_img, const int32_t* __restrict__ seq) {
  constexpr int C = HD / 16;
  constexpr int R = KV * C;
  constexpr int ROW = KV * HD;  // floats per cached row
  static_assert(32 % R == 0, "a row must map onto a power-of-two lane group");
  grid_dep_launch();
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= n) return;
  const int r = lane % R, kvh = r / C, chunk = r % C;
  const int t_lane = lane / R;
  // The length, the query and (when the cache row is the sequence's own) the
  // first pass's K/V rows are all requested before any of them is used: one
  // memory round trip instead of two.  Those rows lie inside the cache for
  // any length (t_lane < S) and are replaced by zeros below when past it.
  const int len_b = len[b];
  const int flag_b = flags ? flags[b] : 0;
  float q[REP][16];
#pragma unroll
  for (int j = 0; j < REP; ++j) {
    const float4* qp = reinterpret_cast<const float4*>(qb + (int64_t)b * ldq + (kvh * REP + j) * HD + chunk * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = qp[i];
      q[j][4 * i] = v.x; q[j][4 * i + 1] = v.y; q[j][4 * i + 2] = v.z; q[j][4 * i + 3] = v.w;
    }
  }
  const int64_t crow = seq ? seq[b] : b;
  const KT* kb = kc + crow * cstride + layer_off + r * 16;
  const KT* vb = vc + crow * cstride + layer_off + r * 16;
  constexpr int PPW = 32 / R;
  float4 kn[4], vn[4], kn2[4], vn2[4];
  const bool early = !seq && t_lane < S;
  const bool early2 = DEEP && !seq && t_lane + PPW < S;
  if (early) {
    load_kv16(kb + (int64_t)t_lane * ROW, kn);
    load_kv16(vb + (int64_t)t_lane * ROW, vn);
  }
  if (early2) {
    load_kv16(kb + (int64_t)(t_lane + PPW) * ROW, kn2);
    load_kv16(vb + (int64_t)(t_lane + PPW) * ROW, vn2);
  }
  int T = len_b + len_add;
  T = T > S ? S : T;
  if ((flag_b & SEQ_INVALID) || T <= 0) {
    attn_rows_zero<HD, KV, REP, SPLIT>(b, lane, out, ldo, out_img);
    return;
  }
  if (t_lane < T) {
    if (!early) {
      load_kv16(kb + (int64_t)t_lane * ROW, kn);
      load_kv16(vb + (int64_t)t_lane * ROW, vn);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) kn[i] = vn[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (DEEP) {
    if (t_lane + PPW < T) {
      if (!early2) {
        load_kv16(kb + (int64_t)(t_lane + PPW) * ROW, kn2);
        load_kv16(vb + (int64_t)(t_lane + PPW) * ROW, vn2);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) kn2[i] = vn2[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    attn_rows_body2<HD, KV, REP, SPLIT, KT>(q, kn, vn, kn2, vn2, kb, vb, T, b, lane, denom, out, ldo, out_img);
  } else {
    attn_rows_body<HD, KV, REP, SPLIT, KT>(q, kn, vn, kb, vb, T, b, lane, denom, out, ldo, out_img);
  }
}

// Causal attention of the token rows of a batched prefill (rows of prompt p
// are off[p] .. off[p] + len[p] - 1, row j at position j; torch_benchmark.py's
// per-position step over the prompt, :263-264).  A CTA takes one prompt, one
// KV head and a block of kRB query rows; the keys its rows need (positions
// 0 .. last row) pass through shared memory once, in tiles of kPT positions,
// instead of once per row.  Thread = (query row, q head of the group): q and
// the output accumulator in registers, keys read as shared-memory broadcasts.
// Per key: the dot product as two FP32x2 FMA chains over dimension pairs
// (no register repacking: q and the key rows are read as aligned pairs), score
// = dot / denom, online softmax with expf, the accumulator updated with
// FP32x2 FMAs, output acc / l.  Keys go in position order; results agree
// with the decode path (whose dot is one FMA chain per 16 dimensions and whose
// keys are split over lane groups) to rounding.
constexpr int kPromptThreads = 128;
constexpr int kPT = 64;  // key positions per shared-memory tile

template <int HD, int REP, bool SPLIT, typename KT = float>
__global__ void __launch_bounds__(kPromptThreads) attn_prompt_kernel(
    const float* __restrict__ qb, int ldq, const KT* __restrict__ kc, const KT* __restrict__ vc, int64_t cstride,
    int64_t layer_off, const int32_t* __restrict__ off, const int32_t* __restrict__ lens, int max_len, int KV,
    int64_t rows, const int32_t* __restrict__ flags, float denom, float* __restrict__ out, int ldo,
    uint8_t* __restrict__ out_img) {
  constexpr int kRB = kPromptThreads / REP;  // query rows per CTA
  __shared__ __align__(16) float sk[kPT * HD];
  __shared__ __align__(16) float sv[kPT * HD];
  grid_dep_launch();
  grid_dep_wait();
  const int blocks = (max_len + kRB - 1) / kRB;
  const int p = blockIdx.x / blocks, r0 = (blockIdx.x % blocks) * kRB;
  const int g = blockIdx.y;
  const int L = lens[p];
  if (L < 1 || L > max_len || r0 >= L) return;  // block-uniform
  const int j = threadIdx.x / kRB;
  const int i = r0 + threadIdx.x % kRB;  // position of this thread's query row
  const int64_t row = (int64_t)off[p] + i;
  const bool inside = i < L && row < rows;  // a total shorter than the lengths (flagged) ends the rows
  const bool act = inside && !(flags[row] & SEQ_INVALID);
  const int K = KV * REP * HD;
  const int h = g * REP + j;
  float2 q2[HD / 2];
#pragma unroll
  for (int c = 0; c < HD / 2; ++c) q2[c] = make_float2(0.0f, 0.0f);
  if (act) {
    const float4* qp = reinterpret_cast<const float4*>(qb + row * ldq + h * HD);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) {
      const float4 v = qp[c];
      q2[2 * c] = make_float2(v.x, v.y);
      q2[2 * c + 1] = make_float2(v.z, v.w);
    }
  }
  float2 acc[HD / 2];
#pragma unroll
  for (int c = 0; c < HD / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);
  float m = -INFINITY, l = 0.0f;
  const bool pow2 = denom > 0.0f && __float_as_uint(denom) << 9 == 0u;  // x / 2^e == x * 2^-e exactly
  const float inv = pow2 ? 1.0f / denom : 0.0f;
  const int kend = min(L, r0 + kRB);  // keys the block needs
  const int64_t ROW = (int64_t)KV * HD;
  const KT* kb = kc + (int64_t)p * cstride + layer_off + g * HD;
  const KT* vb = vc + (int64_t)p * cstride + layer_off + g * HD;
  for (int t0 = 0; t0 < kend; t0 += kPT) {
    const int tn = min(kPT, kend - t0);
    __syncthreads();  // the previous tile is consumed
    for (int e = threadIdx.x; e < tn * (HD / 4); e += kPromptThreads) {
      const int t = e / (HD / 4), c4 = e % (HD / 4);
      reinterpret_cast<float4*>(sk)[e] = load_kv4(kb + (t0 + t) * ROW + 4 * c4);
      reinterpret_cast<float4*>(sv)[e] = load_kv4(vb + (t0 + t) * ROW + 4 * c4);
    }
    __syncthreads();
    const int mine = act ? min(tn, i + 1 - t0) : 0;  // keys <= i in this tile
    for (int tt = 0; tt < mine; ++tt) {
      // q.k over dimension pairs: two FP32x2 FMA chains (dims 4c, 4c+1 and 4c+2, 4c+3), then their lanes added
      const float* kr = sk + tt * HD;
      float2 da = make_float2(0.0f, 0.0f), db = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) {
        const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * c);
        da = __ffma2_rn(q2[2 * c], make_float2(k4.x, k4.y), da);
        db = __ffma2_rn(q2[2 * c + 1], make_float2(k4.z, k4.w), db);
      }
      const float2 d = __fadd2_rn(da, db);
      const float dot = __fadd_rn(d.x, d.y);
      const float sc = pow2 ? dot * inv : __fdiv_rn(dot, denom);
      if (sc > m) {
        const float cf = expf(m - sc);
        l *= cf;
#pragma unroll
        for (int c = 0; c < HD / 2; ++c) acc[c] = __fmul2_rn(acc[c], make_float2(cf, cf));
        m = sc;
      }
      const float pr = expf(sc - m);
      l += pr;
      const float2 p2 = make_float2(pr, pr);
      const float* vr = sv + tt * HD;
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) {
        const float4 v = *reinterpret_cast<const float4*>(vr + 4 * c);
        acc[2 * c] = __ffma2_rn(p2, make_float2(v.x, v.y), acc[2 * c]);
        acc[2 * c + 1] = __ffma2_rn(p2, make_float2(v.z, v.w), acc[2 * c + 1]);
      }
    }
  }
  if (!inside) return;
  float o[HD];
#pragma unroll
  for (int c = 0; c < HD / 2; ++c) {
    o[2 * c] = act ? __fdiv_rn(acc[c].x, l) : 0.0f;
    o[2 * c + 1] = act ? __fdiv_rn(acc[c].y, l) : 0.0f;
  }
  if (SPLIT) {
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
      const float o8[8] = {o[8 * c], o[8 * c + 1], o[8 * c + 2], o[8 * c + 3],
                           o[8 * c + 4], o[8 * c + 5], o[8 * c + 6], o[8 * c + 7]};
      tc::img_store8(out_img, row, h * HD + 8 * c, K, o8);
    }
  } else {
    float4* op = reinterpret_cast<float4*>(out + row * ldo + h * HD);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) op[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
  }
}

// The per-sequence kernel for one instantiation.
template <int HD, int KV, int REP, bool SPLIT, typename KT>
static void launch_rows(int n, cudaStream_t st, bool pdl, bool deep, const float* qb, int ldq, const KT* kc,
                        const KT* vc, int64_t cstride, int64_t layer_off, const int32_t* len, int len_add,
                        const int32_t* flags, float* out, int ldo, int S, float denom, uint8_t* out_img,
                        const int32_t* seq) {
  if (deep)
    (void)launch_k(attn_warp_kernel<HD, KV, REP, SPLIT, KT, true>, dim3((n + 3) / 4), dim3(128), 0, st, pdl, qb,
                   ldq, kc, vc, cstride, layer_off, len, len_add, flags, out, ldo, S, denom, n, out_img, seq);
  else
    (void)launch_k(attn_warp_kernel<HD, KV, REP, SPLIT, KT>, dim3((n + 3) / 4), dim3(128), 0, st, pdl, qb, ldq,
                   kc, vc, cstride, layer_off, len, len_add, flags, out, ldo, S, denom, n, out_img, seq);
}

// Launch the streaming kernel when the shape has an instantiation; returns
// false to fall back to the per-head kernel.
static bool launch_attn_rows(int hd, int KV, int rep, dim3 grid, cudaStream_t st, const float* qb, int ldq,
                             const void* kc, const void* vc, int64_t cstride, int64_t layer_off,
                             const int32_t* len, int len_add, const int32_t* flags, float* out, int ldo,
                             int S, float denom, uint8_t* out_img = nullptr, const int32_t* seq = nullptr,
                             bool kv_half = false, bool pdl = false, bool deep = false) {
  // a launch error is left for the caller's launch check (cudaGetLastError)
  const float* kf = static_cast<const float*>(kc);
  const float* vf = static_cast<const float*>(vc);
  const __half* kh = static_cast<const __half*>(kc);
  const __half* vh = static_cast<const __half*>(vc);
#define Q6W_ROWS(HDV, KVV, REPV)                                                                           \
  if (hd == HDV && KV == KVV && rep == REPV) {                                                             \
    const int n = (int)grid.x;                                                                             \
    if (kv_half && out_img)                                                                                \
      launch_rows<HDV, KVV, REPV, true, __half>(n, st, pdl, deep, qb, ldq, kh, vh, cstride, layer_off, len,      \
                                                len_add, flags, out, ldo, S, denom, out_img, seq);         \
    else if (kv_half)                                                                                      \
      launch_rows<HDV, KVV, REPV, false, __half>(n, st, pdl, deep, qb, ldq, kh, vh, cstride, layer_off, len,     \
                                                 len_add, flags, out, ldo, S, denom, nullptr, seq);        \
    else if (out_img)                                                                                      \
      launch_rows<HDV, KVV, REPV, true, float>(n, st, pdl, deep, qb, ldq, kf, vf, cstride, layer_off, len,       \
                                               len_add, flags, out, ldo, S, denom, out_img, seq);          \
    else                                                                                                   \
      launch_rows<HDV, KVV, REPV, false, float>(n, st, pdl, deep, qb, ldq, kf, vf, cstride, layer_off, len,      \
                                                len_add, flags, out, ldo, S, denom, nullptr, seq);         \
    return true;                                                                                           \
  }
  Q6W_ROWS(16, 1, 1) Q6W_ROWS(16, 2, 1) Q6W_ROWS(16, 4, 1) Q6W_ROWS(16, 8, 1)
  Q6W_ROWS(16, 1, 2) Q6W_ROWS(16, 2, 2) Q6W_ROWS(16, 4, 2) Q6W_ROWS(16, 8, 2)
  Q6W_ROWS(16, 1, 4) Q6W_ROWS(16, 2, 4) Q6W_ROWS(16, 4, 4) Q6W_ROWS(16, 8, 4)
  Q6W_ROWS(32, 1, 1) Q6W_ROWS(32, 2, 1) Q6W_ROWS(32, 4, 1)
  Q6W_ROWS(32, 1, 2) Q6W_ROWS(32, 2, 2) Q6W_ROWS(32, 4, 2)
  Q6W_ROWS(32, 1, 4) Q6W_ROWS(32, 2, 4) Q6W_ROWS(32, 4, 4)
#undef Q6W_ROWS
  return false;
}

// The prefill's causal attention (attn_prompt_kernel) when the head layout has
// an instantiation; returns false to fall back to the per-row kernels.
static bool launch_attn_prompt(int hd, int KV, int rep, int n_prompts, int max_len, int64_t rows, cudaStream_t st,
                               const float* qb, int ldq, const void* kc, const void* vc, int64_t cstride,
                               int64_t layer_off, const int32_t* off, const int32_t* lens, const int32_t* flags,
                               float denom, float* out, int ldo, uint8_t* out_img, bool kv_half,
                               bool pdl = false) {
  // a launch error is left for the caller's launch check (cudaGetLastError)
  const float* kf = static_cast<const float*>(kc);
  const float* vf = static_cast<const float*>(vc);
  const __half* kh = static_cast<const __half*>(kc);
  const __half* vh = static_cast<const __half*>(vc);
#define Q6W_PROMPT(HDV, REPV)                                                                               \
  if (hd == HDV && rep == REPV) {                                                                           \
    constexpr int rb = kPromptThreads / REPV;                                                               \
    const dim3 grid((unsigned)((int64_t)n_prompts * ((max_len + rb - 1) / rb)), (unsigned)KV);              \
    const dim3 bl(kPromptThreads);                                                                          \
    if (kv_half && out_img)                                                                                 \
      (void)launch_k(attn_prompt_kernel<HDV, REPV, true, __half>, grid, bl, 0, st, pdl, qb, ldq, kh, vh,      \
                   cstride, layer_off, off, lens, max_len, KV, rows, flags, denom, out, ldo, out_img);      \
    else if (kv_half)                                                                                       \
      (void)launch_k(attn_prompt_kernel<HDV, REPV, false, __half>, grid, bl, 0, st, pdl, qb, ldq, kh, vh,     \
                   cstride, layer_off, off, lens, max_len, KV, rows, flags, denom, out, ldo,                \
                   (uint8_t*)nullptr);                                                                      \
    else if (out_img)                                                                                       \
      (void)launch_k(attn_prompt_kernel<HDV, REPV, true>, grid, bl, 0, st, pdl, qb, ldq, kf, vf, cstride,     \
                   layer_off, off, lens, max_len, KV, rows, flags, denom, out, ldo, out_img);               \
    else                                                                                                    \
      (void)launch_k(attn_prompt_kernel<HDV, REPV, false>, grid, bl, 0, st, pdl, qb, ldq, kf, vf, cstride,    \
                   layer_off, off, lens, max_len, KV, rows, flags, denom, out, ldo, (uint8_t*)nullptr);     \
    return true;                                                                                            \
  }
  Q6W_PROMPT(16, 1) Q6W_PROMPT(16, 2) Q6W_PROMPT(16, 4) Q6W_PROMPT(32, 1) Q6W_PROMPT(32, 2) Q6W_PROMPT(32, 4)
#undef Q6W_PROMPT
  return false;
}

struct StopSet {
  int32_t n, min_new;
  int32_t ids[kMaxStop];
};

// Greedy control for one step (torch_benchmark.py:272-293 at temperature 0,
// prepare_e2e.py:129-143): consume the argmax key, record the pick, stop on
// a stop id once min_new_tokens exist, otherwise feed the next token.
__global__ void advance_kernel(int n, Work w, const int32_t* __restrict__ prompts, int32_t stride,
                               int32_t new_tokens, StopSet stop, int32_t* sampled,
                               int32_t* n_sampled, int32_t* stop_reason) {
  grid_dep_launch();
  grid_dep_wait();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n; b += gridDim.x * blockDim.x) {
    const unsigned long long key = w.keys[b];
    w.keys[b] = 0ull;
    const int f = w.flags[b];
    if (f & (SEQ_DONE | SEQ_INVALID)) {
      w.flags[b] = f | SEQ_DONE;
      continue;
    }
    const int p = w.pos[b], L = w.plen[b];
    if (p < L - 1) {  // still inside the prompt
      w.tok[b] = prompts[(int64_t)b * stride + p + 1];
      w.pos[b] = p + 1;
      continue;
    }
    const int g = w.gen[b];
    const int t = argmax_index(key);
    sampled[(int64_t)b * new_tokens + g] = t;
    n_sampled[b] = g + 1;
    bool is_stop = false;
    for (int i = 0; i < stop.n; ++i) is_stop |= (stop.ids[i] == t);
    if (is_stop && g >= stop.min_new) {
      stop_reason[b] = t;
      w.flags[b] = f | SEQ_DONE;
      continue;
    }
    w.gen[b] = g + 1;
    if (g + 1 >= new_tokens) {
      w.flags[b] = f | SEQ_DONE;
      continue;
    }
    w.tok[b] = t;
    w.pos[b] = p + 1;
  }
}

__global__ void keys_to_argmax_kernel(int n, unsigned long long* keys, int32_t* argmax) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n; b += gridDim.x * blockDim.x) {
    argmax[b] = argmax_index(keys[b]);
    keys[b] = 0ull;
  }
}

// ---- step enqueue --------------------------------------------------------------

// Whether the decode attention of a step over n sequences keeps two passes of
// K/V rows in flight per warp (202 registers: 8 warps an SM) instead of one
// (152: 12 warps).  Measured on the tiny model (a generation of 128 tokens):
// 1024 sequences 35.9 -> 35.2 ms, 2048 48.3 -> 47.4 ms, 512 unchanged, 8192
// 107.2 -> 114.3 ms; so by default up to 16 sequences an SM (two waves of the
// deeper kernel).
static bool attn_deep(const q6w_model* M, int n) {
  if (M->attn_deep_mode >= 0) return M->attn_deep_mode == 1;
  return (int64_t)n <= 16LL * M->sm_count;
}

static int32_t enqueue_step_tc(const q6w_model* M, int n, const Work& w, float* kc, float* vc, int64_t cstride,
                               const EpiArgs& vocab_ep, cudaStream_t st, bool with_vocab);
static int tc_min_seqs();
static int tcg_min_rows();
static int32_t enqueue_step_tcg(const q6w_model* M, int n, const Work& w, float* kc, float* vc, int64_t cstride,
                                const EpiArgs& vocab_ep, cudaStream_t st, bool with_vocab);
static int32_t enqueue_step_pdec(const q6w_model* M, const Work& w, float* kc, float* vc, const EpiArgs& vocab_ep,
                                 cudaStream_t st);

// One model step for n activation rows: embedding, the layers, and (unless
// with_vocab is false) the vocab projection + argmax of every row.
static int32_t enqueue_step(const q6w_model* M, int n, const Work& w, float* kc, float* vc,
                            int64_t cstride, const EpiArgs& vocab_ep, cudaStream_t st, bool with_vocab = true) {
  if (n == 1 && M->use_pdec && with_vocab && !w.seq) return enqueue_step_pdec(M, w, kc, vc, vocab_ep, st);
  if (M->use_tc && n >= tc_min_seqs()) return enqueue_step_tc(M, n, w, kc, vc, cstride, vocab_ep, st, with_vocab);
  if (M->use_tcg && n >= tcg_min_rows()) return enqueue_step_tcg(M, n, w, kc, vc, cstride, vocab_ep, st, with_vocab);
  const q6w_model_desc& d = M->d;
  const int dim = d.dim, kvr = M->kv_rows, hid = d.hidden_dim, S = d.max_seq_len;
  embed_kernel<<<n < 2048 ? n : 2048, 128, 0, st>>>(d.tok_embeddings.packed,
                                                    d.tok_embeddings.scales, dim, d.vocab_size, S,
                                                    n, w);
  Q6W_LAUNCH_CHECK("embed_kernel");
  EpiArgs ep;
  memset(&ep, 0, sizeof(ep));
  ep.pos = w.pos;
  ep.flags = w.flags;
  ep.seq = w.seq;
  ep.kv_half = M->kv_half;
  const int warps = d.n_heads < 8 ? d.n_heads : 8;
  const dim3 agrid(n, (d.n_heads + warps - 1) / warps);
  const size_t asmem = (size_t)warps * S * sizeof(float);
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    const int64_t layer_off = (int64_t)l * S * kvr;
    cudaError_t e;
    {
      MatSet ms = {L.wq.packed, L.wk.packed, L.wv.packed, L.wq.scales, L.wk.scales, L.wv.scales,
                   dim, dim + kvr, dim, 0, (dim + 2 * kvr) / 2};
      EpiArgs q = ep;
      q.qbuf = w.qb;
      q.ldq = dim;
      q.kc = kc;
      q.vc = vc;
      q.cache_stride = cstride;
      q.layer_off = layer_off;
      q.rope_cos = d.rope_cos;
      q.rope_sin = d.rope_sin;
      q.hd = M->hd;
      q.q_rows = dim;
      q.kv_rows = kvr;
      e = LinearLauncher<true, EPI_QKV>::run(w.x, dim, n, L.attention_norm, d.norm_eps, ms, q, st);
      if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "qkv linear: %s", cudaGetErrorString(e));
    }
    if (w.poff && launch_attn_prompt(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, w.n_prompts, w.max_len, n, st,
                                     w.qb, dim, kc, vc, cstride, layer_off, w.poff, w.plens, w.flags, M->denom,
                                     w.att, dim, nullptr, M->kv_half)) {
      Q6W_LAUNCH_CHECK("attn_prompt_kernel");
    } else if (launch_attn_rows(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, agrid, st, w.qb, dim, kc, vc,
                                cstride, layer_off, w.pos, 1, w.flags, w.att, dim, S, M->denom, nullptr, w.seq,
                                M->kv_half, false, attn_deep(M, n))) {
      Q6W_LAUNCH_CHECK("attn_rows_kernel");
    } else if (launch_attn_head(M->hd, n, d.n_heads, d.n_kv_heads, st, w.qb, dim, kc, vc, cstride, layer_off,
                                w.pos, 1, w.flags, w.att, dim, S, M->denom, w.seq, M->kv_half)) {
      Q6W_LAUNCH_CHECK("attn_head_kernel");
    } else if (M->kv_half) {
      return fail(Q6W_ERR_ARG, "no FP16-KV attention kernel for this head layout");
    } else {
    switch (M->hd) {
#define Q6W_ATTN(HDV)                                                                          \
  case HDV:                                                                                    \
    attn_kernel<HDV / 16><<<agrid, warps * 32, asmem, st>>>(w.qb, dim, kc, vc, cstride,        \
                                                            layer_off, w.pos, 1, w.flags, w.att, \
                                                            dim, d.n_heads, d.n_kv_heads, S,   \
                                                            M->denom, w.seq);                  \
    break;
      Q6W_ATTN(16) Q6W_ATTN(32) Q6W_ATTN(64) Q6W_ATTN(128) Q6W_ATTN(256) Q6W_ATTN(512)
#undef Q6W_ATTN
      default:
        return fail(Q6W_ERR_ARG, "unsupported head_dim %d", M->hd);
    }
    Q6W_LAUNCH_CHECK("attn_kernel");
    }
    {
      MatSet ms = {L.wo.packed, nullptr, nullptr, L.wo.scales, nullptr, nullptr,
                   dim, dim, dim, 0, dim / 2};
      EpiArgs r = ep;
      r.y = w.x;
      r.ldy = dim;
      e = LinearLauncher<false, EPI_RESID>::run(w.att, dim, n, nullptr, 0.f, ms, r, st);
      if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "wo linear: %s", cudaGetErrorString(e));
    }
    {
      MatSet ms = {L.w1.packed, L.w3.packed, nullptr, L.w1.scales, L.w3.scales, nullptr,
                   hid, hid, dim, 1, hid};
      EpiArgs gl = ep;
      gl.y = w.hb;
      gl.ldy = hid;
      e = LinearLauncher<true, EPI_GLU>::run(w.x, dim, n, L.ffn_norm, d.norm_eps, ms, gl, st);
      if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "w1/w3 linear: %s", cudaGetErrorString(e));
    }
    {
      MatSet ms = {L.w2.packed, nullptr, nullptr, L.w2.scales, nullptr, nullptr,
                   dim, dim, hid, 0, dim / 2};
      EpiArgs r = ep;
      r.y = w.x;
      r.ldy = dim;
      e = LinearLauncher<false, EPI_RESID>::run(w.hb, hid, n, nullptr, 0.f, ms, r, st);
      if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "w2 linear: %s", cudaGetErrorString(e));
    }
  }
  if (!with_vocab) return Q6W_OK;
  MatSet mv = {d.tok_embeddings.packed, nullptr, nullptr, d.tok_embeddings.scales, nullptr, nullptr,
               d.vocab_size, d.vocab_size, dim, 0, d.vocab_size / 2};
  EpiArgs v = vocab_ep;
  v.pos = w.pos;
  v.flags = w.flags;
  v.keys = w.keys;
  v.gen = w.gen;
  v.plen = w.plen;
  v.vocab = d.vocab_size;
  cudaError_t e = LinearLauncher<true, EPI_VOCAB>::run(w.x, dim, n, d.norm, d.norm_eps, mv, v, st);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "vocab linear: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

// Tensor-core path: x[b] = dequant(E[token]) and the layer-0 activation image
// of RMSNorm(x) * attention_norm[0] (torch_benchmark.py:97, 104).  Sixteen
// lanes per sequence, eight values each (dim 128).
__global__ void embed_tc_kernel(const uint8_t* __restrict__ E, const float* __restrict__ Es, int vocab,
                                int max_seq, int n, Work w, const float* __restrict__ g, float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const int gl = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = gl >> 4, l = gl & 15;
  const bool inb = b < n;
  const int t = inb ? w.tok[b] : 0, p = inb ? w.pos[b] : 0;
  const bool ok = inb && t >= 0 && t < vocab && p >= 0 && p < max_seq;
  if (inb && l == 0) {
    const int f = w.flags[b];
    w.flags[b] = ok ? (f & ~SEQ_INVALID) : (f | SEQ_INVALID);
    if (!ok && !(f & SEQ_DONE)) atomicOr(w.err, 1);
  }
  float v[8];
  if (ok) {
    const uint8_t* row = E + (int64_t)t * 96 + l * 6;
    const float s = __ldg(Es + t);
    const uint32_t g0 = load_group(row), g1 = load_group(row + 3);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __fmul_rn((float)group_code(g0, i), s);
      v[4 + i] = __fmul_rn((float)group_code(g1, i), s);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!inb) return;
  float4* xr = reinterpret_cast<float4*>(w.x + (int64_t)b * 128 + l * 8);
  xr[0] = make_float4(v[0], v[1], v[2], v[3]);
  xr[1] = make_float4(v[4], v[5], v[6], v[7]);
  const float r = rms_scale(ss, 128, eps);
  float u[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) u[i] = __fmul_rn(__fmul_rn(v[i], r), __ldg(g + l * 8 + i));
  tc::img_store8(w.xs_img, b, l * 8, 128, u);
}

static int32_t tc_launch(int epi, const tc::TcArgs& a, int sms, cudaStream_t st, bool pdl = false) {
  const int items = ((a.n + tc::kM - 1) / tc::kM) * a.n_tiles;
  const int grid = items < sms ? items : sms;
  const size_t smem = tc::smem_bytes_for(epi);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(tc::threads_for(epi));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cudaError_t e;
  if (epi == tc::TEPI_RESNORM && a.pair) {
    // one item per CTA, the column blocks of an M tile in one cluster
    cfg.gridDim = dim3((unsigned)items);
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)a.pair;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
    cfg.numAttrs = na;
    e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_RESNORM>, a);
  } else {
    cfg.numAttrs = na;
    switch (epi) {
      case tc::TEPI_QKV: e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_QKV>, a); break;
      case tc::TEPI_RESNORM: e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_RESNORM>, a); break;
      case tc::TEPI_GLU: e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_GLU>, a); break;
      case tc::TEPI_STORE: e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_STORE>, a); break;
      default: e = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::TEPI_VOCAB>, a); break;
    }
  }
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "tc_gemm_kernel launch: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

// RESNORM tiles (dim 128): the 128 columns of an M tile split into P blocks
// of 128 / P columns, one CTA each, in one P-CTA cluster (P times the CTAs,
// 1/P of the epilogue each), with P = 4 when every M tile can have four CTAs
// at once (up to 37 tiles, 4736 sequences), else 2 when it can have two;
// otherwise one CTA takes all 128 columns.
static void tc_resnorm_tiles(tc::TcArgs& a, int n, int sms) {
  const int m_tiles = (n + tc::kM - 1) / tc::kM;
  const int P = 4 * m_tiles <= sms ? 4 : 2 * m_tiles <= sms ? 2 : 1;
  a.N = 128 / P;
  a.n_tiles = P;
  a.pair = P > 1 ? P : 0;
}

// Rows per N tile of the QKV and SwiGLU linears.  Few M tiles (a small
// batch) leave most SMs idle at the default tiles, so the tiles narrow to 64
// rows (QKV) or 32 W1 + 32 W3 rows (SwiGLU) while the items still fit one
// CTA each on the SMs; each item's epilogue is then half as long.
static int tc_qkv_rows_per_tile(int n, int qkv_rows, int sms) {
  const int m_tiles = (n + tc::kM - 1) / tc::kM;
  if (m_tiles * (qkv_rows / 64) <= sms) return 64;
  return qkv_rows % 128 == 0 ? 128 : qkv_rows;
}
static int tc_glu_rows_per_tile(int n, int hid, int sms) {
  const int m_tiles = (n + tc::kM - 1) / tc::kM;
  return m_tiles * (hid / 32) <= sms ? 64 : 128;
}

static int32_t tc_set_attrs() {
  const int smem = (int)tc::smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::TEPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::TEPI_RESNORM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tc::smem_bytes_for(tc::TEPI_RESNORM));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::TEPI_GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::TEPI_VOCAB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::TEPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "tensor-core kernel attributes: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

// The batched step on tensor cores (same kernels sequence and semantics as
// enqueue_step; RMSNorm moves from the linear prologues into the epilogues
// that produce each linear's input).
static int32_t enqueue_step_tc(const q6w_model* M, int n, const Work& w, float* kc, float* vc, int64_t cstride,
                               const EpiArgs& vocab_ep, cudaStream_t st, bool with_vocab) {
  const q6w_model_desc& d = M->d;
  const int dim = d.dim, kvr = M->kv_rows, hid = d.hidden_dim, S = d.max_seq_len;
  cudaError_t le = launch_k(embed_tc_kernel, dim3((n * 16 + 127) / 128), dim3(128), 0, st, w.pdl,
                            d.tok_embeddings.packed, d.tok_embeddings.scales, d.vocab_size, S, n, w,
                            M->layers[0].attention_norm, d.norm_eps);
  if (le != cudaSuccess) return fail(Q6W_ERR_CUDA, "embed_tc_kernel launch: %s", cudaGetErrorString(le));
  tc::TcArgs base;
  memset(&base, 0, sizeof(base));
  base.n = n;
  base.err = w.err;
  base.eps = d.norm_eps;
  base.ep.pos = w.pos;
  base.ep.flags = w.flags;
  base.ep.seq = w.seq;
  base.ep.kv_half = M->kv_half;
  int32_t rc;
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    const int64_t layer_off = (int64_t)l * S * kvr;
    {
      tc::TcArgs a = base;
      a.a_img = w.xs_img;
      a.K = dim;
      a.q0 = L.wq.packed; a.q1 = L.wk.packed; a.q2 = L.wv.packed;
      a.s0 = L.wq.scales; a.s1 = L.wk.scales; a.s2 = L.wv.scales;
      a.end0 = dim; a.end1 = dim + kvr;
      // two tiles of 128 rows (q | k v) give twice the CTAs when the rows
      // divide; tiles of 64 rows at small batches
      const int qkv_rows = dim + 2 * kvr;
      a.N = tc_qkv_rows_per_tile(n, qkv_rows, M->sm_count);
      a.n_tiles = qkv_rows / a.N;
      a.ep.qbuf = w.qb; a.ep.ldq = dim;
      a.ep.kc = kc; a.ep.vc = vc; a.ep.cache_stride = cstride; a.ep.layer_off = layer_off;
      a.ep.rope_cos = d.rope_cos; a.ep.rope_sin = d.rope_sin;
      a.ep.hd = M->hd; a.ep.q_rows = dim; a.ep.kv_rows = kvr;
      if ((rc = tc_launch(tc::TEPI_QKV, a, M->sm_count, st, w.pdl))) return rc;
    }
    if (w.poff && launch_attn_prompt(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, w.n_prompts, w.max_len, n, st,
                                     w.qb, dim, kc, vc, cstride, layer_off, w.poff, w.plens, w.flags, M->denom,
                                     nullptr, dim, w.att_img, M->kv_half, w.pdl)) {
      Q6W_LAUNCH_CHECK("attn_prompt_kernel");
    } else {
      if (!launch_attn_rows(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, dim3(n), st, w.qb, dim, kc, vc,
                            cstride, layer_off, w.pos, 1, w.flags, nullptr, dim, S, M->denom, w.att_img, w.seq,
                            M->kv_half, w.pdl, attn_deep(M, n)))
        return fail(Q6W_ERR_ARG, "no attention kernel for this head layout");
      Q6W_LAUNCH_CHECK("attn_rows_kernel");
    }
    {
      tc::TcArgs a = base;
      a.a_img = w.att_img;
      a.K = dim;
      a.q0 = L.wo.packed; a.s0 = L.wo.scales;
      a.end0 = a.end1 = dim;
      tc_resnorm_tiles(a, n, M->sm_count);
      a.x = w.x; a.gnorm = L.ffn_norm; a.out_img = w.xs_img; a.out_K = dim;
      if ((rc = tc_launch(tc::TEPI_RESNORM, a, M->sm_count, st, w.pdl))) return rc;
    }
    {
      tc::TcArgs a = base;
      a.a_img = w.xs_img;
      a.K = dim;
      a.q0 = L.w1.packed; a.s0 = L.w1.scales; a.q1 = L.w3.packed; a.s1 = L.w3.scales;
      // tiles of 64 W1 + 64 W3 rows (32 + 32 at small batches): more, smaller
      // items spread over the SMs (each CTA keeps its activation tile across
      // consecutive items)
      a.N = tc_glu_rows_per_tile(n, hid, M->sm_count);
      a.n_tiles = hid / (a.N / 2);
      a.out_img = w.hs_img; a.out_K = hid;
      if ((rc = tc_launch(tc::TEPI_GLU, a, M->sm_count, st, w.pdl))) return rc;
    }
    {
      tc::TcArgs a = base;
      a.a_img = w.hs_img;
      a.K = hid;
      a.q0 = L.w2.packed; a.s0 = L.w2.scales;
      a.end0 = a.end1 = dim;
      tc_resnorm_tiles(a, n, M->sm_count);
      a.x = w.x;
      a.gnorm = l + 1 < d.n_layers ? M->layers[l + 1].attention_norm : d.norm;
      a.out_img = w.xs_img; a.out_K = dim;
      if ((rc = tc_launch(tc::TEPI_RESNORM, a, M->sm_count, st, w.pdl))) return rc;
    }
  }
  if (!with_vocab) return Q6W_OK;
  tc::TcArgs a = base;
  a.a_img = w.xs_img;
  a.K = dim;
  a.q0 = d.tok_embeddings.packed; a.s0 = d.tok_embeddings.scales;
  a.end0 = a.end1 = d.vocab_size;
  a.N = 256;
  a.n_tiles = d.vocab_size / 256;
  a.ep = vocab_ep;
  a.ep.pos = w.pos;
  a.ep.flags = w.flags;
  a.ep.keys = w.keys;
  a.ep.gen = w.gen;
  a.ep.plen = w.plen;
  a.ep.vocab = d.vocab_size;
  return tc_launch(tc::TEPI_VOCAB, a, M->sm_count, st, w.pdl);
}

// ---- batched prefill: rows are prompt tokens --------------------------------

// Row offset of every prompt (exclusive prefix sum of the lengths) and the
// total, by one CTA; a length outside [1, max_len] counts as 0 and is flagged.
__global__ void prefill_scan_kernel(int n, const int32_t* __restrict__ lens, int max_len, int32_t* __restrict__ off,
                                    int32_t* err) {
  __shared__ int64_t carry;
  __shared__ int32_t part[32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int v = 0;
    if (i < n) {
      v = lens[i];
      if (v < 1 || v > max_len) {
        atomicOr(err, 1);
        v = 0;
      }
    }
    int x = v;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) part[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int t = lane < (int)(blockDim.x >> 5) ? part[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      part[lane] = t;
    }
    __syncthreads();
    const int64_t before = carry + (warp ? part[warp - 1] : 0) + x - v;
    if (i < n) off[i] = (int32_t)(before > 0x7fffffff ? 0x7fffffff : before);
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) off[n] = (int32_t)(carry > 0x7fffffff ? 0x7fffffff : carry);
}

// Token rows: row off[i] + j is token j of prompt i (cache row i, position j).
// The prompts cover rows [0, off[n]) exactly once; rows from off[n] on (a
// total that does not match the lengths) stay invalid and write nothing.
__global__ void prefill_rows_kernel(int n, int rows, const int32_t* __restrict__ prompts, int stride,
                                    const int32_t* __restrict__ lens, int max_len, int vocab,
                                    const int32_t* __restrict__ off, Work w, int32_t* seq) {
  const int covered = off[n] < rows ? off[n] : rows;
  if (off[n] != rows && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(w.err, 1);
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = covered + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += nthreads) {
    w.flags[r] = SEQ_INVALID;
    w.tok[r] = -1;  // the embedding step re-validates rows: an invalid token keeps this one out
    w.pos[r] = 0;
    seq[r] = 0;
  }
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int L = lens[i];
    if (L < 1 || L > max_len) continue;
    const int o = off[i];
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
      const int64_t r = (int64_t)o + j;
      if (r >= rows) break;
      const int t = prompts[(int64_t)i * stride + j];
      const bool ok = t >= 0 && t < vocab;
      w.tok[r] = t;  // an out-of-range token is flagged (and kept out) by the embedding step
      w.pos[r] = j;
      w.flags[r] = ok ? 0 : SEQ_INVALID;
      seq[r] = i;
    }
  }
}

// Final residual row of every prompt's last token -> row i of dst, argmax key cleared.
__global__ void prefill_gather_kernel(int n, int rows, int dim, const int32_t* __restrict__ lens,
                                      const int32_t* __restrict__ off, const float* __restrict__ x,
                                      float* __restrict__ dst, unsigned long long* keys) {
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    int64_t r = (int64_t)off[i] + lens[i] - 1;
    if (r < 0 || r >= rows) r = 0;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) dst[(int64_t)i * dim + k] = x[r * dim + k];
    if (threadIdx.x == 0) keys[i] = 0ull;
  }
}

__global__ void prefill_argmax_kernel(int n, const unsigned long long* __restrict__ keys, int32_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = argmax_index(keys[i]);
}

// Cross entropy of each token row against its target, as F.cross_entropy
// with ignore_index=-1 (training/model.py:262): -(log_softmax(x)[t]) =
// -((x[t] - max) - log(sum exp(x - max))).  One CTA per row (grid-stride);
// a row whose target is -1, or that is invalid, counts 0; a target outside
// [0, vocab) otherwise is flagged in err.
__global__ void __launch_bounds__(256) row_nll_kernel(int rows, int vocab, const float* __restrict__ logits,
                                                      const int32_t* __restrict__ targets, int stride,
                                                      const int32_t* __restrict__ seq, const int32_t* __restrict__ pos,
                                                      const int32_t* __restrict__ flags, float* __restrict__ nll,
                                                      int32_t* __restrict__ counted, int32_t* err) {
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int t = targets[(int64_t)seq[r] * stride + pos[r]];
    const bool in = !(flags[r] & SEQ_INVALID) && t != -1;
    if (in && (t < 0 || t >= vocab)) {
      if (threadIdx.x == 0) atomicOr(err, 1);
    }
    if (!in || t < 0 || t >= vocab) {
      if (threadIdx.x == 0) {
        nll[r] = 0.0f;
        counted[r] = 0;
      }
      continue;
    }
    const float* x = logits + (int64_t)r * vocab;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < vocab; c += blockDim.x) m = fmaxf(m, x[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (int c = threadIdx.x; c < vocab; c += blockDim.x) s += expf(__fsub_rn(x[c], m));
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = red[0];
      for (int i = 1; i < 8; ++i) tot += red[i];
      nll[r] = -__fsub_rn(__fsub_rn(x[t], m), logf(tot));
      counted[r] = 1;
    }
    __syncthreads();
  }
}

// Mean of the counted rows' cross entropies (FP64 sums, fixed order): the
// reduction='mean' of F.cross_entropy; NaN when every target is ignored.
__global__ void __launch_bounds__(256) mean_loss_kernel(int rows, const float* __restrict__ nll,
                                                        const int32_t* __restrict__ counted, float* loss) {
  __shared__ double rs[8];
  __shared__ long long rc[8];
  double s = 0.0;
  long long c = 0;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    s += (double)nll[r];
    c += counted[r];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if (lane == 0) {
    rs[warp] = s;
    rc[warp] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0.0;
    long long tc = 0;
    for (int i = 0; i < 8; ++i) {
      ts += rs[i];
      tc += rc[i];
    }
    *loss = tc ? (float)(ts / (double)tc) : __int_as_float(0x7FC00000);
  }
}

// ---- general tensor-core step (tcg.cuh) -------------------------------------

// Shapes the general tensor-core linears handle: K (dim, hidden) multiples of
// 64; wq|wk|wv, wo, w2 and vocab rows in whole 128-row tiles; W1/W3 in
// 64-pair tiles.
static bool tcg_shapes_ok(const q6w_model_desc& d, int kvr) {
  if (d.dim > tcg::kImgMaxK || d.hidden_dim > tcg::kImgMaxK) return false;
  // K (dim, hidden) in whole packed groups of kG x 64 columns
  return d.dim % (64 * tcg::kG) == 0 && d.hidden_dim % (64 * tcg::kG) == 0 && d.dim >= 256 && d.dim % 128 == 0 &&
         kvr % 128 == 0 && d.vocab_size % 128 == 0;
}

// Clusters of C CTAs (index log2 C) that can be resident at once: a cluster
// sits inside one GPC, so fewer than sm_count / C clusters fit.
static int g_tcg_clusters[4] = {0, 0, 0, 0};

static cudaError_t tcg_set_attrs() {
  const int smem = (int)tcg::kSmem;
  cudaError_t e = cudaFuncSetAttribute(tcg::tcg_kernel<tcg::GEPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tcg::tcg_kernel<tcg::GEPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tcg::tcg_kernel<tcg::GEPI_GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tcg::tcg_kernel<tcg::GEPI_VOCAB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tcg::tcg_kernel<tcg::GEPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  for (int l = 0; l < 4 && e == cudaSuccess; ++l) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(1 << l));
    cfg.blockDim = dim3(tcg::kThreads);
    cfg.dynamicSmemBytes = tcg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1u << l;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, tcg::tcg_kernel<tcg::GEPI_RESID>, &cfg);
    g_tcg_clusters[l] = n;
  }
  return e;
}

// Activation rows from which the general tensor-core linears run (below: the
// SIMT GEMV / GEMM).
static int tcg_min_rows() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q6W_TCG_MIN_ROWS");
    v = e ? atoi(e) : 16;
    if (v < 1) v = 1;
  }
  return v;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link to libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

// 2-D uint8 tensor map over a packed matrix [rows][K*3/4], box 48 kG bytes x box_rows.
static int32_t weight_map(CUtensorMap* map, const uint8_t* q, int rows, int K, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(Q6W_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (!aligned(q, 16)) return fail(Q6W_ERR_ALIGN, "weights must be 16-byte aligned for the tensor-core linears");
  const cuuint64_t rb = (cuuint64_t)K * 3 / 4;
  cuuint64_t gdim[2] = {rb, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {rb};
  cuuint32_t box[2] = {48 * tcg::kG, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q6W_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q6W_OK;
}

static int32_t tcg_launch(int epi, const tcg::GArgs& a, int sms, cudaStream_t st) {
  const bool glu = epi == tcg::GEPI_GLU;
  const int wtiles = tcg::weight_tiles(epi, a.ms);
  const int items = wtiles * ((a.n + tcg::kAR - 1) / tcg::kAR);
  const int nks = a.K / (64 * tcg::kG);  // K steps
  // split K over a cluster while the tiles alone would leave SMs idle and
  // every cluster is resident at once (a second wave would double the time)
  int C = 1, l = 0;
  while (C < tcg::kMaxSplit && items * C * 2 <= sms && nks % (C * 2) == 0 && items <= g_tcg_clusters[l + 1]) {
    C *= 2;
    ++l;
  }
  tcg::GMaps maps;
  memset(&maps, 0, sizeof(maps));
  int32_t rc;
  if (glu) {
    if ((rc = weight_map(&maps.m[0], a.ms.q0, a.ms.n_pairs, a.ms.cols, tcg::kWR / 2))) return rc;
    if ((rc = weight_map(&maps.m[1], a.ms.q1, a.ms.n_pairs, a.ms.cols, tcg::kWR / 2))) return rc;
  } else {
    const int total = 2 * a.ms.n_pairs;
    if ((rc = weight_map(&maps.m[0], a.ms.q0, a.ms.end0, a.ms.cols, tcg::kWR))) return rc;
    if (a.ms.end1 > a.ms.end0 && (rc = weight_map(&maps.m[1], a.ms.q1, a.ms.end1 - a.ms.end0, a.ms.cols, tcg::kWR)))
      return rc;
    if (total > a.ms.end1 && (rc = weight_map(&maps.m[2], a.ms.q2, total - a.ms.end1, a.ms.cols, tcg::kWR)))
      return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items * C));
  cfg.blockDim = dim3(tcg::kThreads);
  cfg.dynamicSmemBytes = tcg::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (epi) {
    case tcg::GEPI_QKV: e = cudaLaunchKernelEx(&cfg, tcg::tcg_kernel<tcg::GEPI_QKV>, a, maps); break;
    case tcg::GEPI_RESID: e = cudaLaunchKernelEx(&cfg, tcg::tcg_kernel<tcg::GEPI_RESID>, a, maps); break;
    case tcg::GEPI_GLU: e = cudaLaunchKernelEx(&cfg, tcg::tcg_kernel<tcg::GEPI_GLU>, a, maps); break;
    case tcg::GEPI_STORE: e = cudaLaunchKernelEx(&cfg, tcg::tcg_kernel<tcg::GEPI_STORE>, a, maps); break;
    default: e = cudaLaunchKernelEx(&cfg, tcg::tcg_kernel<tcg::GEPI_VOCAB>, a, maps); break;
  }
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "tcg_kernel launch: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

static int32_t tcg_image(const float* x, int ldx, int n, int K, const float* g, float eps, uint8_t* img,
                         cudaStream_t st, bool permuted = true) {
  if (K % 16 || K > tcg::kImgMaxK) return fail(Q6W_ERR_ARG, "image of K=%d unsupported", K);
  if (permuted)
    tcg::image_kernel<true><<<n, tcg::kImgThreads, 0, st>>>(x, ldx, n, K, g, eps, img);
  else
    tcg::image_kernel<false><<<n, tcg::kImgThreads, 0, st>>>(x, ldx, n, K, g, eps, img);
  Q6W_LAUNCH_CHECK("image_kernel");
  return Q6W_OK;
}

// The batched step with every linear on the general tensor-core kernel: the
// inputs of the linears become activation images (RMSNorm fused where the
// reference normalises), attention as in the SIMT step.
static int32_t enqueue_step_tcg(const q6w_model* M, int n, const Work& w, float* kc, float* vc, int64_t cstride,
                                const EpiArgs& vocab_ep, cudaStream_t st, bool with_vocab) {
  const q6w_model_desc& d = M->d;
  const int dim = d.dim, kvr = M->kv_rows, hid = d.hidden_dim, S = d.max_seq_len;
  embed_kernel<<<n < 2048 ? n : 2048, 128, 0, st>>>(d.tok_embeddings.packed, d.tok_embeddings.scales, dim,
                                                    d.vocab_size, S, n, w);
  Q6W_LAUNCH_CHECK("embed_kernel");
  tcg::GArgs base;
  memset(&base, 0, sizeof(base));
  base.n = n;
  base.err = w.err;
  base.ep.pos = w.pos;
  base.ep.flags = w.flags;
  base.ep.seq = w.seq;
  base.ep.kv_half = M->kv_half;
  int32_t rc;
  const int warps = d.n_heads < 8 ? d.n_heads : 8;
  const dim3 agrid(n, (d.n_heads + warps - 1) / warps);
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    const int64_t layer_off = (int64_t)l * S * kvr;
    if ((rc = tcg_image(w.x, dim, n, dim, L.attention_norm, d.norm_eps, w.xs_img, st))) return rc;
    {
      tcg::GArgs a = base;
      a.img = w.xs_img;
      a.K = dim;
      a.ms = {L.wq.packed, L.wk.packed, L.wv.packed, L.wq.scales, L.wk.scales, L.wv.scales,
              dim, dim + kvr, dim, 0, (dim + 2 * kvr) / 2};
      a.ep.qbuf = w.qb; a.ep.ldq = dim;
      a.ep.kc = kc; a.ep.vc = vc; a.ep.cache_stride = cstride; a.ep.layer_off = layer_off;
      a.ep.rope_cos = d.rope_cos; a.ep.rope_sin = d.rope_sin;
      a.ep.hd = M->hd; a.ep.q_rows = dim; a.ep.kv_rows = kvr;
      if ((rc = tcg_launch(tcg::GEPI_QKV, a, M->sm_count, st))) return rc;
    }
    if (w.poff && launch_attn_prompt(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, w.n_prompts, w.max_len, n, st,
                                     w.qb, dim, kc, vc, cstride, layer_off, w.poff, w.plens, w.flags, M->denom,
                                     w.att, dim, nullptr, M->kv_half)) {
      Q6W_LAUNCH_CHECK("attn_prompt_kernel");
    } else if (launch_attn_rows(M->hd, d.n_kv_heads, d.n_heads / d.n_kv_heads, agrid, st, w.qb, dim, kc, vc,
                                cstride, layer_off, w.pos, 1, w.flags, w.att, dim, S, M->denom, nullptr, w.seq,
                                M->kv_half, false, attn_deep(M, n))) {
      Q6W_LAUNCH_CHECK("attn_rows_kernel");
    } else if (launch_attn_head(M->hd, n, d.n_heads, d.n_kv_heads, st, w.qb, dim, kc, vc, cstride, layer_off,
                                w.pos, 1, w.flags, w.att, dim, S, M->denom, w.seq, M->kv_half)) {
      Q6W_LAUNCH_CHECK("attn_head_kernel");
    } else if (M->kv_half) {
      return fail(Q6W_ERR_ARG, "no FP16-KV attention kernel for this head layout");
    } else {
      return fail(Q6W_ERR_ARG, "no attention kernel for head_dim %d on the tensor-core step", M->hd);
    }
    if ((rc = tcg_image(w.att, dim, n, dim, nullptr, 0.f, w.att_img, st))) return rc;
    {
      tcg::GArgs a = base;
      a.img = w.att_img;
      a.K = dim;
      a.ms = {L.wo.packed, nullptr, nullptr, L.wo.scales, nullptr, nullptr, dim, dim, dim, 0, dim / 2};
      a.ep.y = w.x; a.ep.ldy = dim;
      if ((rc = tcg_launch(tcg::GEPI_RESID, a, M->sm_count, st))) return rc;
    }
    if ((rc = tcg_image(w.x, dim, n, dim, L.ffn_norm, d.norm_eps, w.xs_img, st))) return rc;
    {
      tcg::GArgs a = base;
      a.img = w.xs_img;
      a.K = dim;
      a.ms = {L.w1.packed, L.w3.packed, nullptr, L.w1.scales, L.w3.scales, nullptr, hid, hid, dim, 1, hid};
      a.ep.y = w.hb; a.ep.ldy = hid;
      if ((rc = tcg_launch(tcg::GEPI_GLU, a, M->sm_count, st))) return rc;
    }
    if ((rc = tcg_image(w.hb, hid, n, hid, nullptr, 0.f, w.hs_img, st))) return rc;
    {
      tcg::GArgs a = base;
      a.img = w.hs_img;
      a.K = hid;
      a.ms = {L.w2.packed, nullptr, nullptr, L.w2.scales, nullptr, nullptr, dim, dim, hid, 0, dim / 2};
      a.ep.y = w.x; a.ep.ldy = dim;
      if ((rc = tcg_launch(tcg::GEPI_RESID, a, M->sm_count, st))) return rc;
    }
  }
  if (!with_vocab) return Q6W_OK;
  if ((rc = tcg_image(w.x, dim, n, dim, d.norm, d.norm_eps, w.xs_img, st))) return rc;
  tcg::GArgs a = base;
  a.img = w.xs_img;
  a.K = dim;
  a.ms = {d.tok_embeddings.packed, nullptr, nullptr, d.tok_embeddings.scales, nullptr, nullptr,
          d.vocab_size, d.vocab_size, dim, 0, d.vocab_size / 2};
  a.ep = vocab_ep;
  a.ep.pos = w.pos;
  a.ep.flags = w.flags;
  a.ep.keys = w.keys;
  a.ep.gen = w.gen;
  a.ep.plen = w.plen;
  a.ep.vocab = d.vocab_size;
  return tcg_launch(tcg::GEPI_VOCAB, a, M->sm_count, st);
}

// ---- persistent B=1 step (pdec.cuh) -------------------------------------------

// Shapes the persistent step takes: K (dim, hidden) = 512 WC with WC in
// {1, 2, 4, 8, 11} (the streaming GEMV's layouts), row counts in multiples of 4
// (16-byte scale copies), head dims 64 / 128, at most one query head per CTA,
// and every matrix and its scales 16-byte aligned for the bulk copies.
static bool pdec_wc_ok(int K) {
  if (K % 512) return false;
  const int wc = K / 512;
  return wc == 1 || wc == 2 || wc == 4 || wc == 8 || wc == 11;
}

static bool pdec_shapes_ok(const q6w_model* M) {
  const q6w_model_desc& d = M->d;
  if (!pdec_wc_ok(d.dim) || !pdec_wc_ok(d.hidden_dim) || (M->hd != 64 && M->hd != 128)) return false;
  if (d.dim % 8 || M->kv_rows % 8 || d.vocab_size % 8 || d.hidden_dim % 8) return false;
  if (d.n_layers > pdec::kMaxLayers || d.max_seq_len > pdec::kMaxSeq || d.n_heads % d.n_kv_heads) return false;
  auto al = [](const q6w_qmat& m) { return aligned(m.packed, 16) && aligned(m.scales, 16); };
  if (!al(d.tok_embeddings)) return false;
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    if (!al(L.wq) || !al(L.wk) || !al(L.wv) || !al(L.wo) || !al(L.w1) || !al(L.w2) || !al(L.w3)) return false;
  }
  return true;
}

// Attributes and the cooperative grid (one CTA per SM, all resident) of the
// persistent step; false leaves the model on the per-kernel step.
// Why the persistent step is off, on stderr when Q6W_DEBUG_PDEC=1.
static bool pdec_off(const char* why, cudaError_t e = cudaSuccess) {
  const char* dbg = getenv("Q6W_DEBUG_PDEC");
  if (dbg && dbg[0] == '1') fprintf(stderr, "q6w: persistent B=1 step off: %s (%s)\n", why, cudaGetErrorString(e));
  cudaGetLastError();
  return false;
}

static bool pdec_setup(q6w_model* M) {
  int coop = 0;
  cudaError_t e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, M->device);
  if (e != cudaSuccess || !coop) return pdec_off("no cooperative launch", e);
  const size_t smem = pdec::smem_bytes(M->hd, M->d.max_seq_len);
  e = cudaFuncSetAttribute(pdec::pdec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return pdec_off("shared-memory attribute", e);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pdec::pdec_kernel, pdec::kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) {
    const char* dbg = getenv("Q6W_DEBUG_PDEC");
    if (dbg && dbg[0] == '1') {
      cudaFuncAttributes fa;
      cudaFuncGetAttributes(&fa, pdec::pdec_kernel);
      int no_smem = 0;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&no_smem, pdec::pdec_kernel, pdec::kThreads, 0);
      fprintf(stderr, "q6w: pdec regs %d, max threads %d, static smem %zu, max dyn smem %d, local %zu; "
                      "asked %zu dyn smem; resident per SM %d (with 0 dyn smem: %d)\n",
              fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, fa.maxDynamicSharedSizeBytes, fa.localSizeBytes,
              smem, per_sm, no_smem);
    }
    return pdec_off("no resident CTA per SM", e);
  }
  M->pdec_grid = M->sm_count;  // one CTA per SM
  M->pdec_smem = smem;
  return M->d.n_heads <= M->pdec_grid;
}

// One B=1 model step as embed + one cooperative launch of the persistent kernel.
static int32_t enqueue_step_pdec(const q6w_model* M, const Work& w, float* kc, float* vc, const EpiArgs& vocab_ep,
                                 cudaStream_t st) {
  const q6w_model_desc& d = M->d;
  embed_kernel<<<1, 128, 0, st>>>(d.tok_embeddings.packed, d.tok_embeddings.scales, d.dim, d.vocab_size,
                                  d.max_seq_len, 1, w);
  Q6W_LAUNCH_CHECK("embed_kernel");
  Q6W_CUDA_TRY(cudaMemsetAsync(w.sync, 0, 8, st));
  pdec::Args a;
  memset(&a, 0, sizeof(a));
  a.dim = d.dim; a.hidden = d.hidden_dim; a.n_layers = d.n_layers; a.n_heads = d.n_heads; a.n_kv = d.n_kv_heads;
  a.hd = M->hd; a.vocab = d.vocab_size; a.max_seq = d.max_seq_len; a.kvr = M->kv_rows;
  a.eps = d.norm_eps; a.denom = M->denom;
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    a.layers[l] = {{L.wq.packed, L.wq.scales}, {L.wk.packed, L.wk.scales}, {L.wv.packed, L.wv.scales},
                   {L.wo.packed, L.wo.scales}, {L.w1.packed, L.w1.scales}, {L.w2.packed, L.w2.scales},
                   {L.w3.packed, L.w3.scales}, L.attention_norm, L.ffn_norm};
  }
  a.tok = {d.tok_embeddings.packed, d.tok_embeddings.scales};
  a.norm = d.norm; a.rope_cos = d.rope_cos; a.rope_sin = d.rope_sin;
  a.x = w.x; a.qb = w.qb; a.att = w.att; a.hb = w.hb;
  a.kc = kc; a.vc = vc; a.kv_half = M->kv_half;
  a.pos = w.pos; a.flags = w.flags;
  a.vep = vocab_ep;
  a.vep.pos = w.pos; a.vep.flags = w.flags; a.vep.keys = w.keys; a.vep.gen = w.gen; a.vep.plen = w.plen;
  a.vep.vocab = d.vocab_size;
  a.sync = w.sync;
  a.err = w.err;
  a.fc = stream::field_consts();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)M->pdec_grid);
  cfg.blockDim = dim3(pdec::kThreads);
  cfg.dynamicSmemBytes = M->pdec_smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, pdec::pdec_kernel, a);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "pdec_kernel launch: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

// Shapes the tensor-core step handles: dim 128, [wq|wk|wv] one N tile of at
// most 256 rows in 32-row chunks, hidden a multiple of 128 whose packed w2
// rows fit the staging area at the widest residual tile (128 rows: hidden at
// most 384), vocab a multiple of 256, and an instantiated streaming-attention
// layout.  Wider hidden layers take the general tensor-core step.
static bool tc_shapes_ok(const q6w_model_desc& d, int hd, int kvr) {
  const int rep = d.n_heads / d.n_kv_heads;
  return d.dim == 128 && kvr % 32 == 0 && d.dim + 2 * kvr <= 256 && d.hidden_dim % 128 == 0 &&
         tc::stage_fits(128, d.hidden_dim) && d.vocab_size % 256 == 0 && (hd == 16 || hd == 32) && rep <= 4 &&
         d.n_kv_heads * hd / 16 <= 32;
}

static int tc_min_seqs() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q6W_TC_MIN_SEQS");
    v = e ? atoi(e) : 64;
    if (v < 1) v = 1;
  }
  return v;
}

static int32_t check_qmat(const q6w_qmat& m, int rows, int cols, const char* name) {
  if (!m.packed || !m.scales) return fail(Q6W_ERR_ARG, "%s: null pointer", name);
  if (m.rows != rows || m.cols != cols)
    return fail(Q6W_ERR_ARG, "%s: shape [%d, %d], expected [%d, %d]", name, m.rows, m.cols, rows, cols);
  if (!aligned(m.packed, 4) || !aligned(m.scales, 4))
    return fail(Q6W_ERR_ALIGN, "%s: packed rows and scales must be 4-byte aligned", name);
  return Q6W_OK;
}

static int attn_smem_ok(const q6w_model* M) {
  const int warps = M->d.n_heads < 8 ? M->d.n_heads : 8;
  return (size_t)warps * M->d.max_seq_len * sizeof(float) <= 200 * 1024;
}

static int32_t set_attn_attrs(const q6w_model* M) {
  const int warps = M->d.n_heads < 8 ? M->d.n_heads : 8;
  const int smem = warps * M->d.max_seq_len * (int)sizeof(float);
  if (smem <= 48 * 1024) return Q6W_OK;
  cudaError_t e = cudaSuccess;
  switch (M->hd) {
    case 16: e = cudaFuncSetAttribute(attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 32: e = cudaFuncSetAttribute(attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 64: e = cudaFuncSetAttribute(attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 128: e = cudaFuncSetAttribute(attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 256: e = cudaFuncSetAttribute(attn_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 512: e = cudaFuncSetAttribute(attn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
  }
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

static void b1_fill(const q6w_model* M, b1::Args& a) {
  memset(&a, 0, sizeof(a));
  const q6w_model_desc& d = M->d;
  a.dim = d.dim; a.n_layers = d.n_layers; a.n_heads = d.n_heads; a.n_kv = d.n_kv_heads; a.hd = M->hd;
  a.hidden = d.hidden_dim; a.vocab = d.vocab_size; a.max_seq = d.max_seq_len;
  a.eps = d.norm_eps; a.denom = M->denom;
  a.tok = {d.tok_embeddings.packed, d.tok_embeddings.scales};
  a.norm = d.norm; a.rope_cos = d.rope_cos; a.rope_sin = d.rope_sin;
  for (int l = 0; l < d.n_layers && l < b1::kMaxLayers; ++l) {
    const q6w_layer_weights& L = M->layers[l];
    a.layers[l].wq = {L.wq.packed, L.wq.scales}; a.layers[l].wk = {L.wk.packed, L.wk.scales};
    a.layers[l].wv = {L.wv.packed, L.wv.scales}; a.layers[l].wo = {L.wo.packed, L.wo.scales};
    a.layers[l].w1 = {L.w1.packed, L.w1.scales}; a.layers[l].w2 = {L.w2.packed, L.w2.scales};
    a.layers[l].w3 = {L.w3.packed, L.w3.scales};
    a.layers[l].attn_norm = L.attention_norm; a.layers[l].ffn_norm = L.ffn_norm;
  }
}

// Shapes the cluster kernel handles: dim 128, at most 8 layers and 8 query
// heads (one per CTA), head_dim 16 or 32, hidden and vocab multiples of 16,
// and every CTA's weights plus vectors within the shared-memory cap.
static bool b1_shapes_ok(const q6w_model* M, size_t* smem) {
  const q6w_model_desc& d = M->d;
  if (d.dim != 128 || d.n_layers > b1::kMaxLayers || d.n_heads > b1::kCtas || (M->hd != 16 && M->hd != 32) ||
      d.n_heads * M->hd != d.dim || d.n_heads % d.n_kv_heads || d.hidden_dim % 16 || d.vocab_size % 16)
    return false;
  b1::Args a;
  b1_fill(M, a);
  size_t mx = 0;
  for (int c = 0; c < b1::kCtas; ++c) {
    b1::Plan p;
    b1::make_plan(a, c, p);
    mx = p.bytes > mx ? p.bytes : mx;
  }
  *smem = mx;
  return mx <= b1::kMaxSmem;
}

}  // namespace q6w

using namespace q6w;

extern "C" int32_t q6w_model_create(const q6w_model_desc* desc, q6w_model** out) {
  clear_error();
  if (!desc || !out) return fail(Q6W_ERR_ARG, "q6w_model_create: null argument");
  *out = nullptr;
  const q6w_model_desc& d = *desc;
  if (d.dim <= 0 || d.n_layers <= 0 || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.vocab_size <= 0 ||
      d.hidden_dim <= 0 || d.max_seq_len <= 0)
    return fail(Q6W_ERR_ARG, "model dimensions must be positive");
  if (d.dim % d.n_heads || d.n_heads % d.n_kv_heads)
    return fail(Q6W_ERR_ARG, "dim %% n_heads and n_heads %% n_kv_heads must be 0");
  const int hd = d.dim / d.n_heads;
  if (hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256 && hd != 512)
    return fail(Q6W_ERR_ARG, "head_dim %d unsupported (16, 32, 64, 128, 256 or 512)", hd);
  if (d.dim % 16 || d.hidden_dim % 16)
    return fail(Q6W_ERR_ARG, "dim and hidden_dim must be multiples of 16");
  if (d.vocab_size % 2) return fail(Q6W_ERR_ARG, "vocab_size must be even");
  if (!(d.norm_eps >= 0.0f)) return fail(Q6W_ERR_ARG, "norm_eps must be >= 0");
  if (!d.layers || !d.norm || !d.rope_cos || !d.rope_sin)
    return fail(Q6W_ERR_ARG, "q6w_model_create: null weight pointer");
  const int kvr = d.n_kv_heads * hd;
  int32_t st = check_qmat(d.tok_embeddings, d.vocab_size, d.dim, "tok_embeddings");
  if (st) return st;
  for (int l = 0; l < d.n_layers; ++l) {
    const q6w_layer_weights& L = d.layers[l];
    if ((st = check_qmat(L.wq, d.dim, d.dim, "wq")) || (st = check_qmat(L.wk, kvr, d.dim, "wk")) ||
        (st = check_qmat(L.wv, kvr, d.dim, "wv")) || (st = check_qmat(L.wo, d.dim, d.dim, "wo")) ||
        (st = check_qmat(L.w1, d.hidden_dim, d.dim, "w1")) ||
        (st = check_qmat(L.w2, d.dim, d.hidden_dim, "w2")) ||
        (st = check_qmat(L.w3, d.hidden_dim, d.dim, "w3")))
      return st;
    if (!L.attention_norm || !L.ffn_norm) return fail(Q6W_ERR_ARG, "layer %d: null norm", l);
  }
  q6w_model* M = new (std::nothrow) q6w_model();
  if (!M) return fail(Q6W_ERR_ARG, "out of host memory");
  M->d = d;
  M->layers.assign(d.layers, d.layers + d.n_layers);
  M->d.layers = M->layers.data();
  M->hd = hd;
  M->kv_rows = kvr;
  M->denom = (float)sqrt((double)hd);
  cudaGetDevice(&M->device);
  if (!attn_smem_ok(M)) {
    delete M;
    return fail(Q6W_ERR_ARG, "max_seq_len %d too large for the attention score buffer", d.max_seq_len);
  }
  if ((st = set_attn_attrs(M))) {
    delete M;
    return st;
  }
  cudaDeviceGetAttribute(&M->sm_count, cudaDevAttrMultiProcessorCount, M->device);
  if (M->sm_count <= 0) M->sm_count = 148;
  {
    const char* off = getenv("Q6W_DISABLE_TC");
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, M->device);
    M->use_tc = !(off && off[0] == '1') && major == 10 && tc_shapes_ok(d, hd, kvr);
    if (M->use_tc && (st = tc_set_attrs())) {
      delete M;
      return st;
    }
    const char* offg = getenv("Q6W_DISABLE_TCG");
    M->use_tcg = !M->use_tc && !(offg && offg[0] == '1') && major == 10 && tcg_shapes_ok(d, kvr);
    // the image kernel reads the norm weights as float4
    for (int l = 0; l < d.n_layers && M->use_tcg; ++l)
      M->use_tcg = aligned(M->layers[l].attention_norm, 16) && aligned(M->layers[l].ffn_norm, 16);
    M->use_tcg = M->use_tcg && aligned(d.norm, 16);
    attn_group_setup();
    if (M->use_tcg && tcg_set_attrs() != cudaSuccess) {
      cudaGetLastError();
      M->use_tcg = false;  // the SIMT kernels still serve every shape
    }
    const char* off1 = getenv("Q6W_DISABLE_B1");
    M->use_b1 = !(off1 && off1[0] == '1') && major == 10 && b1_shapes_ok(M, &M->b1_smem);
    if (M->use_b1) {
      // the attribute belongs to the function, not the model: allow the cap every model is held to
      cudaError_t e = cudaFuncSetAttribute(b1::b1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)b1::kMaxSmem);
      if (e != cudaSuccess) {
        cudaGetLastError();
        M->use_b1 = false;  // the batched step still serves single requests
      }
    }
    // The persistent B=1 step is opt-in: on the 1.1B shape it measured 1047 us a token against 717 us
    // for the per-kernel step (per-phase L2 round trips at one CTA per SM cost more than the
    // launches they replace).
    const char* onp = getenv("Q6W_PDEC");
    M->use_pdec = (onp && onp[0] == '1') && major == 10 && (pdec_shapes_ok(M) || pdec_off("shapes")) &&
                  pdec_setup(M);
    // Programmatic dependent launch across the tensor-core step: Q6W_PDL=1 / 0 force it on / off;
    // unset, the decode step uses it at small batches only (step_pdl).
    const char* pdl = getenv("Q6W_PDL");
    M->pdl_mode = !pdl || !pdl[0] ? -1 : pdl[0] == '1' ? 1 : 0;
    const char* deep = getenv("Q6W_ATTN_DEEP");
    M->attn_deep_mode = !deep || !deep[0] ? -1 : deep[0] == '1' ? 1 : 0;
  }
  *out = M;
  return Q6W_OK;
}

extern "C" int32_t q6w_model_set_kv_dtype(q6w_model* M, int32_t kv_dtype) {
  clear_error();
  if (!M) return fail(Q6W_ERR_ARG, "null model");
  if (kv_dtype != Q6W_KV_F32 && kv_dtype != Q6W_KV_F16)
    return fail(Q6W_ERR_ARG, "kv_dtype must be Q6W_KV_F32 or Q6W_KV_F16");
  if (kv_dtype == Q6W_KV_F16) {
    const int KV = M->d.n_kv_heads, rep = M->d.n_heads / KV, hd = M->hd;
    const bool ok = attn_rows_instantiated(hd, KV, rep) ||
                    ((hd == 64 || hd == 128) && attn_head_smem(hd, M->d.max_seq_len) <= 48 * 1024);
    if (!ok) return fail(Q6W_ERR_ARG, "FP16 KV storage is not available for head_dim %d with %d kv heads", hd, KV);
  }
  const bool half = kv_dtype == Q6W_KV_F16;
  if (half != M->kv_half && M->exec) {  // the captured step graph bakes in the cache type
    cudaGraphExecDestroy(M->exec);
    M->exec = nullptr;
    M->have_key = false;
  }
  M->kv_half = half;
  return Q6W_OK;
}

extern "C" void q6w_model_destroy(q6w_model* M) {
  if (!M) return;
  if (M->exec) cudaGraphExecDestroy(M->exec);
  if (M->cap_stream) cudaStreamDestroy(M->cap_stream);
  delete M;
}

extern "C" size_t q6w_workspace_bytes(const q6w_model* M, int32_t max_seqs) {
  if (!M || max_seqs < 0) return 0;
  return layout(M, max_seqs, nullptr, nullptr, true);
}

static int32_t check_ws(const q6w_model* M, int n, void* ws, size_t bytes, Work* w, bool sample = false) {
  if (!ws) return fail(Q6W_ERR_ARG, "null workspace");
  if (!aligned(ws, 256)) return fail(Q6W_ERR_ALIGN, "workspace must be 256-byte aligned");
  const size_t need = layout(M, n, nullptr, nullptr, sample);
  if (need > bytes)
    return fail(Q6W_ERR_ARG, "workspace of %zu bytes too small for %d sequences (%zu needed)", bytes, n, need);
  layout(M, n, (char*)ws, w, sample);
  return Q6W_OK;
}

// Sampler parameters from the C struct (validated as torch_benchmark.generate
// validates them, :246-255); the Python-float values rounded to FP32 where
// the reference applies them to FP32 tensors.
static int32_t make_sample_params(const q6w_sample_args* s, int vocab, const StopSet& stop, smp::Params* p) {
  memset(p, 0, sizeof(*p));
  if (!(s->temperature >= 0.0f) || !isfinite(s->temperature))
    return fail(Q6W_ERR_ARG, "temperature must be finite and >= 0");
  if (!(s->repetition_penalty > 0.0f) || !isfinite(s->stop_token_bias) || s->stop_token_bias_after < 0 ||
      s->no_repeat_ngram_size < 0)
    return fail(Q6W_ERR_ARG, "repetition_penalty must be positive, stop_token_bias finite, min_new_tokens within "
                             "the limit, and bias/ngram settings nonnegative");
  if (vocab > smp::kMaxVocab) return fail(Q6W_ERR_ARG, "sampling supports vocabularies up to %d", smp::kMaxVocab);
  p->temperature = s->temperature;
  p->repetition_penalty = s->repetition_penalty;
  p->stop_bias = s->stop_token_bias;
  p->top_p = s->top_p;
  p->nucleus = s->top_p > 0.0 && s->top_p < 1.0;
  p->cutoff = (float)((1.0 - s->top_p) / (double)(vocab - 1));
  p->ngram = s->no_repeat_ngram_size;
  p->bias_after = s->stop_token_bias_after;
  p->min_new = stop.min_new;
  p->n_stop = stop.n;
  for (int i = 0; i < kMaxStop; ++i) p->stop_ids[i] = stop.ids[i];
  return Q6W_OK;
}

// Whether the step needs the sampler (anything but a plain greedy pick).
static bool needs_sampler(const smp::Params& p) {
  return p.temperature != 0.0f || p.repetition_penalty != 1.0f || p.ngram != 0 || (p.n_stop && p.stop_bias != 0.0f);
}

static int32_t sample_attr(int vocab) {
  static std::mutex mu;
  static size_t set_to[64] = {0};
  int dev = 0;
  Q6W_CUDA_TRY(cudaGetDevice(&dev));
  const size_t need = smp::smem_bytes(vocab);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && set_to[dev] >= need) return Q6W_OK;
  Q6W_CUDA_TRY(cudaFuncSetAttribute(smp::sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need));
  if (dev >= 0 && dev < 64) set_to[dev] = need;
  return Q6W_OK;
}

static int32_t check_cache(const q6w_model* M, const float* kc, const float* vc, int64_t stride, int n) {
  if (!kc || !vc) return fail(Q6W_ERR_ARG, "null KV cache");
  if (!aligned(kc, 16) || !aligned(vc, 16)) return fail(Q6W_ERR_ALIGN, "KV cache must be 16-byte aligned");
  const int64_t per = (int64_t)M->d.n_layers * M->d.max_seq_len * M->kv_rows;
  if (n > 1 && (stride < per || stride % 4))
    return fail(Q6W_ERR_ARG, "cache_seq_stride %lld must be >= %lld and a multiple of 4", (long long)stride,
                (long long)per);
  return Q6W_OK;
}

extern "C" int32_t q6w_step(const q6w_model* M, int32_t token_id, int32_t position, float* k_cache,
                            float* v_cache, float* logits, void* workspace, size_t workspace_bytes,
                            q6w_stream_t stream) {
  clear_error();
  if (!M) return fail(Q6W_ERR_ARG, "null model");
  if (token_id < 0 || token_id >= M->d.vocab_size)
    return fail(Q6W_ERR_RANGE, "token id %d outside [0, %d)", token_id, M->d.vocab_size);
  if (position < 0 || position >= M->d.max_seq_len)
    return fail(Q6W_ERR_RANGE, "position %d outside [0, %d)", position, M->d.max_seq_len);
  if (!logits || !aligned(logits, 8)) return fail(Q6W_ERR_ARG, "logits must be non-null and 8-byte aligned");
  Work w;
  int32_t st = check_ws(M, 1, workspace, workspace_bytes, &w);
  if (st) return st;
  if ((st = check_cache(M, k_cache, v_cache, 0, 1))) return st;
  cudaStream_t s = (cudaStream_t)stream;
  init_batch_kernel<<<1, 32, 0, s>>>(1, nullptr, nullptr, token_id, position, w);
  Q6W_LAUNCH_CHECK("init_batch_kernel");
  EpiArgs v;
  memset(&v, 0, sizeof(v));
  v.y = logits;
  v.ldy = M->d.vocab_size;
  return enqueue_step(M, 1, w, k_cache, v_cache, 0, v, s);
}

extern "C" int32_t q6w_forward_batch(const q6w_model* M, int32_t n, const int32_t* tokens,
                                     const int32_t* positions, float* k_cache, float* v_cache,
                                     int64_t cache_seq_stride, float* logits, int32_t* argmax,
                                     void* workspace, size_t workspace_bytes, q6w_stream_t stream) {
  clear_error();
  if (!M) return fail(Q6W_ERR_ARG, "null model");
  if (n < 0) return fail(Q6W_ERR_ARG, "n_seqs must be >= 0");
  if (n == 0) return Q6W_OK;
  if (!tokens || !positions) return fail(Q6W_ERR_ARG, "null tokens/positions");
  if (logits && !aligned(logits, 8)) return fail(Q6W_ERR_ALIGN, "logits must be 8-byte aligned");
  Work w;
  int32_t st = check_ws(M, n, workspace, workspace_bytes, &w);
  if (st) return st;
  if ((st = check_cache(M, k_cache, v_cache, cache_seq_stride, n))) return st;
  cudaStream_t s = (cudaStream_t)stream;
  init_batch_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, tokens, positions, 0, 0, w);
  Q6W_LAUNCH_CHECK("init_batch_kernel");
  EpiArgs v;
  memset(&v, 0, sizeof(v));
  v.y = logits;
  v.ldy = M->d.vocab_size;
  if ((st = enqueue_step(M, n, w, k_cache, v_cache, cache_seq_stride, v, s))) return st;
  if (argmax) {
    keys_to_argmax_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, w.keys, argmax);
    Q6W_LAUNCH_CHECK("keys_to_argmax_kernel");
  }
  return Q6W_OK;
}

// Whether the decode step of n sequences launches its kernels with
// programmatic dependencies (each kernel's setup and weight copies overlap the
// previous kernel's tail).  Measured on the tensor-core step: faster at small
// batches (1024 sequences 37.1 -> 35.9 ms a generation, 4096 70.2 -> 69.3 ms),
// slower at 8192 (109.5 against 107.2-107.5 ms), so by default it is used
// while the batch has at most sm_count / 4 M tiles, the batches that also take
// the narrow tiles.
static bool step_pdl(const q6w_model* M, int n) {
  if (M->pdl_mode >= 0) return M->pdl_mode == 1;
  return 4 * ((n + tc::kM - 1) / tc::kM) <= M->sm_count;
}

static int32_t capture_step(q6w_model* M, const q6w_greedy_args* a, const Work& w,
                            const StopSet& stop, const smp::Params* sp) {
  if (!M->cap_stream) Q6W_CUDA_TRY(cudaStreamCreateWithFlags(&M->cap_stream, cudaStreamNonBlocking));
  if (M->exec) {
    cudaGraphExecDestroy(M->exec);
    M->exec = nullptr;
    M->have_key = false;
  }
  Q6W_CUDA_TRY(cudaStreamBeginCapture(M->cap_stream, cudaStreamCaptureModeRelaxed));
  EpiArgs v;
  memset(&v, 0, sizeof(v));
  v.step_logits = a->step_logits;
  v.new_tokens = a->new_tokens;
  v.min_new = stop.min_new;
  v.n_stop = sp ? 0 : stop.n;  // with the sampler, the stop ids are handled there
  for (int i = 0; i < kMaxStop; ++i) v.stop_ids[i] = stop.ids[i];
  if (sp) {
    v.y = w.logits;  // the raw logits row of every sequence, for the sampler
    v.ldy = M->d.vocab_size;
  }
  Work wp = w;
  wp.pdl = step_pdl(M, a->n_seqs);
  int32_t st = enqueue_step(M, a->n_seqs, wp, a->k_cache, a->v_cache, a->cache_seq_stride, v,
                            M->cap_stream);
  if (st == Q6W_OK && sp) {
    smp::Args sa;
    memset(&sa, 0, sizeof(sa));
    sa.logits = w.logits;
    sa.ld = M->d.vocab_size;
    sa.vocab = M->d.vocab_size;
    sa.hist = a->sampled;
    sa.hist_ld = a->new_tokens;
    sa.hist_len = w.gen;
    sa.rng = w.rng;
    sa.keys = w.keys;
    sa.flags = w.flags;
    sa.pos = w.pos;
    sa.plen = w.plen;
    sa.p = *sp;
    if (launch_k(smp::sample_kernel, dim3(a->n_seqs), dim3(smp::kThreads), smp::smem_bytes(M->d.vocab_size),
                 M->cap_stream, wp.pdl, sa) != cudaSuccess)
      st = fail(Q6W_ERR_CUDA, "sample_kernel launch failed");
  }
  if (st == Q6W_OK) {
    if (launch_k(advance_kernel, dim3(grid_for(a->n_seqs, 256)), dim3(256), 0, M->cap_stream, wp.pdl, a->n_seqs, w,
                 a->prompts, a->prompt_stride, a->new_tokens, stop, a->sampled, a->n_sampled,
                 a->stop_reason) != cudaSuccess)
      st = fail(Q6W_ERR_CUDA, "advance_kernel launch failed");
  }
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(M->cap_stream, &graph);
  if (st) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&M->exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    M->exec = nullptr;
    return fail(Q6W_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
  }
  return Q6W_OK;
}

// Rows of one q6w_prefill call (the tiled GEMM's grid has a 65535 x 128 row limit).
constexpr int64_t kMaxPrefillRows = 1 << 22;

// Workspace of q6w_prefill: the step workspace for total_tokens rows, then the
// row -> cache-row map and the prompt offsets.
static size_t prefill_layout(const q6w_model* M, int32_t n_prompts, int64_t total, char* base, Work* w,
                             int32_t** seq, int32_t** off) {
  const size_t step = layout(M, (int)total, base, w);
  char* p = base ? base + step : nullptr;
  const size_t a = ((size_t)4 * total + 255) & ~(size_t)255;
  const size_t b = ((size_t)4 * (n_prompts + 1) + 255) & ~(size_t)255;
  if (base) {
    *seq = reinterpret_cast<int32_t*>(p);
    *off = reinterpret_cast<int32_t*>(p + a);
  }
  return step + a + b;
}

extern "C" size_t q6w_prefill_workspace_bytes(const q6w_model* M, int32_t n_prompts, int64_t total_tokens) {
  if (!M || n_prompts < 0 || total_tokens < 0 || total_tokens > kMaxPrefillRows) return 0;
  return prefill_layout(M, n_prompts, total_tokens, nullptr, nullptr, nullptr, nullptr);
}

extern "C" int32_t q6w_prefill(const q6w_model* M, int32_t n_prompts, const int32_t* prompts,
                               const int32_t* prompt_lens, int32_t prompt_stride, int32_t max_prompt_len,
                               int64_t total_tokens, float* k_cache, float* v_cache, int64_t cache_seq_stride,
                               float* last_logits, int32_t* last_argmax, void* workspace, size_t workspace_bytes,
                               q6w_stream_t stream) {
  clear_error();
  if (!M) return fail(Q6W_ERR_ARG, "null model");
  if (n_prompts < 0 || total_tokens < 0) return fail(Q6W_ERR_ARG, "n_prompts and total_tokens must be >= 0");
  if (n_prompts == 0) return Q6W_OK;
  if (total_tokens < n_prompts || total_tokens > kMaxPrefillRows)
    return fail(Q6W_ERR_ARG, "total_tokens %lld must be in [n_prompts, %lld]", (long long)total_tokens,
                (long long)kMaxPrefillRows);
  if (!prompts || !prompt_lens) return fail(Q6W_ERR_ARG, "null prompts / prompt_lens");
  if (max_prompt_len < 1 || max_prompt_len > M->d.max_seq_len || prompt_stride < max_prompt_len)
    return fail(Q6W_ERR_ARG, "need 1 <= max_prompt_len <= max_seq_len (%d) and prompt_stride >= max_prompt_len",
                M->d.max_seq_len);
  if (last_logits && !aligned(last_logits, 8)) return fail(Q6W_ERR_ALIGN, "last_logits must be 8-byte aligned");
  if (!workspace) return fail(Q6W_ERR_ARG, "null workspace");
  if (!aligned(workspace, 256)) return fail(Q6W_ERR_ALIGN, "workspace must be 256-byte aligned");
  const size_t need = prefill_layout(M, n_prompts, total_tokens, nullptr, nullptr, nullptr, nullptr);
  if (workspace_bytes < need)
    return fail(Q6W_ERR_ARG, "workspace of %zu bytes too small (%zu needed)", workspace_bytes, need);
  int32_t st;
  if ((st = check_cache(M, k_cache, v_cache, cache_seq_stride, n_prompts))) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != M->device) return fail(Q6W_ERR_ARG, "model was created on device %d, current is %d", M->device, dev);
  Work w;
  int32_t *seq, *off;
  prefill_layout(M, n_prompts, total_tokens, (char*)workspace, &w, &seq, &off);
  const int rows = (int)total_tokens;
  cudaStream_t s = (cudaStream_t)stream;
  prefill_scan_kernel<<<1, 1024, 0, s>>>(n_prompts, prompt_lens, max_prompt_len, off, w.err);
  Q6W_LAUNCH_CHECK("prefill_scan_kernel");
  const int pgrid = n_prompts < 4096 ? n_prompts : 4096;
  prefill_rows_kernel<<<pgrid, 256, 0, s>>>(
      n_prompts, rows, prompts, prompt_stride, prompt_lens, max_prompt_len, M->d.vocab_size, off, w, seq);
  Q6W_LAUNCH_CHECK("prefill_rows_kernel");
  w.seq = seq;
  w.poff = off;
  w.plens = prompt_lens;
  w.n_prompts = n_prompts;
  w.max_len = max_prompt_len;
  w.pdl = M->pdl_mode == 1;
  EpiArgs none;
  memset(&none, 0, sizeof(none));
  if ((st = enqueue_step(M, rows, w, k_cache, v_cache, cache_seq_stride, none, s, false))) return st;
  // vocab of the last token of each prompt, on the gathered rows
  const int dim = M->d.dim;
  prefill_gather_kernel<<<n_prompts < 4096 ? n_prompts : 4096, 128, 0, s>>>(n_prompts, rows, dim, prompt_lens, off,
                                                                          w.x, w.qb, w.keys);
  Q6W_LAUNCH_CHECK("prefill_gather_kernel");
  const q6w_model_desc& d = M->d;
  MatSet mv = {d.tok_embeddings.packed, nullptr, nullptr, d.tok_embeddings.scales, nullptr, nullptr,
               d.vocab_size, d.vocab_size, dim, 0, d.vocab_size / 2};
  EpiArgs v;
  memset(&v, 0, sizeof(v));
  v.y = last_logits;
  v.ldy = d.vocab_size;
  v.keys = w.keys;
  v.vocab = d.vocab_size;
  cudaError_t e = LinearLauncher<true, EPI_VOCAB>::run(w.qb, dim, n_prompts, d.norm, d.norm_eps, mv, v, s);
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "prefill vocab linear: %s", cudaGetErrorString(e));
  if (last_argmax) {
    prefill_argmax_kernel<<<grid_for(n_prompts, 256), 256, 0, s>>>(n_prompts, w.keys, last_argmax);
    Q6W_LAUNCH_CHECK("prefill_argmax_kernel");
  }
  return Q6W_OK;
}

extern "C" int32_t q6w_forward_all(const q6w_model* M, int32_t n_prompts, const int32_t* prompts,
                                   const int32_t* prompt_lens, int32_t prompt_stride, int32_t max_prompt_len,
                                   int64_t total_tokens, float* k_cache, float* v_cache, int64_t cache_seq_stride,
                                   float* logits, const int32_t* targets, float* loss, void* workspace,
                                   size_t workspace_bytes, q6w_stream_t stream) {
  clear_error();
  if (!M) return fail(Q6W_ERR_ARG, "null model");
  if (n_prompts < 0 || total_tokens < 0) return fail(Q6W_ERR_ARG, "n_prompts and total_tokens must be >= 0");
  if (n_prompts == 0) return Q6W_OK;
  if (total_tokens < n_prompts || total_tokens > kMaxPrefillRows)
    return fail(Q6W_ERR_ARG, "total_tokens %lld must be in [n_prompts, %lld]", (long long)total_tokens,
                (long long)kMaxPrefillRows);
  if (!prompts || !prompt_lens || !logits) return fail(Q6W_ERR_ARG, "null prompts / prompt_lens / logits");
  if ((targets == nullptr) != (loss == nullptr)) return fail(Q6W_ERR_ARG, "targets and loss go together");
  if (max_prompt_len < 1 || max_prompt_len > M->d.max_seq_len || prompt_stride < max_prompt_len)
    return fail(Q6W_ERR_ARG, "need 1 <= max_prompt_len <= max_seq_len (%d) and prompt_stride >= max_prompt_len",
                M->d.max_seq_len);
  if (!aligned(logits, 16) || M->d.vocab_size % 4) return fail(Q6W_ERR_ALIGN, "logits must be 16-byte aligned");
  if (!workspace) return fail(Q6W_ERR_ARG, "null workspace");
  if (!aligned(workspace, 256)) return fail(Q6W_ERR_ALIGN, "workspace must be 256-byte aligned");
  const size_t need = prefill_layout(M, n_prompts, total_tokens, nullptr, nullptr, nullptr, nullptr);
  if (workspace_bytes < need)
    return fail(Q6W_ERR_ARG, "workspace of %zu bytes too small (%zu needed)", workspace_bytes, need);
  int32_t st;
  if ((st = check_cache(M, k_cache, v_cache, cache_seq_stride, n_prompts))) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != M->device) return fail(Q6W_ERR_ARG, "model was created on device %d, current is %d", M->device, dev);
  Work w;
  int32_t *seq, *off;
  prefill_layout(M, n_prompts, total_tokens, (char*)workspace, &w, &seq, &off);
  const int rows = (int)total_tokens;
  cudaStream_t s = (cudaStream_t)stream;
  prefill_scan_kernel<<<1, 1024, 0, s>>>(n_prompts, prompt_lens, max_prompt_len, off, w.err);
  Q6W_LAUNCH_CHECK("prefill_scan_kernel");
  prefill_rows_kernel<<<n_prompts < 4096 ? n_prompts : 4096, 256, 0, s>>>(
      n_prompts, rows, prompts, prompt_stride, prompt_lens, max_prompt_len, M->d.vocab_size, off, w, seq);
  Q6W_LAUNCH_CHECK("prefill_rows_kernel");
  w.seq = seq;
  w.poff = off;
  w.plens = prompt_lens;
  w.n_prompts = n_prompts;
  w.max_len = max_prompt_len;
  w.pdl = M->pdl_mode == 1;
  // every row through the layers and the vocab head (final RMSNorm + tied embedding): the logits of
  // every position, row off[i] + j for position j of prompt i
  EpiArgs v;
  memset(&v, 0, sizeof(v));
  v.y = logits;
  v.ldy = M->d.vocab_size;
  if ((st = enqueue_step(M, rows, w, k_cache, v_cache, cache_seq_stride, v, s, true))) return st;
  if (targets) {
    // per-row cross entropy into the (now unused) query buffer, row flags into gen
    row_nll_kernel<<<rows < 8192 ? rows : 8192, 256, 0, s>>>(rows, M->d.vocab_size, logits, targets, prompt_stride,
                                                             seq, w.pos, w.flags, w.qb, w.gen, w.err);
    Q6W_LAUNCH_CHECK("row_nll_kernel");
    mean_loss_kernel<<<1, 256, 0, s>>>(rows, w.qb, w.gen, loss);
    Q6W_LAUNCH_CHECK("mean_loss_kernel");
  }
  return Q6W_OK;
}

extern "C" int32_t q6w_generate(q6w_model* M, const q6w_greedy_args* a, const q6w_sample_args* sampling,
                                void* workspace, size_t workspace_bytes, q6w_stream_t stream) {
  clear_error();
  if (!M || !a) return fail(Q6W_ERR_ARG, "null argument");
  const int n = a->n_seqs;
  if (n < 0) return fail(Q6W_ERR_ARG, "n_seqs must be >= 0");
  if (n == 0) return Q6W_OK;
  if (!a->prompts || !a->prompt_lens || !a->sampled || !a->n_sampled || !a->stop_reason)
    return fail(Q6W_ERR_ARG, "null prompt/output pointer");
  if (a->max_prompt_len < 1 || a->prompt_stride < a->max_prompt_len)
    return fail(Q6W_ERR_ARG, "need 1 <= max_prompt_len <= prompt_stride");
  if (a->new_tokens < 1) return fail(Q6W_ERR_ARG, "new_tokens must be >= 1");
  if ((int64_t)a->max_prompt_len + a->new_tokens - 1 > M->d.max_seq_len)
    return fail(Q6W_ERR_RANGE, "prompt plus generated tokens exceeds the model context (%d)", M->d.max_seq_len);
  if (a->n_stop < 0 || a->n_stop > kMaxStop || (a->n_stop && !a->stop_ids))
    return fail(Q6W_ERR_ARG, "n_stop must be in [0, %d]", kMaxStop);
  if (a->min_new_tokens < 0 || a->min_new_tokens > a->new_tokens)
    return fail(Q6W_ERR_ARG, "min_new_tokens must be within the token limit");
  if (a->step_logits && !aligned(a->step_logits, 8)) return fail(Q6W_ERR_ALIGN, "step_logits must be 8-byte aligned");
  StopSet stop;
  memset(&stop, 0, sizeof(stop));
  stop.n = a->n_stop;
  stop.min_new = a->min_new_tokens;
  for (int i = 0; i < a->n_stop; ++i) {
    if (a->stop_ids[i] < 0 || a->stop_ids[i] >= M->d.vocab_size)
      return fail(Q6W_ERR_RANGE, "stop id %d outside the vocabulary", a->stop_ids[i]);
    stop.ids[i] = a->stop_ids[i];
  }
  smp::Params sp;
  bool sampler = false;
  int32_t st;
  if (sampling) {
    if ((st = make_sample_params(sampling, M->d.vocab_size, stop, &sp))) return st;
    sampler = needs_sampler(sp);
    if (sampler && sp.temperature != 0.0f && !sampling->seeds)
      return fail(Q6W_ERR_ARG, "sampling at temperature > 0 needs one seed per sequence");
    if (sampler && a->new_tokens > smp::kMaxHistory)
      return fail(Q6W_ERR_ARG, "sampling supports at most %d new tokens per request", smp::kMaxHistory);
    if (sampler && (st = sample_attr(M->d.vocab_size))) return st;
  }
  Work w;
  st = check_ws(M, n, workspace, workspace_bytes, &w, sampler);
  if (st) return st;
  if ((st = check_cache(M, a->k_cache, a->v_cache, a->cache_seq_stride, n))) return st;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != M->device) return fail(Q6W_ERR_ARG, "model was created on device %d, current is %d", M->device, dev);

  if (n == 1 && M->use_b1 && !sampler && !M->kv_half) {  // one greedy request: the cluster kernel runs the loop
    cudaStream_t s = (cudaStream_t)stream;
    b1::Args ba;
    b1_fill(M, ba);
    ba.prompt = a->prompts;
    ba.prompt_len = a->prompt_lens;
    ba.max_prompt_len = a->max_prompt_len;
    ba.new_tokens = a->new_tokens;
    ba.n_stop = stop.n;
    ba.min_new = stop.min_new;
    for (int i = 0; i < kMaxStop; ++i) ba.stop_ids[i] = stop.ids[i];
    ba.kc = a->k_cache;
    ba.vc = a->v_cache;
    ba.sampled = a->sampled;
    ba.n_sampled = a->n_sampled;
    ba.stop_reason = a->stop_reason;
    ba.step_logits = a->step_logits;
    ba.state = reinterpret_cast<int32_t*>(w.x);  // 5 ints of the (unused) residual-stream row
    ba.err = w.err;
    b1::b1_init_kernel<<<1, 32, 0, s>>>(a->prompts, a->prompt_lens, a->max_prompt_len, M->d.vocab_size, ba.state,
                                       a->n_sampled, a->stop_reason, w.err);
    Q6W_LAUNCH_CHECK("b1_init_kernel");
    const int total = a->max_prompt_len + a->new_tokens - 1;
    const int cuts[3] = {0, a->max_prompt_len, total};
    for (int part = 0; part < 2; ++part) {
      if (cuts[part + 1] > cuts[part]) {
        ba.step_begin = cuts[part];
        ba.step_end = cuts[part + 1];
        b1::b1_kernel<<<b1::kCtas, b1::kThreads, M->b1_smem, s>>>(ba);
        Q6W_LAUNCH_CHECK("b1_kernel");
      }
      if (part == 0 && a->prefill_event) Q6W_CUDA_TRY(cudaEventRecord((cudaEvent_t)a->prefill_event, s));
    }
    return Q6W_OK;
  }

  GraphKey key;
  memset(&key, 0, sizeof(key));
  key.a = *a;
  key.a.stop_ids = nullptr;
  key.a.prefill_event = nullptr;
  memcpy(key.stop, stop.ids, sizeof(key.stop));
  key.ws = workspace;
  key.sampler = sampler;
  if (sampler) key.sp = sp;
  if (!M->exec || !M->have_key || memcmp(&key, &M->key, sizeof(key)) != 0) {
    if ((st = capture_step(M, a, w, stop, sampler ? &sp : nullptr))) return st;
    M->key = key;
    M->have_key = true;
  }
  cudaStream_t s = (cudaStream_t)stream;
  init_greedy_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, a->prompts, a->prompt_lens, a->prompt_stride,
                                                      a->max_prompt_len, w, a->n_sampled, a->stop_reason,
                                                      sampler ? reinterpret_cast<const unsigned long long*>(
                                                                    sampling->seeds) : nullptr);
  Q6W_LAUNCH_CHECK("init_greedy_kernel");
  const int steps = a->max_prompt_len + a->new_tokens - 1;
  for (int i = 0; i < steps; ++i) {
    Q6W_CUDA_TRY(cudaGraphLaunch(M->exec, s));
    if (i + 1 == a->max_prompt_len && a->prefill_event)
      Q6W_CUDA_TRY(cudaEventRecord((cudaEvent_t)a->prefill_event, s));
  }
  return Q6W_OK;
}

extern "C" int32_t q6w_generate_greedy(q6w_model* M, const q6w_greedy_args* a, void* workspace,
                                       size_t workspace_bytes, q6w_stream_t stream) {
  return q6w_generate(M, a, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int32_t q6w_sample(const float* logits, int64_t ld, int32_t n, int32_t vocab, const int32_t* history,
                              int64_t history_ld, const int32_t* history_len, uint64_t* rng_state,
                              const q6w_sample_args* sampling, const int32_t* stop_ids, int32_t n_stop,
                              int32_t min_new_tokens, int32_t* tokens, q6w_stream_t stream) {
  clear_error();
  if (n < 0 || vocab < 2 || ld < vocab || history_ld < 0) return fail(Q6W_ERR_ARG, "q6w_sample: bad shape");
  if (!sampling) return fail(Q6W_ERR_ARG, "q6w_sample: null sampling arguments");
  if (n_stop < 0 || n_stop > kMaxStop || (n_stop && !stop_ids)) return fail(Q6W_ERR_ARG, "n_stop must be in [0, %d]", kMaxStop);
  if (n == 0) return Q6W_OK;
  if (!logits || !history_len || !rng_state || !tokens || (history_ld > 0 && !history))
    return fail(Q6W_ERR_ARG, "q6w_sample: null pointer");
  StopSet stop;
  memset(&stop, 0, sizeof(stop));
  stop.n = n_stop;
  stop.min_new = min_new_tokens;
  for (int i = 0; i < n_stop; ++i) stop.ids[i] = stop_ids[i];
  smp::Params sp;
  int32_t st = make_sample_params(sampling, vocab, stop, &sp);
  if (st) return st;
  if ((st = sample_attr(vocab))) return st;
  smp::Args sa;
  memset(&sa, 0, sizeof(sa));
  sa.logits = logits;
  sa.ld = ld;
  sa.vocab = vocab;
  sa.hist = history;
  sa.hist_ld = history_ld;
  sa.hist_len = history_len;
  sa.rng = reinterpret_cast<unsigned long long*>(rng_state);
  sa.tokens = tokens;
  sa.p = sp;
  smp::sample_kernel<<<n, smp::kThreads, smp::smem_bytes(vocab), (cudaStream_t)stream>>>(sa);
  Q6W_LAUNCH_CHECK("sample_kernel");
  return Q6W_OK;
}

extern "C" int32_t q6w_workspace_status(void* workspace, q6w_stream_t stream) {
  clear_error();
  if (!workspace) return fail(Q6W_ERR_ARG, "null workspace");
  cudaStream_t s = (cudaStream_t)stream;
  int32_t flag = 0;
  Q6W_CUDA_TRY(cudaMemcpyAsync(&flag, workspace, sizeof(flag), cudaMemcpyDeviceToHost, s));
  Q6W_CUDA_TRY(cudaStreamSynchronize(s));
  if (flag) {
    Q6W_CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(flag), s));
    Q6W_CUDA_TRY(cudaStreamSynchronize(s));
    if (flag & tc::kErrTimeout)
      return fail(Q6W_ERR_DEVICE, "a device-side wait ran out of time (error word 0x%x); the kernel stopped early",
                  flag);
    return fail(Q6W_ERR_DEVICE, "a kernel rejected a token, position or prompt length (sequence skipped)");
  }
  return Q6W_OK;
}

// One CTA waits on an mbarrier that no thread arrives at, through the
// bounded-wait routine every pipeline wait uses, limited to `cycles`; when it
// runs out the CTA records the timeout in the error word and returns.
__global__ void selftest_wait_kernel(uint64_t cycles, int32_t* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_for(&bar, 0, cycles)) atomicOr(err, tc::kErrTimeout);
}

extern "C" int32_t q6w_selftest_wait_timeout(void* workspace, int64_t wait_cycles, q6w_stream_t stream) {
  clear_error();
  if (!workspace || !aligned(workspace, 4)) return fail(Q6W_ERR_ARG, "q6w_selftest_wait_timeout: bad workspace");
  if (wait_cycles < 1 || wait_cycles > (int64_t(1) << 31))
    return fail(Q6W_ERR_ARG, "wait_cycles must be in [1, 2^31]");
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((uint64_t)wait_cycles, static_cast<int32_t*>(workspace));
  Q6W_LAUNCH_CHECK("selftest_wait_kernel");
  return Q6W_OK;
}

static int32_t attn_attr(int hd, int smem) {
  if (smem <= 48 * 1024) return Q6W_OK;
  cudaError_t e = cudaSuccess;
  switch (hd) {
    case 16: e = cudaFuncSetAttribute(attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 32: e = cudaFuncSetAttribute(attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 64: e = cudaFuncSetAttribute(attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 128: e = cudaFuncSetAttribute(attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 256: e = cudaFuncSetAttribute(attn_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 512: e = cudaFuncSetAttribute(attn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
  }
  if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
  return Q6W_OK;
}

extern "C" int32_t q6w_gqa_attention(const float* queries, const float* keys, const float* values,
                                     float* output, const int32_t* lengths, int32_t n,
                                     int32_t kv_heads, int32_t groups_per_kv, int32_t head_dim,
                                     int32_t max_len, int64_t kv_seq_stride, q6w_stream_t stream) {
  clear_error();
  if (n < 0 || kv_heads <= 0 || groups_per_kv <= 0 || max_len <= 0)
    return fail(Q6W_ERR_ARG, "q6w_gqa_attention: n >= 0, kv_heads, groups_per_kv, max_len > 0 required");
  if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512)
    return fail(Q6W_ERR_ARG, "head_dim %d unsupported (16, 32, 64, 128, 256 or 512)", head_dim);
  if (n == 0) return Q6W_OK;
  if (!queries || !keys || !values || !output || !lengths) return fail(Q6W_ERR_ARG, "q6w_gqa_attention: null pointer");
  if (!aligned(queries, 16) || !aligned(keys, 16) || !aligned(values, 16) || !aligned(output, 16))
    return fail(Q6W_ERR_ALIGN, "q6w_gqa_attention: tensors must be 16-byte aligned");
  const int64_t per = (int64_t)max_len * kv_heads * head_dim;
  if (n > 1 && (kv_seq_stride < per || kv_seq_stride % 4))
    return fail(Q6W_ERR_ARG, "kv_seq_stride must be >= max_len*kv_heads*head_dim and a multiple of 4");
  const int H = kv_heads * groups_per_kv;
  const int warps = H < 8 ? H : 8;
  const size_t smem = (size_t)warps * max_len * sizeof(float);
  if (smem > 200 * 1024) return fail(Q6W_ERR_ARG, "max_len %d too large", max_len);
  int32_t st = attn_attr(head_dim, (int)smem);
  if (st) return st;
  const dim3 grid(n, (H + warps - 1) / warps);
  const float denom = (float)sqrt((double)head_dim);
  cudaStream_t s = (cudaStream_t)stream;
  const int ld = H * head_dim;
  if (launch_attn_rows(head_dim, kv_heads, groups_per_kv, grid, s, queries, ld, keys, values, kv_seq_stride, 0,
                       lengths, 0, nullptr, output, ld, max_len, denom)) {
    Q6W_LAUNCH_CHECK("attn_rows_kernel");
    return Q6W_OK;
  }
  attn_group_setup();
  if (launch_attn_head(head_dim, n, H, kv_heads, s, queries, ld, keys, values, kv_seq_stride, 0, lengths, 0, nullptr,
                       output, ld, max_len, denom)) {
    Q6W_LAUNCH_CHECK("attn_head_kernel");
    return Q6W_OK;
  }
  switch (head_dim) {
#define Q6W_ATTN2(HDV)                                                                               \
  case HDV:                                                                                          \
    attn_kernel<HDV / 16><<<grid, warps * 32, smem, s>>>(queries, ld, keys, values, kv_seq_stride, 0, \
                                                         lengths, 0, nullptr, output, ld, H,         \
                                                         kv_heads, max_len, denom, nullptr);         \
    break;
    Q6W_ATTN2(16) Q6W_ATTN2(32) Q6W_ATTN2(64) Q6W_ATTN2(128) Q6W_ATTN2(256) Q6W_ATTN2(512)
#undef Q6W_ATTN2
  }
  Q6W_LAUNCH_CHECK("attn_kernel");
  return Q6W_OK;
}

// ---- q6w_linear_ex: the batched linear on tensor cores ---------------------------
//
// For n >= 16 activation rows of a matrix whose width is a multiple of 128 (at
// most 8192), x is written once as the three-part bf16 activation image (in
// the caller's workspace) and a tcgen05 kernel runs with a plain store
// epilogue: the persistent dim-128 kernel (tc.cuh; activations as the MMA's
// 128-row M operand, weight tiles of 64-256 rows) when a weight tile with all
// of K fits its staging area (K = 128 or 384 and the like), else the general
// kernel (tcg.cuh; weights as M, split K across clusters).  Other shapes and
// smaller n take q6w_linear's kernels.

static bool linear_tc_ok(int64_t rows, int64_t cols, int64_t n) {
  return n >= tcg_min_rows() && rows >= 2 && rows % 2 == 0 && cols % 128 == 0 && cols <= tcg::kImgMaxK &&
         rows <= (1 << 24) && n <= (1 << 24);
}

// Per device: kernel attributes and the resident-cluster counts, set once.
static int32_t linear_tc_setup() {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  Q6W_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(Q6W_ERR_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    int major = 0;
    Q6W_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return fail(Q6W_ERR_ARG, "the tensor-core linear needs an sm_100 device");
    const cudaError_t e = tcg_set_attrs();
    if (e != cudaSuccess) return fail(Q6W_ERR_CUDA, "tensor-core linear attributes: %s", cudaGetErrorString(e));
    int32_t st = tc_set_attrs();
    if (st) return st;
    done[dev] = true;
  }
  return Q6W_OK;
}

extern "C" size_t q6w_linear_workspace_bytes(int64_t rows, int64_t cols, int64_t n) {
  if (rows < 0 || cols < 0 || n < 0 || !linear_tc_ok(rows, cols, n)) return 0;
  return 256 + tc::img_bytes(n, (int)cols);  // the error word (offset 0), then the activation image
}

extern "C" int32_t q6w_linear_ex(const uint8_t* packed, const float* scales, const float* x, float* y, int64_t rows,
                                 int64_t cols, int64_t n, void* workspace, size_t workspace_bytes,
                                 q6w_stream_t stream) {
  clear_error();
  if (rows < 0 || cols < 0 || n < 0) return fail(Q6W_ERR_ARG, "q6w_linear_ex: negative shape");
  if (!workspace || !linear_tc_ok(rows, cols, n) || !aligned(packed, 16) || !aligned(scales, 4) ||
      !aligned(x, 16) || !aligned(y, 8))
    return q6w_linear(packed, scales, x, y, rows, cols, n, stream);
  if (!packed || !scales || !x || !y) return fail(Q6W_ERR_ARG, "q6w_linear_ex: null pointer");
  const size_t need = q6w_linear_workspace_bytes(rows, cols, n);
  if (workspace_bytes < need)
    return fail(Q6W_ERR_ARG, "q6w_linear_ex: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(Q6W_ERR_ALIGN, "q6w_linear_ex: workspace must be 256-byte aligned");
  int32_t st = linear_tc_setup();
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // error word at offset 0 (q6w_workspace_status reads it), the image from byte 256
  int32_t* err = static_cast<int32_t*>(workspace);
  uint8_t* img = static_cast<uint8_t*>(workspace) + 256;
  const int tile = tc::store_tile_rows(rows, cols);
  if (tile && aligned(y, 16) && aligned(packed, 16) && aligned(scales, 16)) {
    if ((st = tcg_image(x, (int)cols, (int)n, (int)cols, nullptr, 0.f, img, s, false))) return st;
    tc::TcArgs t;
    memset(&t, 0, sizeof(t));
    t.a_img = img;
    t.n = (int)n;
    t.K = (int)cols;
    t.q0 = packed;
    t.s0 = scales;
    t.end0 = t.end1 = (int32_t)rows;
    t.N = tile;
    t.n_tiles = (int32_t)(rows / tile);
    t.ep.y = y;
    t.ep.ldy = (int32_t)rows;
    t.err = err;
    return tc_launch(tc::TEPI_STORE, t, sm_count(), s);
  }
  if ((st = tcg_image(x, (int)cols, (int)n, (int)cols, nullptr, 0.f, img, s))) return st;
  tcg::GArgs a;
  memset(&a, 0, sizeof(a));
  a.img = img;
  a.n = (int)n;
  a.K = (int)cols;
  a.err = err;
  a.ms = {packed, nullptr, nullptr, scales, nullptr, nullptr, (int32_t)rows, (int32_t)rows, (int32_t)cols, 0,
          (int32_t)(rows / 2)};
  a.ep.y = y;
  a.ep.ldy = (int32_t)rows;
  return tcg_launch(tcg::GEPI_STORE, a, sm_count(), s);
}
