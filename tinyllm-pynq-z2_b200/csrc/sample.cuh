// Sampling on the device: the logit processors and the sampler of
// benchmarks/torch_benchmark.py -- penalize_repeated_tokens (:188-198),
// block_repeated_ngrams (:211-230), the stop-id masking / bias of generate
// (:277-283, bias_stop_tokens :201-208), and sample_token with XorShift64
// (:133-185) -- one CTA of kThreads per sequence over its logits row.
//
// Exactness.  The processors use the reference's FP32 operations (the
// Python-float parameters rounded to FP32 first, as torch does for a float32
// tensor and a Python scalar).  The softmax is max, exp(z - max), an FP32
// sum and a multiply by its reciprocal -- the same steps, but expf and the
// summation order are CUDA's, so probabilities can differ from torch CPU's
// in the last bits.
//
// Nucleus (0 < top_p < 1) without a sort.  The reference sorts the
// probabilities in descending order, keeps those >= cutoff = (1 - top_p) /
// (V - 1), accumulates them in FP64 until the sum exceeds top_p, scales the
// coin by that sum and walks the kept list again.  Every kept value is a
// float32 >= cutoff; when cutoff >= 2^-29 (any top_p <= 1 - 2^-29 (V - 1))
// such values lie on the 2^-52 grid and their partial sums stay below 2, so
// every FP64 sum of them is exact: the same in any order.  The crossing of a
// running sum in descending order is then found by a radix select over the
// float bit patterns (the exponent, then the significand in passes of 8 + 8
// + 7 bits, a histogram of exact fixed-point sums per pass): the largest
// value v with sum_{p >= v} p > T.  The exponent pass is shared by the two
// selections (the top-p crossing, then the coin's) and gives the kept total.  Equal values (a tie group) are taken in ascending
// token order; the reference's unstable sort may order such a group
// differently, which changes the pick only when it lands in the group.
//
// Plain scan (top_p <= 0 or >= 1): the cumulative FP64 sum in token order is
// a block-wide prefix sum (per-thread chunks summed in order, then an
// exclusive scan); it can round differently from the sequential sum only
// when values below 2^-29 are added, by at most V * 2^-53.
#pragma once

#include "linear.cuh"

namespace q6w {
namespace smp {

constexpr int kThreads = 512;
constexpr int kMaxVocab = 32768;
constexpr int kMaxHistory = 4096;

struct Params {
  float temperature;         // float32 of the reference's value; 0: argmax of the processed logits
  float repetition_penalty;  // 1: off
  float stop_bias;           // added to stop-id logits from index bias_after on (0: off)
  float cutoff;              // float32((1 - top_p) / (vocab - 1))
  double top_p;
  int32_t nucleus;           // 0 < top_p < 1
  int32_t ngram;             // no_repeat_ngram_size (0: off)
  int32_t bias_after;
  int32_t min_new;
  int32_t n_stop;
  int32_t stop_ids[kMaxStop];
};

struct Args {
  const float* logits;       // row b at logits + b * ld
  int64_t ld;
  int32_t vocab;
  const int32_t* hist;       // generated tokens of sequence b at hist + b * hist_ld
  int64_t hist_ld;
  const int32_t* hist_len;   // tokens generated so far = the decode index
  unsigned long long* rng;   // XorShift64 state per sequence (read and advanced)
  int32_t* tokens;           // output (standalone op), or
  unsigned long long* keys;  // output in argmax-key form (generation loop)
  const int32_t* flags;      // generation loop: skip finished / invalid sequences and prompt steps
  const int32_t* pos;
  const int32_t* plen;
  Params p;
};

__host__ __device__ inline size_t smem_bytes(int vocab) {
  return (size_t)vocab * 4 + (size_t)kMaxHistory * 4 + (size_t)(vocab + 31) / 32 * 4 + 256 * 28 + 1024;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block reductions (every thread gets the result).
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T t = red[0];
  for (int i = 1; i < nw; ++i) t = op(t, red[i]);
  return t;
}

// Exclusive prefix of per-thread values in thread order (double).
__device__ __forceinline__ double block_exclusive_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  double before = 0.0;
  for (int i = 0; i < warp; ++i) before += red[i];
  (void)nw;
  return before + x - v;
}

__device__ __forceinline__ float xorshift_coin(unsigned long long& s) {
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  const unsigned long long value = s * 0x2545F4914F6CDD1Dull;
  return (float)(uint32_t)(value >> 40) * (1.0f / 16777216.0f);  // (u32 >> 8) / 2^24, exact
}

// Exact sums of kept probabilities in 2^-52 fixed point.  A float32 p >= 2^-29
// is an integer multiple of 2^-52 and the kept values sum to about 1, so
// p * 2^52 and every sum of kept values are exact integers below 2^53: the
// FP64 sums the reference forms, exact in any order.  Per histogram bin all
// values share one exponent e, so a bin holds the integer sum S of their
// 24-bit significands M (p = M * 2^(e - 150)) and its fixed-point sum is
// S * 2^(e - 98).  S is accumulated as two 32-bit halves (sums of M >> 12 and
// of M & 0xFFF, each below 2^27 for up to 32768 values) with native 32-bit
// shared-memory atomics.  Below 2^-29 (a cutoff under 2^-29) the scaling
// truncates, by less than 2^-52 a value.
__device__ __forceinline__ unsigned long long fix52(float p) {
  return (unsigned long long)((double)p * 4503599627370496.0);
}
// S > T for a fixed-point S  <=>  S > floor(T * 2^52)  (T * 2^52 is exact in FP64).
__device__ __forceinline__ unsigned long long fix52_floor(double T) {
  return (unsigned long long)floor(T * 4503599627370496.0);
}
__device__ __forceinline__ double unfix52(unsigned long long s) { return (double)s * (1.0 / 4503599627370496.0); }
__device__ __forceinline__ unsigned long long scale_exp(unsigned long long S, int e) {
  const int k = e - 98;
  return k >= 0 ? (k < 64 ? S << k : 0ull) : (k > -64 ? S >> -k : 0ull);
}

// Shared histogram of one radix pass (256 bins) and the saved exponent pass.
struct Hist {
  uint32_t* hi;               // sum of M >> 12 per bin
  uint32_t* lo;               // sum of M & 0xFFF per bin
  int* cnt;                   // values per bin
  unsigned long long* sum0;   // exponent pass: fixed-point sum per exponent
  int* cnt0;
};

// One pass over the row: candidates (p >= cutoff) whose bits under mask equal
// prefix, binned by (bits >> sh) & (nb - 1).  Strided over the threads (order
// is free: the sums are exact).
__device__ __forceinline__ void hist_pass(const float* p, int V, float cutoff, uint32_t prefix, uint32_t mask, int sh,
                                          int nb, const Hist& h) {
  for (int t = threadIdx.x; t < V; t += blockDim.x) {
    const float v = p[t];
    const uint32_t u = __float_as_uint(v);
    if (!(v >= cutoff) || (u & mask) != prefix) continue;
    const uint32_t m = (u & 0x7FFFFFu) | 0x800000u;
    const int bin = (int)((u >> sh) & (uint32_t)(nb - 1));
    atomicAdd(h.hi + bin, m >> 12);
    atomicAdd(h.lo + bin, m & 0xFFFu);
    atomicAdd(h.cnt + bin, 1);
  }
}

__device__ __forceinline__ void hist_clear(const Hist& h) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    h.hi[i] = 0u;
    h.lo[i] = 0u;
    h.cnt[i] = 0;
  }
}

// The exponent pass, shared by both selections: fixed-point sum and count of
// the candidates per exponent; returns the total of the kept values (fixed
// point) to every thread.
__device__ unsigned long long exponent_pass(const float* p, int V, float cutoff, const Hist& h) {
  __shared__ unsigned long long s_total;
  hist_clear(h);
  __syncthreads();
  hist_pass(p, V, cutoff, 0u, 0u, 23, 256, h);
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long part = 0ull;
    for (int bin = threadIdx.x; bin < 256; bin += 32) {
      const unsigned long long s = scale_exp(((unsigned long long)h.hi[bin] << 12) + h.lo[bin], bin);
      h.sum0[bin] = s;
      h.cnt0[bin] = h.cnt[bin];
      part += s;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (threadIdx.x == 0) s_total = part;
  }
  __syncthreads();
  return s_total;
}

// Largest candidate value v with sum_{cand p >= v} p > T, with G = the sum of
// candidates above v and k = the 1-based position inside v's tie group where
// the running sum first exceeds T.  Candidates: p >= cutoff.  Tf =
// fix52_floor(T); sums are fixed point.  Requires exponent_pass first.
struct Sel {
  float v;
  unsigned long long G;
  int k;
  unsigned long long cum;  // G + k v
};

// Warp 0: walk the nb bins from the top, accumulating bin sums onto acc0, and
// take the first bin where the running sum exceeds Tf.  lane l holds bins
// nb-1-q*l .. nb-q(l+1) (q = nb / 32).
template <typename BinSum>
__device__ __forceinline__ void pick_bin(int nb, unsigned long long acc0, unsigned long long Tf, BinSum bin_sum,
                                         int* chosen_out, unsigned long long* acc_out) {
  const int lane = threadIdx.x & 31, q = nb / 32;
  unsigned long long mine = 0ull;
  for (int i = 0; i < q; ++i) mine += bin_sum(nb - 1 - q * lane - i);
  unsigned long long incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const unsigned ball = __ballot_sync(0xffffffffu, acc0 + incl > Tf);
  const int L = ball ? __ffs(ball) - 1 : 31;  // a crossing exists whenever Tf < the candidates' total
  if (lane == L) {
    unsigned long long acc = acc0 + incl - mine;
    int chosen = nb - q * (L + 1);
    for (int i = 0; i < q; ++i) {
      const int bin = nb - 1 - q * L - i;
      const unsigned long long s = bin_sum(bin);
      if (acc + s > Tf) {
        chosen = bin;
        break;
      }
      acc += s;
    }
    *chosen_out = chosen;
    *acc_out = acc;
  }
}

__device__ Sel radix_select(const float* p, int V, float cutoff, unsigned long long Tf, const Hist& h) {
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ unsigned long long s_acc;
  __shared__ int s_cnt, s_bin;
  __syncthreads();  // every thread has read the previous call's result
  if (threadIdx.x < 32) {
    pick_bin(256, 0ull, Tf, [&](int bin) { return h.sum0[bin]; }, &s_bin, &s_acc);
    __syncwarp();
    if (threadIdx.x == 0) {
      s_cnt = h.cnt0[s_bin];
      s_prefix = (uint32_t)s_bin << 23;
      s_mask = 0xFFu << 23;
    }
  }
  __syncthreads();
  // significand bits 22..15, 14..7, 6..0 inside the chosen exponent
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = pass < 2 ? 15 - 8 * pass : 0, nb = pass < 2 ? 256 : 128;
    hist_clear(h);
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    hist_pass(p, V, cutoff, prefix, mask, sh, nb, h);
    __syncthreads();
    if (threadIdx.x < 32) {
      const int e = (int)(prefix >> 23);
      pick_bin(nb, s_acc, Tf,
               [&](int bin) { return scale_exp(((unsigned long long)h.hi[bin] << 12) + h.lo[bin], e); }, &s_bin,
               &s_acc);
      __syncwarp();
      if (threadIdx.x == 0) {
        s_cnt = h.cnt[s_bin];
        s_prefix = prefix | ((uint32_t)s_bin << sh);
        s_mask = mask | ((uint32_t)(nb - 1) << sh);
      }
    }
    __syncthreads();
  }
  Sel r;
  r.v = __uint_as_float(s_prefix);
  r.G = s_acc;
  const unsigned long long vf = fix52(r.v);
  unsigned long long s = r.G;
  int k = 0;
  const int cnt = s_cnt;
  do {
    s += vf;
    ++k;
  } while (s <= Tf && k < cnt);
  r.k = k;
  r.cum = s;
  return r;
}

// Index of the k-th (1-based) token, in ascending order, whose value equals v.
__device__ int kth_equal(const float* p, int V, float v, int k, double* red, int* ired) {
  if (k == 1) {  // the usual case: the first equal value
    int found = 0x7fffffff;
    for (int t = threadIdx.x; t < V; t += blockDim.x)
      if (p[t] == v) {
        found = t;
        break;
      }
    return block_reduce<int>(found, ired, [](int a, int b) { return a < b ? a : b; });
  }
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per, b1 = min(V, b0 + per);
  int c = 0;
  for (int t = b0; t < b1; ++t) c += p[t] == v;
  const double before = block_exclusive_d((double)c, red);
  int found = 0x7fffffff;
  int run = (int)before;
  for (int t = b0; t < b1; ++t)
    if (p[t] == v && ++run == k) found = t;
  return block_reduce<int>(found, ired, [](int a, int b) { return a < b ? a : b; });
}

__global__ void __launch_bounds__(kThreads) sample_kernel(Args a) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  __shared__ float redf[32];
  __shared__ double redd[32];
  __shared__ int redi[32];
  __shared__ unsigned long long redk[32];
  __shared__ float s_coin;
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  if (a.flags) {
    const int f = a.flags[b];
    if (f & (SEQ_DONE | SEQ_INVALID)) return;
    if (a.pos[b] < a.plen[b] - 1) return;  // still inside the prompt: nothing is sampled
  }
  const int V = a.vocab;
  float* l = reinterpret_cast<float*>(sm_raw);
  int32_t* hist = reinterpret_cast<int32_t*>(sm_raw + (size_t)V * 4);
  uint32_t* ban = reinterpret_cast<uint32_t*>(sm_raw + (size_t)V * 4 + (size_t)kMaxHistory * 4);
  Hist h;
  h.sum0 = reinterpret_cast<unsigned long long*>(sm_raw + (size_t)V * 4 + (size_t)kMaxHistory * 4 +
                                                  ((size_t)(V + 31) / 32 * 4 + 7) / 8 * 8);
  h.hi = reinterpret_cast<uint32_t*>(h.sum0 + 256);
  h.lo = h.hi + 256;
  h.cnt = reinterpret_cast<int*>(h.lo + 256);
  h.cnt0 = h.cnt + 256;
  const Params& P = a.p;
  const int g = a.hist_len[b];
  const int gh = g < kMaxHistory ? g : kMaxHistory;
  const float* row = a.logits + (int64_t)b * a.ld;
  for (int t = threadIdx.x; t < V; t += blockDim.x) l[t] = row[t];
  for (int i = threadIdx.x; i < gh; i += blockDim.x) hist[i] = a.hist[(int64_t)b * a.hist_ld + i];
  __syncthreads();

  // ---- repetition penalty on each distinct generated token (torch_benchmark.py:188-198)
  if (P.repetition_penalty != 1.0f && gh > 0) {
    // once per distinct token: the thread that sets the token's bit applies it
    const int words = (V + 31) / 32;
    for (int i = threadIdx.x; i < words; i += blockDim.x) ban[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < gh; i += blockDim.x) {
      const int t = hist[i];
      if (t < 0 || t >= V) continue;
      const uint32_t bit = 1u << (t & 31);
      if (atomicOr(ban + (t >> 5), bit) & bit) continue;
      const float v = l[t];
      l[t] = v < 0.0f ? __fmul_rn(v, P.repetition_penalty) : __fdiv_rn(v, P.repetition_penalty);
    }
    __syncthreads();
  }

  // ---- n-gram blocking (torch_benchmark.py:211-230)
  if (P.ngram > 0 && gh > 0 && (P.ngram == 1 || gh >= P.ngram - 1)) {
    const int words = (V + 31) / 32;
    for (int i = threadIdx.x; i < words; i += blockDim.x) ban[i] = 0u;
    __syncthreads();
    int any = 0;
    if (P.ngram == 1) {
      for (int i = threadIdx.x; i < gh; i += blockDim.x) {
        const int t = hist[i];
        if (t >= 0 && t < V) {
          atomicOr(ban + (t >> 5), 1u << (t & 31));
          any = 1;
        }
      }
    } else {
      const int n1 = P.ngram - 1, base = gh - n1;
      for (int i = threadIdx.x; i <= gh - P.ngram; i += blockDim.x) {
        bool match = true;
        for (int k = 0; k < n1 && match; ++k) match = hist[i + k] == hist[base + k];
        const int t = hist[i + n1];
        if (match && t >= 0 && t < V) {
          atomicOr(ban + (t >> 5), 1u << (t & 31));
          any = 1;
        }
      }
    }
    any = block_reduce<int>(any, redi, [](int x, int y) { return x | y; });
    if (any) {
      // banned tokens become -inf unless that leaves no finite logit at all
      int fin = 0;
      for (int t = threadIdx.x; t < V; t += blockDim.x)
        fin |= !((ban[t >> 5] >> (t & 31)) & 1u) && isfinite(l[t]);
      fin = block_reduce<int>(fin, redi, [](int x, int y) { return x | y; });
      if (fin)
        for (int t = threadIdx.x; t < V; t += blockDim.x)
          if ((ban[t >> 5] >> (t & 31)) & 1u) l[t] = -INFINITY;
    }
    __syncthreads();
  }

  // ---- stop ids: masked before min_new_tokens, biased from bias_after on (:277-283)
  if (P.n_stop && threadIdx.x == 0) {
    for (int s = 0; s < P.n_stop; ++s) {
      const int t = P.stop_ids[s];
      if (t < 0 || t >= V) continue;
      if (g < P.min_new)
        l[t] = -INFINITY;
      else if (g >= P.bias_after && P.stop_bias != 0.0f)
        l[t] = __fadd_rn(l[t], P.stop_bias);
    }
  }
  __syncthreads();

  int token;
  if (P.temperature == 0.0f) {
    // argmax, first maximum (torch.argmax)
    unsigned long long key = 0ull;
    for (int t = threadIdx.x; t < V; t += blockDim.x) key = umax64(key, argmax_key(l[t], t));
    key = block_reduce<unsigned long long>(key, redk, [](unsigned long long x, unsigned long long y) {
      return x > y ? x : y;
    });
    token = argmax_index(key);
  } else {
    if (threadIdx.x == 0) {
      unsigned long long s = a.rng[b];
      s_coin = xorshift_coin(s);
      a.rng[b] = s;
    }
    // softmax(logits / temperature): max, exp(z - max), FP32 sum, times 1/sum
    float m = -INFINITY;
    for (int t = threadIdx.x; t < V; t += blockDim.x) {
      const float z = __fdiv_rn(l[t], P.temperature);
      l[t] = z;
      m = fmaxf(m, z);
    }
    m = block_reduce<float>(m, redf, [](float x, float y) { return fmaxf(x, y); });
    float sum = 0.0f;
    for (int t = threadIdx.x; t < V; t += blockDim.x) {
      const float e = expf(__fsub_rn(l[t], m));
      l[t] = e;
      sum = __fadd_rn(sum, e);
    }
    sum = block_reduce<float>(sum, redf, [](float x, float y) { return __fadd_rn(x, y); });
    const float inv = __fdiv_rn(1.0f, sum);
    for (int t = threadIdx.x; t < V; t += blockDim.x) l[t] = __fmul_rn(l[t], inv);
    __syncthreads();
    const double coin = (double)s_coin;
    const int per = (V + blockDim.x - 1) / blockDim.x;
    const int b0 = threadIdx.x * per, b1 = min(V, b0 + per);
    if (!P.nucleus) {
      // cumulative sum in token order; first token whose running sum exceeds the coin
      double cs = 0.0;
      for (int t = b0; t < b1; ++t) cs += (double)l[t];
      double run = block_exclusive_d(cs, redd);
      int found = 0x7fffffff;
      for (int t = b0; t < b1; ++t) {
        run += (double)l[t];
        if (coin < run) {
          found = t;
          break;
        }
      }
      found = block_reduce<int>(found, redi, [](int x, int y) { return x < y ? x : y; });
      token = found == 0x7fffffff ? V - 1 : found;
    } else {
      const unsigned long long tot = exponent_pass(l, V, P.cutoff, h);
      const unsigned long long top = fix52_floor(P.top_p);
      double cum_last;
      if (tot > top) {
        cum_last = unfix52(radix_select(l, V, P.cutoff, top, h).cum);
      } else {
        cum_last = unfix52(tot);  // the whole kept list (the reference's last_index = len - 1)
      }
      const double target = coin * cum_last;
      const Sel s = radix_select(l, V, P.cutoff, fix52_floor(target), h);
      token = kth_equal(l, V, s.v, s.k, redd, redi);
      if (token == 0x7fffffff) token = V - 1;  // not reached: the select always lands on a kept value
    }
  }
  if (threadIdx.x == 0) {
    if (a.tokens) a.tokens[b] = token;
    if (a.keys) a.keys[b] = (1ull << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)token);
  }
}

}  // namespace smp
}  // namespace q6w
