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
// float bit patterns (31 value bits in passes of 7 + 8 + 8 + 8 bits, a
// histogram of FP64 sums per pass): the largest value v with
// sum_{p >= v} p > T.  Equal values (a tie group) are taken in ascending
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
  return (size_t)vocab * 4 + (size_t)kMaxHistory * 4 + (size_t)(vocab + 31) / 32 * 4 + 256 * 12 + 1024;
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

// Largest candidate value v with sum_{cand p >= v} p > T, with G = the sum of
// candidates above v and k = the 1-based position inside v's tie group where
// the running sum first exceeds T.  Candidates: p >= cutoff.
struct Sel {
  float v;
  double G;
  int k;
  double cum;  // G + k v
};

__device__ Sel radix_select(const float* p, int V, float cutoff, double T, double* hsum, int* hcnt, double* red) {
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ double s_acc;
  __shared__ int s_cnt;
  __syncthreads();  // every thread has read the previous call's result
  if (threadIdx.x == 0) {
    s_prefix = 0u;
    s_mask = 0u;
    s_acc = 0.0;
  }
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per, b1 = min(V, b0 + per);
  const int shifts[4] = {24, 16, 8, 0}, widths[4] = {7, 8, 8, 8};
  for (int pass = 0; pass < 4; ++pass) {
    const int sh = shifts[pass], nb = 1 << widths[pass];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      hsum[i] = 0.0;
      hcnt[i] = 0;
    }
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    int cur = -1, cn = 0;
    double cs = 0.0;
    for (int t = b0; t < b1; ++t) {
      const float v = p[t];
      const uint32_t u = __float_as_uint(v);
      if (!(v >= cutoff) || (u & mask) != prefix) continue;
      const int bin = (int)((u >> sh) & (uint32_t)(nb - 1));
      if (bin != cur) {
        if (cur >= 0) {
          atomicAdd(hsum + cur, cs);
          atomicAdd(hcnt + cur, cn);
        }
        cur = bin;
        cs = 0.0;
        cn = 0;
      }
      cs += (double)v;
      ++cn;
    }
    if (cur >= 0) {
      atomicAdd(hsum + cur, cs);
      atomicAdd(hcnt + cur, cn);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double acc = s_acc;
      int chosen = 0;
      for (int bin = nb - 1; bin >= 0; --bin) {
        if (acc + hsum[bin] > T) {
          chosen = bin;
          break;
        }
        acc += hsum[bin];
      }
      s_acc = acc;
      s_cnt = hcnt[chosen];
      s_prefix = prefix | ((uint32_t)chosen << sh);
      s_mask = mask | ((uint32_t)(nb - 1) << sh);
    }
    __syncthreads();
  }
  Sel r;
  r.v = __uint_as_float(s_prefix);
  r.G = s_acc;
  double s = r.G;
  int k = 0;
  const int cnt = s_cnt;
  do {
    s += (double)r.v;
    ++k;
  } while (s <= T && k < cnt);
  r.k = k;
  r.cum = s;
  (void)red;
  return r;
}

// Index of the k-th (1-based) token, in ascending order, whose value equals v.
__device__ int kth_equal(const float* p, int V, float v, int k, double* red, int* ired) {
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
  double* hsum = reinterpret_cast<double*>(sm_raw + (size_t)V * 4 + (size_t)kMaxHistory * 4 +
                                           ((size_t)(V + 31) / 32 * 4 + 7) / 8 * 8);
  int* hcnt = reinterpret_cast<int*>(hsum + 256);
  const Params& P = a.p;
  const int g = a.hist_len[b];
  const int gh = g < kMaxHistory ? g : kMaxHistory;
  const float* row = a.logits + (int64_t)b * a.ld;
  for (int t = threadIdx.x; t < V; t += blockDim.x) l[t] = row[t];
  for (int i = threadIdx.x; i < gh; i += blockDim.x) hist[i] = a.hist[(int64_t)b * a.hist_ld + i];
  __syncthreads();

  // ---- repetition penalty on each distinct generated token (torch_benchmark.py:188-198)
  if (P.repetition_penalty != 1.0f && gh > 0) {
    for (int i = threadIdx.x; i < gh; i += blockDim.x) {
      const int t = hist[i];
      bool first = t >= 0 && t < V;
      for (int j = 0; j < i && first; ++j) first = hist[j] != t;
      if (first) {
        const float v = l[t];
        l[t] = v < 0.0f ? __fmul_rn(v, P.repetition_penalty) : __fdiv_rn(v, P.repetition_penalty);
      }
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
      double tot = 0.0;
      for (int t = b0; t < b1; ++t)
        if (l[t] >= P.cutoff) tot += (double)l[t];
      tot = block_reduce<double>(tot, redd, [](double x, double y) { return x + y; });
      double cum_last;
      if (tot > P.top_p) {
        cum_last = radix_select(l, V, P.cutoff, P.top_p, hsum, hcnt, redd).cum;
      } else {
        cum_last = tot;  // the whole kept list (the reference's last_index = len - 1)
      }
      const double target = coin * cum_last;
      const Sel s = radix_select(l, V, P.cutoff, target, hsum, hcnt, redd);
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
