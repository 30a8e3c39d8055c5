// Tensor-core (tcgen05) path for the batched step: n >= 64 sequences of a
// model with dim 128.
//
// GEMM shape per CTA: D[128 sequences, N weight rows] += A[128, K] . B[N, K]^T
// with A = activations, B = Q6W weights, both bf16 K-major in shared memory
// with the 128-byte swizzle, D in FP32 in tensor memory (TMEM).
//
// Exactness.  A Q6W code is an integer in [-32, 31]: exact in bf16.  An FP32
// activation u is carried as three bf16 parts u = hi + mid + lo (each part the
// bf16 rounding of what the previous parts left; together they hold u's 24-bit
// significand), so sum_k q_k u_k is formed from exact products with FP32
// accumulation -- three MMAs per K step instead of one.  The row scale is
// applied once in the epilogue: y = scale * sum_k q_k u_k.
//
// Activation images.  Producers (embed, attention, the wo / w2 / W1-W3
// epilogues) write the next GEMM's A operand directly as a pre-swizzled tile
// image: for 128-row tile t, part p, 64-column chunk c, row r, the 128 bytes
// of the row are eight 16-byte units stored at unit index (u ^ (r & 7)) --
// the byte image of the UMMA K-major SWIZZLE_128B canonical layout -- so a
// CTA copies a whole A tile into shared memory with contiguous vector loads.
//
// Weights are expanded from the packed int6 rows into the same layout in
// shared memory by the CTA itself (three 32-bit loads -> 16 bf16 codes).
//
// Tiles.  An item is (128-sequence M tile, N-row weight tile).  QKV uses two
// 128-row tiles (q | k v) when the rows divide, GLU tiles of 64 W1 + 64 W3
// rows, VOCAB 256 rows; at small batches (few M tiles) QKV and GLU narrow to
// 64-row tiles so more SMs take part.  RESNORM needs whole rows for its
// RMSNorm and runs each M tile either in one CTA (N = 128) or, when every M
// tile can have two (four) CTAs at once, as a 2-CTA (4-CTA) cluster of 64-
// (32-) column blocks that add their per-row sums of squares through
// distributed shared memory.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "async.cuh"
#include "linear.cuh"

namespace q6w {
namespace tc {

constexpr int kM = 128;             // sequences per tile (MMA M, TMEM lanes)
constexpr int kKC = 128;            // K per shared-memory stage
constexpr int kThreads = 256;       // 8 warps; warps w and w+4 share TMEM lanes 32(w%4).. (sequence rows), splitting the columns
constexpr int kErrTimeout = 4;      // workspace error bit: an MMA wait timed out

// ---- image addressing ---------------------------------------------------------

// Byte offset, inside an activation image of K columns, of element (row, part, k).
__host__ __device__ __forceinline__ int64_t img_offset(int64_t row, int part, int k, int K) {
  const int64_t tile = row >> 7;
  const int r = (int)(row & 127);
  const int c = k >> 6, u = (k & 63) >> 3;
  return tile * (3 * (int64_t)K * 256) + (int64_t)part * K * 256 + (int64_t)c * 16384 + r * 128 +
         ((u ^ (r & 7)) << 4) + ((k & 7) << 1);
}

__host__ __device__ inline size_t img_bytes(int64_t n, int K) {
  return (size_t)((n + 127) / 128) * 3 * (size_t)K * 256;
}

__device__ __forceinline__ uint32_t bf16_bits_rn(float x) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// u -> (hi, mid, lo) bf16 bit patterns, each the rounding of the remainder.
__device__ __forceinline__ void split3(float u, uint32_t& h, uint32_t& m, uint32_t& l) {
  h = bf16_bits_rn(u);
  const float r1 = __fsub_rn(u, __uint_as_float(h << 16));
  m = bf16_bits_rn(r1);
  const float r2 = __fsub_rn(r1, __uint_as_float(m << 16));
  l = bf16_bits_rn(r2);
}

// Write 8 consecutive values (k0 % 8 == 0) of one row into an image as three
// 16-byte stores.
__device__ __forceinline__ void img_store8(uint8_t* img, int64_t row, int k0, int K, const float (&v)[8]) {
  uint32_t h[4], m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h0, m0, l0, h1, m1, l1;
    split3(v[2 * i], h0, m0, l0);
    split3(v[2 * i + 1], h1, m1, l1);
    h[i] = h0 | (h1 << 16);
    m[i] = m0 | (m1 << 16);
    l[i] = l0 | (l1 << 16);
  }
  const int64_t off = img_offset(row, 0, k0, K);
  const int64_t ps = (int64_t)K * 256;
  *reinterpret_cast<uint4*>(img + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(img + off + ps) = make_uint4(m[0], m[1], m[2], m[3]);
  *reinterpret_cast<uint4*>(img + off + 2 * ps) = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---- PTX wrappers (mbarrier and bulk-copy helpers are in async.cuh) ------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B
// apart (stride byte offset), tile bases 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: A and B bf16, D f32, both K-major, M=128.
__host__ __device__ constexpr uint32_t idesc_bf16(int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// A from tensor memory (rows on lanes, two bf16 K elements per column), B from
// shared memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive FP32 columns of this thread's TMEM lane.
// Split cluster barrier: arrive (release) now, wait (acquire) later.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 16-column TMEM loads in flight together, one wait (the wait names the
// destination registers, so no use of them is scheduled before it).
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, float (&va)[16], uint32_t tb, float (&vb)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(ta));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(r[16 + i]);
  }
}

// Two 32-column TMEM loads in flight together, one wait (as tmem_ld16x2).
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, float (&va)[32], uint32_t tb, float (&vb)[32]) {
  uint32_t r[64];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(ta));
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
               : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(r[32 + i]);
  }
}

// Two 8-column TMEM loads in flight together, one wait (as tmem_ld16x2).
__device__ __forceinline__ void tmem_ld8x2(uint32_t ta, float (&va)[8], uint32_t tb, float (&vb)[8]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(ta));
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                 "=r"(r[15])
               : "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(r[8 + i]);
  }
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- GEMM --------------------------------------------------------------------

enum { TEPI_QKV = 0, TEPI_RESNORM = 1, TEPI_GLU = 2, TEPI_VOCAB = 3, TEPI_STORE = 4 };

// Threads per CTA.  The weight expansion and the SwiGLU / argmax / residual
// + RMSNorm epilogues are latency-bound at one CTA per SM, so those kernels
// run 16 warps (each TMEM lane quadrant read by four warps, a quarter of the
// columns each; a warp takes 8 rows of the residual pass instead of 16); the
// QKV epilogue keeps 8 warps.
__host__ __device__ constexpr int threads_for(int epi) {
  return (epi == TEPI_GLU || epi == TEPI_VOCAB || epi == TEPI_RESNORM) ? 512 : kThreads;
}

// Bytes of the staging area that receives an item's packed weight rows (all
// of K) and their scales: 128 rows of K = 384.
constexpr int kStageBytes = 128 * (288 + 4);

// Whether N packed rows of K plus their scales fit the staging area.
__host__ __device__ constexpr bool stage_fits(int64_t N, int64_t K) { return N * (K * 3 / 4 + 4) <= kStageBytes; }

// Rows per N tile of the plain linear (TEPI_STORE) on this kernel, or 0 when
// the shape does not fit it: K a multiple of 128, N in {256, 128, 64}
// dividing rows, and the tile's packed rows within the staging area.
__host__ __device__ inline int store_tile_rows(int64_t rows, int64_t K) {
  if (K <= 0 || K % kKC) return 0;
  for (int N = 256; N >= 64; N >>= 1)
    if (rows % N == 0 && stage_fits(N, K)) return N;
  return 0;
}

struct TcArgs {
  const uint8_t* a_img;  // activation image [ceil(n/128) tiles][3][K]
  int32_t n, K;
  // weights: B tile rows come from up to three matrices (see row_src)
  const uint8_t* q0;
  const uint8_t* q1;
  const uint8_t* q2;
  const float* s0;
  const float* s1;
  const float* s2;
  int32_t end0, end1;  // QKV: virtual-row ends of wq and wk
  int32_t N;           // rows per N tile (64, 128 or 256)
  int32_t n_tiles;     // N tiles per M tile
  int32_t pair;        // RESNORM: 0, or the cluster size (2 or 4) whose CTAs take the N-column blocks of an M tile
  // epilogue
  float* x;            // RESNORM: residual stream [n, 128] (read + written)
  const float* gnorm;  // RESNORM: norm weight applied to the new x for the next image
  float eps;
  uint8_t* out_img;    // RESNORM / GLU: next GEMM's activation image
  int32_t out_K;       // its K
  EpiArgs ep;          // QKV / VOCAB fields (pos, flags, caches, rope, keys, stop set, logits)
  int32_t* err;
};

// The B tile of N tile `nt` as up to three contiguous row segments of the
// weight matrices (rows of one segment are consecutive in the file image):
// QKV: wq | wk | wv; GLU: W1 rows 128nt.. | W3 rows 128nt..; otherwise one.
struct Seg {
  const uint8_t* q;
  const float* s;
  int r0, rows;
};

__device__ __forceinline__ int b_segments(const TcArgs& a, int epi, int nt, Seg (&sg)[3]) {
  if (epi == TEPI_GLU) {  // N / 2 rows of W1, then the same rows of W3
    sg[0] = {a.q0, a.s0, nt * (a.N >> 1), a.N >> 1};
    sg[1] = {a.q1, a.s1, nt * (a.N >> 1), a.N >> 1};
    return 2;
  }
  if (epi == TEPI_QKV) {
    // rows [nt N, nt N + N) of the concatenation wq | wk | wv (end0, end1: its
    // matrix boundaries; the last matrix ends at n_tiles N)
    const int v0 = nt * a.N, v1 = v0 + a.N;
    const int lo[3] = {0, a.end0, a.end1}, hi[3] = {a.end0, a.end1, a.n_tiles * a.N};
    const uint8_t* qs[3] = {a.q0, a.q1, a.q2};
    const float* ss[3] = {a.s0, a.s1, a.s2};
    int k = 0;
    for (int i = 0; i < 3; ++i) {
      const int b0 = v0 > lo[i] ? v0 : lo[i], b1 = v1 < hi[i] ? v1 : hi[i];
      if (b1 > b0) sg[k++] = {qs[i], ss[i], b0 - lo[i], b1 - b0};
    }
    return k;
  }
  sg[0] = {a.q0, a.s0, nt * a.N, a.N};
  return 1;
}

// Thread 0: start the bulk copies of stage `ks` of item (mt, nt): the A
// stage when `want_a`, the packed B rows (all K) and their scales when
// `want_b`; all complete on `bar`.  With `arrive` false the copies only add
// their bytes to the barrier's count (a later call arrives).
__device__ __forceinline__ void issue_loads(const TcArgs& a, int epi, int mt, int nt, int ks, bool want_a,
                                            bool want_b, uint8_t* sA, uint8_t* stage, uint64_t* bar,
                                            bool arrive = true) {
  const uint32_t rb = (uint32_t)a.K * 3 / 4;
  Seg sg[3];
  const int nseg = b_segments(a, epi, nt, sg);
  uint32_t bytes = want_a ? 3 * 32768 : 0;
  if (want_b) bytes += (uint32_t)a.N * (rb + 4);
  if (arrive)
    mbar_expect_tx(bar, bytes);
  else
    mbar_expect_tx_only(bar, bytes);
  if (want_a) {
    const uint8_t* src = a.a_img + (int64_t)mt * 3 * a.K * 256 + (int64_t)ks * 32768;
#pragma unroll
    for (int p = 0; p < 3; ++p) bulk_g2s(sA + p * 32768, src + (int64_t)p * a.K * 256, 32768, bar);
  }
  if (want_b) {
    uint8_t* dst = stage;
    float* sdst = reinterpret_cast<float*>(stage + (size_t)a.N * rb);
    for (int i = 0; i < nseg; ++i) {
      bulk_g2s(dst, sg[i].q + (int64_t)sg[i].r0 * rb, (uint32_t)sg[i].rows * rb, bar);
      bulk_g2s(sdst, sg[i].s + sg[i].r0, (uint32_t)sg[i].rows * 4, bar);
      dst += (size_t)sg[i].rows * rb;
      sdst += sg[i].rows;
    }
  }
}

// Shared memory: [A stage 96 KB][B tile N x 128 bf16, 64 KB][packed B rows + scales, <= 37 KB]

template <int EPI>
__global__ void __launch_bounds__(threads_for(EPI), 1) tc_gemm_kernel(TcArgs a) {
  constexpr int NT = threads_for(EPI);
  constexpr int kParts = NT / 128;  // warps reading each TMEM lane quadrant (column parts)
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t mma_bar, ld_bar, ld_bar1;
  __shared__ uint32_t tmem_base;
  __shared__ __align__(16) float sscale[256];
  __shared__ int timed_out;
  __shared__ int s_ok[kM], s_pos[kM];  // QKV epilogue: per row
  __shared__ int64_t s_crow[kM];
  __shared__ float s_ssp[kM];          // RESNORM pair: this CTA's half of each row's sum of squares
  namespace cg = cooperative_groups;
  int pair_synced = 0;                 // RESNORM pair: cluster barriers taken (two per item)
  const int tid = threadIdx.x, warp = tid >> 5;
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;                       // [3][2][128][128 B] = 96 KB (one K stage)
  uint8_t* sB = smem + 3 * kM * kKC * 2;    // [2][N][128 B]
  // RESNORM in 32-column tiles (4-CTA clusters, one item a CTA) with more
  // than one K stage: the A stages alternate between sA and a second buffer
  // sA1 placed after the 32-row B tile, so the next stage's copy runs under
  // this stage's expansion and MMAs; the staging area then follows sA1
  // (smem_bytes_for).
  const bool dbl = EPI == TEPI_RESNORM && a.pair == 4 && a.K > kKC;
  uint8_t* sA1 = sB + 32 * kKC * 2;
  uint8_t* stage = dbl ? sA1 + 3 * kM * kKC * 2 : sB + 256 * kKC * 2;  // packed rows [N][K*3/4] + scales [N]

  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&mma_bar, 1);
    mbar_init(&ld_bar, 1);
    mbar_init(&ld_bar1, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    timed_out = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = tmem_base;
  const uint32_t idesc = idesc_bf16(a.N);
  const int m_tiles = (a.n + kM - 1) / kM;
  const int items = m_tiles * a.n_tiles;
  const int per = (items + gridDim.x - 1) / gridDim.x;
  const int it0 = blockIdx.x * per, it1 = min(items, it0 + per);
  const int kstages = a.K / kKC;
  const uint32_t rb = (uint32_t)a.K * 3 / 4;
  uint32_t ph_mma = 0, ph_ld = 0, ph_ld1 = 0;
  int pend0 = 0, pend1 = 0;  // dbl: copies in flight on ld_bar / ld_bar1 (the same in every thread)
  // The weights do not depend on the preceding grid: their copies start
  // before the programmatic-dependency wait, the activation tile after it.
  grid_dep_launch();
  if (tid == 0 && it0 < it1)
    issue_loads(a, EPI, it0 / a.n_tiles, it0 % a.n_tiles, 0, false, true, sA, stage, &ld_bar, false);
  grid_dep_wait();
  if (tid == 0 && it0 < it1) issue_loads(a, EPI, it0 / a.n_tiles, it0 % a.n_tiles, 0, true, false, sA, stage, &ld_bar);
  if (dbl && it0 < it1) {
    if (tid == 0) issue_loads(a, EPI, it0 / a.n_tiles, it0 % a.n_tiles, 1, true, false, sA1, stage, &ld_bar1);
    pend0 = pend1 = 1;
  }

  for (int it = it0; it < it1 && !timed_out; ++it) {
    const int mt = it / a.n_tiles, nt = it % a.n_tiles;
    // Epilogue inputs that do not depend on the MMA are loaded first, so they
    // are in flight during the tile loads, the expansion and the MMAs.
    // QKV: this thread's row state and the RoPE rotation of the 16 pairs of a
    // 32-column chunk (chunks start on a head boundary: columns are multiples
    // of 32 and head_dim is 16 or 32, so pair p turns by frequency p mod hd/2).
    bool q_ok = false;
    int q_pos = 0;
    int64_t q_crow = 0;
    float cp[16], sp[16];
    if (EPI == TEPI_QKV) {
      const EpiArgs& ep = a.ep;
      const int64_t me = (int64_t)mt * kM + (((warp & 3) << 5) | (tid & 31));
      q_ok = me < a.n && !(ep.flags[me] & SEQ_INVALID);
      q_pos = q_ok ? ep.pos[me] : 0;
      q_crow = q_ok && ep.seq ? ep.seq[me] : me;
      const int hh = ep.hd >> 1;  // 8 or 16 rotation frequencies
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        cp[p] = q_ok ? __ldg(ep.rope_cos + (int64_t)q_pos * hh + (p & (hh - 1))) : 0.0f;
        sp[p] = q_ok ? __ldg(ep.rope_sin + (int64_t)q_pos * hh + (p & (hh - 1))) : 0.0f;
      }
    }
    // RESNORM: the residual rows of this thread's passes and its norm weights.
    constexpr int kRPW = kM / (NT / 32);  // rows of the residual pass per warp: 16 (8 warps) or 8 (16)
    constexpr int kPass = kRPW / 2;       // at most this many passes of 2 rows (4 in pair mode)
    float4 ox[kPass][2];
    float gw[8];
    if (EPI == TEPI_RESNORM) {
      const int lane = tid & 31;
      const int lpr = a.N >> 3, rpi = 32 / lpr;
      const int sub = lane / lpr, cb = 8 * (lane % lpr);
      const int col = nt * a.N + cb;
      const int npass = kRPW / rpi;
#pragma unroll
      for (int i = 0; i < 8; ++i) gw[i] = __ldg(a.gnorm + col + i);
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        const int64_t mr = (int64_t)mt * kM + kRPW * warp + rpi * i + sub;
        const float4* xr = reinterpret_cast<const float4*>(a.x + mr * 128 + col);
        const bool in = i < npass && mr < a.n;
        ox[i][0] = in ? xr[0] : make_float4(0.f, 0.f, 0.f, 0.f);
        ox[i][1] = in ? xr[1] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    for (int ks = 0; ks < kstages; ++ks) {
      const bool odd = dbl && (ks & 1);  // this stage is in sA1
      if (!mbar_wait(odd ? &ld_bar1 : &ld_bar, odd ? ph_ld1 : ph_ld)) {
        if (tid == 0) atomicOr(a.err, kErrTimeout);
        timed_out = 1;
      }
      if (odd) {
        ph_ld1 ^= 1;
        --pend1;
      } else {
        ph_ld ^= 1;
        if (dbl) --pend0;
      }
      __syncthreads();
      if (timed_out) break;
      // expand N rows x 128 codes (columns 128ks..) from the staged bytes to bf16
      if (ks == 0)
        for (int j = tid; j < a.N; j += NT)
          sscale[j] = reinterpret_cast<const float*>(stage + (size_t)a.N * rb)[j];
      for (int i = tid; i < a.N * 8; i += NT) {
        const int j = i >> 3, u = i & 7;
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(stage + j * rb + (ks * 8 + u) * 12);
        const uint32_t w0 = pw[0], w1 = pw[1], w2 = pw[2];
        const uint32_t f[16] = {w0, w0 >> 6, w0 >> 12, w0 >> 18, w0 >> 24, __funnelshift_r(w0, w1, 30),
                                w1 >> 4, w1 >> 10, w1 >> 16, w1 >> 22, __funnelshift_r(w1, w2, 28),
                                w2 >> 2, w2 >> 8, w2 >> 14, w2 >> 20, w2 >> 26};
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          pk[e] = (__float_as_uint(code_to_float(f[2 * e])) >> 16) |
                  (__float_as_uint(code_to_float(f[2 * e + 1])) & 0xFFFF0000u);
        const int c64 = u >> 2, lu = (u & 3) * 2;
        uint8_t* line = sB + c64 * (a.N * 128) + j * 128;
        reinterpret_cast<uint4*>(line)[lu ^ (j & 7)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        reinterpret_cast<uint4*>(line)[(lu + 1) ^ (j & 7)] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(odd ? sA1 : sA), b0 = smem_u32(sB);
#pragma unroll 1
        for (int p = 0; p < 3; ++p)
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sdesc(a0 + p * 32768 + c * 16384 + kk * 32);
              const uint64_t bd = sdesc(b0 + c * (a.N * 128) + kk * 32);
              umma(taddr, ad, bd, idesc, (ks | p | c | kk) != 0);
            }
        umma_commit(&mma_bar);
      }
      if (!mbar_wait(&mma_bar, ph_mma)) {
        if (tid == 0) atomicOr(a.err, kErrTimeout);
        timed_out = 1;
      }
      ph_mma ^= 1;
      tc_fence_after();
      // prefetch the next stage / item while this one's epilogue runs
      if (dbl) {
        // the buffer just read takes the stage two ahead
        if (!timed_out && ks + 2 < kstages) {
          if (tid == 0) issue_loads(a, EPI, mt, nt, ks + 2, true, false, odd ? sA1 : sA, stage, odd ? &ld_bar1 : &ld_bar);
          if (odd)
            ++pend1;
          else
            ++pend0;
        }
      } else if (tid == 0 && !timed_out) {
        if (ks + 1 < kstages) {
          issue_loads(a, EPI, mt, nt, ks + 1, true, false, sA, stage, &ld_bar);
        } else if (it + 1 < it1) {
          const int mt2 = (it + 1) / a.n_tiles;
          issue_loads(a, EPI, mt2, (it + 1) % a.n_tiles, 0, mt2 != mt || kstages > 1, true, sA, stage, &ld_bar);
        }
      }
      __syncthreads();
      if (timed_out) break;
    }
    if (timed_out) break;

    // ---- epilogue: lane quadrant q = warp & 3 holds sequence rows 32q..32q+31
    // (TMEM lanes); warps q and q + 4 take the two halves of the columns.
    const int row = ((warp & 3) << 5) | (tid & 31);
    const int half = warp >> 2;  // the column part (halves at 8 warps, quarters at 16)
    const int64_t m = (int64_t)mt * kM + row;
    const bool live = m < a.n;
    const uint32_t lane_addr = taddr + ((uint32_t)((warp & 3) * 32) << 16);
    if (EPI == TEPI_VOCAB) {
      const EpiArgs& ep = a.ep;
      const bool mask = live && ep.n_stop && ep.gen[m] < ep.min_new;
      const bool dump = live && ep.step_logits && !(ep.flags[m] & (SEQ_DONE | SEQ_INVALID)) &&
                        ep.pos[m] >= ep.plen[m] - 1;
      float bv = -INFINITY;
      int bi = -1;
      const int cb = half * (a.N / kParts), ce = cb + a.N / kParts;
      for (int c2 = cb; c2 < ce; c2 += 64) {
        // two 32-column chunks loaded together (one when 32 columns remain)
        float vv[2][32];
        const int nh = c2 + 32 < ce ? 2 : 1;
        if (nh == 2)
          tmem_ld32x2(lane_addr + c2, vv[0], lane_addr + c2 + 32, vv[1]);
        else
          tmem_ld32(lane_addr + c2, vv[0]);
        if (!live) continue;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (hh >= nh) break;
          float (&v)[32] = vv[hh];
          const int c0 = c2 + 32 * hh;
          const int r0 = nt * a.N + c0;
          const float4* s4 = reinterpret_cast<const float4*>(sscale + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 sc = s4[i];
            v[4 * i] = __fmul_rn(v[4 * i], sc.x);
            v[4 * i + 1] = __fmul_rn(v[4 * i + 1], sc.y);
            v[4 * i + 2] = __fmul_rn(v[4 * i + 2], sc.z);
            v[4 * i + 3] = __fmul_rn(v[4 * i + 3], sc.w);
          }
          if (ep.y) {
            float4* y = reinterpret_cast<float4*>(ep.y + m * ep.ldy + r0);
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
          if (dump) {
            float4* y = reinterpret_cast<float4*>(ep.step_logits + (m * ep.new_tokens + ep.gen[m]) * ep.vocab + r0);
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
          if (mask) {
            for (int s = 0; s < ep.n_stop; ++s) {
              const int k = ep.stop_ids[s] - r0;
              if (k >= 0 && k < 32) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i == k) v[i] = -INFINITY;
              }
            }
          }
          // first maximum in increasing column order (torch.argmax's tie rule)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (v[i] > bv || bi < 0) {
              bv = v[i];
              bi = r0 + i;
            }
        }
      }
      if (live && bi >= 0) atomicMax(ep.keys + m, argmax_key(bv, bi));
    } else if (EPI == TEPI_STORE) {
      // the plain linear: y[m, nt N + c] = scale * D, 32 consecutive floats per load
      const EpiArgs& ep = a.ep;
      const int cb = half * (a.N >> 1), ce = cb + (a.N >> 1);
      for (int c0 = cb; c0 < ce; c0 += 32) {
        float v[32];
        tmem_ld32(lane_addr + c0, v);
        if (!live) continue;
        const int r0 = nt * a.N + c0;
        const float4* s4 = reinterpret_cast<const float4*>(sscale + c0);
        float4* y = reinterpret_cast<float4*>(ep.y + m * ep.ldy + r0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 sc = s4[i];
          y[i] = make_float4(__fmul_rn(v[4 * i], sc.x), __fmul_rn(v[4 * i + 1], sc.y),
                             __fmul_rn(v[4 * i + 2], sc.z), __fmul_rn(v[4 * i + 3], sc.w));
        }
      }
    } else if (EPI == TEPI_QKV) {
      // Columns in two blocks through shared memory (sB): block 0 the q rows
      // [0, 128), block 1 the k and v rows [128, N).  E1 (this thread's row):
      // scale and RoPE, into sB unit c4 of row r at r*32 + (c4 ^ (r & 7));
      // E2: lanes of a row store contiguous runs of q, k and v.
      const EpiArgs& ep = a.ep;
      const bool ok = q_ok;
      s_ok[row] = ok;
      s_pos[row] = q_pos;
      s_crow[row] = q_crow;
      float4* st4 = reinterpret_cast<float4*>(sB);
      const int lane = tid & 31;
#pragma unroll 1
      for (int b = 0; b < 2; ++b) {
        const int bw = b == 0 ? (a.N < 128 ? a.N : 128) : a.N - 128;  // block width (a multiple of 64)
        if (bw <= 0) break;  // a tile of 128 rows has one block
        const int hw = bw >> 1;
        for (int cc = 0; cc < hw; cc += 32) {
          const int lc = half * hw + cc;  // column in the block
          const int c0 = 128 * b + lc;    // column of the tile
          float v[32];
          tmem_ld32(lane_addr + c0, v);
          const float4* s4 = reinterpret_cast<const float4*>(sscale + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 sc = s4[i];
            v[4 * i] = __fmul_rn(v[4 * i], sc.x);
            v[4 * i + 1] = __fmul_rn(v[4 * i + 1], sc.y);
            v[4 * i + 2] = __fmul_rn(v[4 * i + 2], sc.z);
            v[4 * i + 3] = __fmul_rn(v[4 * i + 3], sc.w);
          }
          const int v0 = nt * a.N + c0;  // first virtual row of this chunk
          if (ok && v0 < ep.q_rows + ep.kv_rows) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float c = cp[i >> 1], sv = sp[i >> 1];
              const float ra = __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(v[i + 1], sv));
              const float rb = __fadd_rn(__fmul_rn(v[i], sv), __fmul_rn(v[i + 1], c));
              v[i] = ra;
              v[i + 1] = rb;
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
            st4[row * 32 + (((lc >> 2) + i) ^ (row & 7))] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
        __syncthreads();
        const int lpr = bw >> 3;  // lanes per row, 8 columns each
        const int rpi = 32 / lpr, sub = lane / lpr, cb = 8 * (lane % lpr);
        for (int r0 = 16 * warp; r0 < 16 * warp + 16; r0 += rpi) {
          const int r = r0 + sub;
          if (!s_ok[r]) continue;
          const int64_t mr = (int64_t)mt * kM + r;
          const float4 p0 = st4[r * 32 + ((cb >> 2) ^ (r & 7))], p1 = st4[r * 32 + (((cb >> 2) + 1) ^ (r & 7))];
          const int v0 = nt * a.N + 128 * b + cb;
          if (v0 < ep.q_rows) {
            float* dst = ep.qbuf + mr * ep.ldq + v0;
            reinterpret_cast<float4*>(dst)[0] = p0;
            reinterpret_cast<float4*>(dst)[1] = p1;
          } else {
            const bool kr = v0 < ep.q_rows + ep.kv_rows;
            const int64_t off = s_crow[r] * ep.cache_stride + ep.layer_off + (int64_t)s_pos[r] * ep.kv_rows +
                                (kr ? v0 - ep.q_rows : v0 - ep.q_rows - ep.kv_rows);
            store_kv8(kr ? ep.kc : ep.vc, off, ep.kv_half, p0, p1);
          }
        }
        __syncthreads();  // the next block reuses sB
      }
    } else if (EPI == TEPI_RESNORM) {  // N == 128 == dim, or N == 128 / a.pair per CTA of a cluster
      // Two passes through shared memory (sB: the weights are consumed once the
      // MMAs are done), so every global access is row-contiguous.
      // E1: this thread's row (TMEM lane) and columns (N/kParts)*part.., scaled,
      // into sB as float4 unit c4 of row r at r*32 + (c4 ^ (r & 7)).
      float4* st4 = reinterpret_cast<float4*>(sB);
      const int hn = a.N / kParts;
      if (hn == 8) {  // N == 32 (a CTA of a 4-CTA cluster) at 16 warps: 8 columns a thread
        const int c0 = half * 8;
        float v[8];
        tmem_ld8(lane_addr + c0, v);
        const float4* s4 = reinterpret_cast<const float4*>(sscale + c0);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float4 sc = s4[i];
          st4[row * 32 + (((c0 >> 2) + i) ^ (row & 7))] =
              make_float4(__fmul_rn(v[4 * i], sc.x), __fmul_rn(v[4 * i + 1], sc.y), __fmul_rn(v[4 * i + 2], sc.z),
                          __fmul_rn(v[4 * i + 3], sc.w));
        }
      }
      for (int cc = 0; hn >= 16 && cc < hn; cc += 16) {
        const int c0 = half * hn + cc;
        float v[16];
        tmem_ld16(lane_addr + c0, v);
        const float4* s4 = reinterpret_cast<const float4*>(sscale + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 sc = s4[i];
          st4[row * 32 + (((c0 >> 2) + i) ^ (row & 7))] =
              make_float4(__fmul_rn(v[4 * i], sc.x), __fmul_rn(v[4 * i + 1], sc.y), __fmul_rn(v[4 * i + 2], sc.z),
                          __fmul_rn(v[4 * i + 3], sc.w));
        }
      }
      __syncthreads();
      // E2: lane groups of N/8 lanes take rows (8 columns a lane): residual add,
      // x written back, the row's sum of squares over the group (plus the
      // peer's half of the row in pair mode, added in rank order), RMSNorm
      // with the next norm weight, and the row's image units.
      const int lane = tid & 31;
      const int lpr = a.N >> 3, rpi = 32 / lpr;  // lanes per row, rows per warp pass
      const int sub = lane / lpr, cl8 = lane % lpr, cb = 8 * cl8;
      const int col = nt * a.N + cb;  // column of x and of the image
      const int npass = kRPW / rpi;
      // ox (the residual rows of all passes) and gw were loaded at the item's start
      float xk[kPass][8];
      float ssk[kPass];
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        ssk[i] = 0.0f;
        const int r = kRPW * warp + rpi * i + sub;
        const int64_t mr = (int64_t)mt * kM + r;
        const bool lv = i < npass && mr < a.n;  // uniform over the lanes of the row
#pragma unroll
        for (int e = 0; e < 8; ++e) xk[i][e] = 0.0f;
        if (i < npass) {
          const float4 p0 = st4[r * 32 + ((cb >> 2) ^ (r & 7))], p1 = st4[r * 32 + (((cb >> 2) + 1) ^ (r & 7))];
          if (lv) {
            float4* xr = reinterpret_cast<float4*>(a.x + mr * 128 + col);
            const float4 o0 = ox[i][0], o1 = ox[i][1];
            xk[i][0] = __fadd_rn(o0.x, p0.x); xk[i][1] = __fadd_rn(o0.y, p0.y);
            xk[i][2] = __fadd_rn(o0.z, p0.z); xk[i][3] = __fadd_rn(o0.w, p0.w);
            xk[i][4] = __fadd_rn(o1.x, p1.x); xk[i][5] = __fadd_rn(o1.y, p1.y);
            xk[i][6] = __fadd_rn(o1.z, p1.z); xk[i][7] = __fadd_rn(o1.w, p1.w);
            xr[0] = make_float4(xk[i][0], xk[i][1], xk[i][2], xk[i][3]);
            xr[1] = make_float4(xk[i][4], xk[i][5], xk[i][6], xk[i][7]);
          }
        }
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(xk[i][e], xk[i][e]));
        for (int o = lpr >> 1; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        ssk[i] = ss;
        if (a.pair && i < npass && cl8 == 0) s_ssp[r] = ss;
      }
      if (a.pair) {
        // every column block of every row: the a.pair partial sums meet
        // through distributed shared memory and are added in rank order (the
        // cluster rank is nt); the second barrier (arrive here, wait before
        // the CTA exits) keeps this CTA's array alive until the peers have
        // read it
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        if (a.pair == 2) {
          const float* peer = cl.map_shared_rank(s_ssp, nt ^ 1);
#pragma unroll
          for (int i = 0; i < kPass; ++i) {
            if (i < npass) {
              const int r = kRPW * warp + rpi * i + sub;
              ssk[i] = nt == 0 ? __fadd_rn(ssk[i], peer[r]) : __fadd_rn(peer[r], ssk[i]);
            }
          }
        } else {  // four blocks (every lane of a row holds the same partial sum as s_ssp)
          const float* p0 = cl.map_shared_rank(s_ssp, 0);
          const float* p1 = cl.map_shared_rank(s_ssp, 1);
          const float* p2 = cl.map_shared_rank(s_ssp, 2);
          const float* p3 = cl.map_shared_rank(s_ssp, 3);
#pragma unroll
          for (int i = 0; i < kPass; ++i) {
            if (i < npass) {
              const int r = kRPW * warp + rpi * i + sub;
              ssk[i] = __fadd_rn(__fadd_rn(__fadd_rn(p0[r], p1[r]), p2[r]), p3[r]);
            }
          }
        }
        cluster_arrive();
        pair_synced = 2;
      }
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        const int64_t mr = (int64_t)mt * kM + kRPW * warp + rpi * i + sub;
        if (i < npass && mr < a.n) {
          const float rstd = rms_scale(ssk[i], 128, a.eps);
          float u8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) u8[e] = __fmul_rn(__fmul_rn(xk[i][e], rstd), gw[e]);
          img_store8(a.out_img, mr, col, 128, u8);
        }
      }
    } else if (EPI == TEPI_GLU) {  // columns j (W1) and H + j (W3), H = N/2; this thread: j in (H/kParts)*part..
      const int H = a.N >> 1, hq = H / kParts;
      if (hq == 8) {  // N == 64 (32 W1 + 32 W3 rows) at 16 warps: 8 columns a thread
        const int c0 = half * 8;
        float va[8], vb[8];
        tmem_ld8x2(lane_addr + c0, va, lane_addr + H + c0, vb);
        if (live) {
          float h8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            h8[i] = swiglu(__fmul_rn(va[i], sscale[c0 + i]), __fmul_rn(vb[i], sscale[H + c0 + i]));
          img_store8(a.out_img, m, nt * H + c0, a.out_K, h8);
        }
      }
#pragma unroll 1
      for (int cc = 0; hq >= 16 && cc < hq; cc += 16) {
        const int c0 = half * hq + cc;
        float va[16], vb[16];
        tmem_ld16x2(lane_addr + c0, va, lane_addr + H + c0, vb);
        if (!live) continue;
#pragma unroll
        for (int k0 = 0; k0 < 16; k0 += 8) {
          float h8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            h8[i] = swiglu(__fmul_rn(va[k0 + i], sscale[c0 + k0 + i]), __fmul_rn(vb[k0 + i], sscale[H + c0 + k0 + i]));
          img_store8(a.out_img, m, nt * H + c0 + k0, a.out_K, h8);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  // a CTA that stopped on a timed-out wait first waits (bounded) for its A
  // copies still in flight, so none lands after it exits
  if (dbl && tid == 0) {
    if (pend0 > 0) (void)mbar_wait(&ld_bar, ph_ld);
    if (pend1 > 0) (void)mbar_wait(&ld_bar1, ph_ld1);
  }
  // a pair CTA that stopped early still takes its two cluster barriers, so
  // the peer's waits end; the second one's wait comes last
  if (EPI == TEPI_RESNORM && a.pair) {
    if (pair_synced < 2) {
      cg::this_cluster().sync();
      cluster_arrive();
    }
    cluster_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(taddr, 256);
  }
}

constexpr size_t smem_bytes() { return 1024 + 3 * kM * kKC * 2 + 256 * kKC * 2 + kStageBytes; }

// Dynamic shared memory of a kernel: RESNORM also fits the double-buffered
// layout of its 32-column tiles (two A stages, the 32-row B tile, and 32
// packed rows of K <= 384 in the staging area after them).
constexpr size_t smem_bytes_for(int epi) {
  return epi == TEPI_RESNORM ? 1024 + 2 * 3 * kM * kKC * 2 + 32 * kKC * 2 + 32 * (384 * 3 / 4 + 4) : smem_bytes();
}
static_assert(smem_bytes_for(TEPI_RESNORM) >= smem_bytes() && smem_bytes_for(TEPI_RESNORM) <= 232448,
              "RESNORM shared memory");

}  // namespace tc
}  // namespace q6w
