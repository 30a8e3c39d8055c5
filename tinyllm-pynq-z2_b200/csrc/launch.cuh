// Host launcher of the Q6W linear kernels: picks the streaming kernel (one
// activation row, large K), the GEMV (few rows) or the tiled GEMM by n.
#pragma once

#include <algorithm>

#include "linear.cuh"
#include "stream.cuh"

namespace q6w {

// Host launcher.  Chooses the kernel by n; returns a status.
int grid_for(int64_t work, int threads);

template <bool RMS, int EPI>
struct LinearLauncher {
  template <int NB, int G>
  static cudaError_t gemv(const float* x, int ldx, int n, const float* g, float eps,
                          const MatSet& ms, const EpiArgs& ep, cudaStream_t st) {
    const int U = ms.cols >> 4;
    const size_t smem = (size_t)NB * U * 64;
    auto kern = gemv_kernel<NB, G, RMS, EPI>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    const int groups_per_cta = 8 * (32 / G);
    int blocks = (ms.n_pairs + groups_per_cta - 1) / groups_per_cta;
    if (blocks < 1) blocks = 1;
    kern<<<blocks, 256, smem, st>>>(x, ldx, n, g, eps, ms, ep);
    return cudaGetLastError();
  }

  template <int NB>
  static cudaError_t gemv_g(const float* x, int ldx, int n, const float* g, float eps,
                            const MatSet& ms, const EpiArgs& ep, cudaStream_t st) {
    if ((ms.cols >> 4) >= 64) return gemv<NB, 32>(x, ldx, n, g, eps, ms, ep, st);
    return gemv<NB, 8>(x, ldx, n, g, eps, ms, ep, st);
  }

  // The streaming kernel needs 16-byte aligned inputs, weights and scales
  // (bulk copies, vector loads) and a row geometry it tiles exactly.
  static bool stream_ok(const float* x, const MatSet& ms, stream::Geometry& geo) {
    if ((ms.glu != 0) != (EPI == EPI_GLU)) return false;
    if (!stream::geometry(ms, geo) || !aligned(x, 16) || !aligned(ms.q0, 16) || !aligned(ms.s0, 16)) return false;
    if (ms.glu) return aligned(ms.q1, 16) && aligned(ms.s1, 16);
    if (ms.end0 < 2 * ms.n_pairs && (!aligned(ms.q1, 16) || !aligned(ms.s1, 16))) return false;
    if (ms.end1 < 2 * ms.n_pairs && (!aligned(ms.q2, 16) || !aligned(ms.s2, 16))) return false;
    return true;
  }

  template <int WC, int MINB>
  static cudaError_t stream_launch_wc(const float* x, const float* g, float eps, const MatSet& ms,
                                      const EpiArgs& ep, const stream::Geometry& geo, cudaStream_t st) {
    auto kern = stream::stream_gemv_kernel<RMS, EPI, WC, MINB>;
    static bool configured = false;  // per instantiation: the size is a compile-time constant
    if (!configured) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)geo.smem);
      if (e != cudaSuccess) return e;
      configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    // two CTAs per SM, three for large matrices (K <= 2048 there: the stages of three fit)
    cfg.gridDim = dim3((unsigned)std::min(geo.tiles, (MINB == 3 ? 3 : 2) * sm_count()));
    cfg.blockDim = dim3((unsigned)geo.threads);
    cfg.dynamicSmemBytes = geo.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int32_t* err = stream::error_word();
    if (!err) return cudaErrorInvalidSymbol;  // the kernel's timeout diagnostic needs its device address
    return cudaLaunchKernelEx(&cfg, kern, x, g, eps, ms, ep, geo, err);
  }

  static cudaError_t stream_launch(const float* x, const float* g, float eps, const MatSet& ms, const EpiArgs& ep,
                                   const stream::Geometry& geo, cudaStream_t st) {
    // with the RMSNorm prologue every CTA normalises the row again: more CTAs cost more than they hide
    const bool big = !RMS && geo.tiles >= 3 * sm_count();
    switch (geo.wc) {
      case 1: return stream_launch_wc<1, 1>(x, g, eps, ms, ep, geo, st);
      case 2: return big ? stream_launch_wc<2, 3>(x, g, eps, ms, ep, geo, st)
                         : stream_launch_wc<2, 1>(x, g, eps, ms, ep, geo, st);
      case 4: return big ? stream_launch_wc<4, 3>(x, g, eps, ms, ep, geo, st)
                         : stream_launch_wc<4, 1>(x, g, eps, ms, ep, geo, st);
      case 8: return stream_launch_wc<8, 1>(x, g, eps, ms, ep, geo, st);
      default: return stream_launch_wc<11, 1>(x, g, eps, ms, ep, geo, st);
    }
  }

  static cudaError_t run(const float* x, int ldx, int n, const float* g, float eps,
                         const MatSet& ms, const EpiArgs& ep, cudaStream_t st) {
    if (n <= 0 || ms.n_pairs <= 0) return cudaSuccess;
    const int nb = n <= 2 ? n : (n <= 4 ? 4 : 8);
    const bool small_ok = n <= 8 && (size_t)nb * ms.cols * sizeof(float) <= 200 * 1024;
    if (!small_ok) {
      dim3 grid((ms.n_pairs + 31) / 32, (n + 127) / 128);
      gemm_kernel<RMS, EPI><<<grid, 256, 0, st>>>(x, ldx, n, g, eps, ms, ep);
      return cudaGetLastError();
    }
    if (n == 1) {
      stream::Geometry geo;
      if (stream_ok(x, ms, geo)) return stream_launch(x, g, eps, ms, ep, geo, st);
      return gemv_g<1>(x, ldx, n, g, eps, ms, ep, st);
    }
    if (n == 2) return gemv_g<2>(x, ldx, n, g, eps, ms, ep, st);
    if (n <= 4) return gemv_g<4>(x, ldx, n, g, eps, ms, ep, st);
    return gemv_g<8>(x, ldx, n, g, eps, ms, ep, st);
  }
};

}  // namespace q6w
