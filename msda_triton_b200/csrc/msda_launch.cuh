// msda_launch.cuh -- map the runtime launch shape (ndim, chunk bytes VB,
// chunks per lane VPL) onto kernel instantiations.  Included once per
// (value dtype, sampling dtype) pair by the msda_inst_*.cu files so those
// compile in parallel.
#pragma once

#include "msda_kernels.cuh"

namespace msda {

struct LaunchShape {
  int ndim;
  int vb;
  int vpl;
  int64_t grid;  // number of CTAs
};

// (chunk bytes, chunks per lane) pairs that are instantiated.  VB = 8 is the
// backward's layout for 16-bit values (see msda_bwd_kernel).
template <int VB, int VPL>
constexpr bool kAllowed = (VB == 16 && (VPL == 1 || VPL == 2 || VPL == 4)) ||
                          (VB == 8 && (VPL == 1 || VPL == 2 || VPL == 4 || VPL == 8)) ||
                          ((VB == 4 || VB == 2) && (VPL == 1 || VPL == 8));

template <typename T, typename TS, int NDIM, int VB, int VPL, bool F>
static cudaError_t fwd_one(const LaunchShape& ls, const Problem& p, void* out, cudaStream_t st) {
  if constexpr (kAllowed<VB, VPL> && VB != 8) {
    if constexpr (F)
      msda_fwd_fused_kernel<T, TS, NDIM, VB, VPL>
          <<<dim3(static_cast<unsigned>(ls.grid)), kThreads, 0, st>>>(p, static_cast<T*>(out));
    else
      msda_fwd_kernel<T, TS, NDIM, VB, VPL>
          <<<dim3(static_cast<unsigned>(ls.grid)), kThreads, 0, st>>>(p, static_cast<T*>(out));
    return cudaGetLastError();
  }
  return cudaErrorInvalidValue;
}

template <typename T, typename TS, int NDIM, int VB, int VPL, bool F>
static cudaError_t bwd_one(const LaunchShape& ls, const Problem& p, const void* grad_out,
                           float* gacc, void* grad_loc, void* grad_attn, cudaStream_t st) {
  if constexpr (kAllowed<VB, VPL> && (VB != 8 || sizeof(T) == 2)) {
    if constexpr (F)
      msda_bwd_fused_kernel<T, TS, NDIM, VB, VPL>
          <<<dim3(static_cast<unsigned>(ls.grid)), kThreads, 0, st>>>(
              p, static_cast<const T*>(grad_out), gacc, static_cast<TS*>(grad_loc),
              static_cast<TS*>(grad_attn));
    else
      msda_bwd_kernel<T, TS, NDIM, VB, VPL>
          <<<dim3(static_cast<unsigned>(ls.grid)), kThreads, 0, st>>>(
              p, static_cast<const T*>(grad_out), gacc, static_cast<TS*>(grad_loc),
              static_cast<TS*>(grad_attn));
    return cudaGetLastError();
  }
  return cudaErrorInvalidValue;
}

template <typename T, typename TS, int NDIM, int VB, bool F>
static cudaError_t fwd_vpl(const LaunchShape& ls, const Problem& p, void* out, cudaStream_t st) {
  switch (ls.vpl) {
    case 1: return fwd_one<T, TS, NDIM, VB, 1, F>(ls, p, out, st);
    case 2: return fwd_one<T, TS, NDIM, VB, 2, F>(ls, p, out, st);
    case 4: return fwd_one<T, TS, NDIM, VB, 4, F>(ls, p, out, st);
    case 8: return fwd_one<T, TS, NDIM, VB, 8, F>(ls, p, out, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, typename TS, int NDIM, int VB, bool F>
static cudaError_t bwd_vpl(const LaunchShape& ls, const Problem& p, const void* grad_out,
                           float* gacc, void* grad_loc, void* grad_attn, cudaStream_t st) {
  switch (ls.vpl) {
    case 1: return bwd_one<T, TS, NDIM, VB, 1, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    case 2: return bwd_one<T, TS, NDIM, VB, 2, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    case 4: return bwd_one<T, TS, NDIM, VB, 4, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    case 8: return bwd_one<T, TS, NDIM, VB, 8, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, typename TS, int NDIM, bool F>
static cudaError_t fwd_vb(const LaunchShape& ls, const Problem& p, void* out, cudaStream_t st) {
  switch (ls.vb) {
    case 16: return fwd_vpl<T, TS, NDIM, 16, F>(ls, p, out, st);
    case 4: return fwd_vpl<T, TS, NDIM, 4, F>(ls, p, out, st);
    case 2:
      if constexpr (sizeof(T) == 2) return fwd_vpl<T, TS, NDIM, 2, F>(ls, p, out, st);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, typename TS, int NDIM, bool F>
static cudaError_t bwd_vb(const LaunchShape& ls, const Problem& p, const void* grad_out,
                          float* gacc, void* grad_loc, void* grad_attn, cudaStream_t st) {
  switch (ls.vb) {
    case 16: return bwd_vpl<T, TS, NDIM, 16, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    case 8:
      if constexpr (sizeof(T) == 2)
        return bwd_vpl<T, TS, NDIM, 8, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
      return cudaErrorInvalidValue;
    case 4: return bwd_vpl<T, TS, NDIM, 4, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
    case 2:
      if constexpr (sizeof(T) == 2)
        return bwd_vpl<T, TS, NDIM, 2, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

// F selects the fused-prologue kernels (see Problem::ref).
template <typename T, typename TS, bool F>
cudaError_t launch_fwd(const LaunchShape& ls, const Problem& p, void* out, cudaStream_t st) {
  return ls.ndim == 2 ? fwd_vb<T, TS, 2, F>(ls, p, out, st) : fwd_vb<T, TS, 3, F>(ls, p, out, st);
}

template <typename T, typename TS, bool F>
cudaError_t launch_bwd(const LaunchShape& ls, const Problem& p, const void* grad_out,
                       float* gacc, void* grad_loc, void* grad_attn, cudaStream_t st) {
  return ls.ndim == 2 ? bwd_vb<T, TS, 2, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st)
                      : bwd_vb<T, TS, 3, F>(ls, p, grad_out, gacc, grad_loc, grad_attn, st);
}

template <typename T>
cudaError_t launch_cast(const float* src, void* dst, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + kThreads * 4 - 1) / (kThreads * 4);
  if (blocks > 148 * 16) blocks = 148 * 16;
  msda_cast_kernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(src, static_cast<T*>(dst), n);
  return cudaGetLastError();
}

// Compacted accumulator -> grad_value rows of the non-direct levels (16-bit T).
template <typename T>
cudaError_t launch_compact_cast(const Problem& p, const float* acc, void* gv, cudaStream_t st) {
  const int64_t row = key_stride(p);
  const bool vec = row % 4 == 0 && reinterpret_cast<uintptr_t>(gv) % 8 == 0;
  const int64_t nrows = p.B * p.acc_keys * (p.head_major ? p.H : 1);
  if (nrows <= 0 || row <= 0) return cudaSuccess;
  // host-resolved levels: one streaming span per (batch entry[, head], level)
  const int64_t spans = p.B * (p.head_major ? p.H : 1) * p.L;
  if (vec && p.shapes_dev == nullptr && spans > 0 && spans <= 65535) {
    int64_t maxn4 = 0;
    for (int64_t l = 0; l < p.L; ++l)
      maxn4 = std::max<int64_t>(
          maxn4, int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2] * row / 4);
    // about 8 float4 per thread on the largest level, at most 16 waves
    int64_t bx = (maxn4 + kThreads * 8 - 1) / (kThreads * 8);
    bx = std::max<int64_t>(1, std::min<int64_t>(bx, (148 * 16 + spans - 1) / spans * 4));
    msda_span_cast_kernel<T><<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(spans)),
                               kThreads, 0, st>>>(p, acc, static_cast<T*>(gv));
    return cudaGetLastError();
  }
  int64_t blocks = (nrows + kThreads / 32 - 1) / (kThreads / 32);  // a grid-stride loop covers the rest
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (vec)
    msda_compact_cast_kernel<T, 4><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
        p, acc, static_cast<T*>(gv));
  else
    msda_compact_cast_kernel<T, 1><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
        p, acc, static_cast<T*>(gv));
  return cudaGetLastError();
}

// Explicit instantiations live in msda_inst_*.cu (plain) and
// msda_inst_fused_*.cu (fused prologue).
#define MSDA_DECLARE_MODE(T, TS, F)                                                           \
  extern template cudaError_t launch_fwd<T, TS, F>(const LaunchShape&, const Problem&, void*,  \
                                                   cudaStream_t);                              \
  extern template cudaError_t launch_bwd<T, TS, F>(const LaunchShape&, const Problem&,         \
                                                   const void*, float*, void*, void*,          \
                                                   cudaStream_t);
#define MSDA_DECLARE_PAIR(T, TS) MSDA_DECLARE_MODE(T, TS, false) MSDA_DECLARE_MODE(T, TS, true)
#define MSDA_INSTANTIATE_MODE(T, TS, F)                                                       \
  template cudaError_t launch_fwd<T, TS, F>(const LaunchShape&, const Problem&, void*,         \
                                            cudaStream_t);                                     \
  template cudaError_t launch_bwd<T, TS, F>(const LaunchShape&, const Problem&, const void*,   \
                                            float*, void*, void*, cudaStream_t);

}  // namespace msda
