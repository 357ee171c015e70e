// msda_sorted_launch.cuh -- launch sequence of the cell-sorted backward
// (msda_sorted.cuh) for one chunk of batch entries.  Included by the
// msda_inst_sorted_*.cu files, which instantiate it per (value dtype,
// sampling dtype) pair.
#pragma once

#include "msda_launch.cuh"
#include "msda_sorted.cuh"

namespace msda {

// Lane shapes: `ls` is the forward's (dots and voxel kernels), `lsd` the
// dense kernel's (8-byte chunks for 16-bit values: one fp32 vector reduction
// per chunk).
template <typename T, typename TS, int NDIM, int VB, int VPL>
static cudaError_t dots_one(const Problem& p, const SortPlan& sp, const void* go, void* gl,
                            void* ga, cudaStream_t st, int64_t grid) {
  if constexpr (kAllowed<VB, VPL> && VB != 8) {
    msda_dots_kernel<T, TS, NDIM, VB, VPL><<<dim3(static_cast<unsigned>(grid)), kThreads, 0, st>>>(
        p, sp, static_cast<const T*>(go), static_cast<TS*>(gl), static_cast<TS*>(ga));
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gl; (void)ga; (void)st; (void)grid;
  return cudaErrorInvalidValue;
}

template <typename T, typename TS, int NDIM, int VB, int VPL>
static cudaError_t sdots_one(const Problem& p, const SortPlan& sp, const void* go, void* gl,
                             void* ga, cudaStream_t st) {
  if constexpr (kAllowed<VB, VPL> && VB != 8) {
    const int64_t grid = p.B * p.H * int64_t{sp.nsl} * sp.sd_chunks;
    msda_sdots_kernel<T, TS, NDIM, VB, VPL><<<dim3(static_cast<unsigned>(grid)), kThreads, 0, st>>>(
        p, sp, static_cast<const T*>(go), static_cast<TS*>(gl), static_cast<TS*>(ga));
    const int64_t n = p.B * p.Q * p.H * int64_t{sp.nsl} * p.P;
    msda_sdots_finish_kernel<TS, NDIM>
        <<<dim3(static_cast<unsigned>((n + kThreads - 1) / kThreads)), kThreads, 0, st>>>(
            p, sp, static_cast<TS*>(gl), static_cast<TS*>(ga));
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gl; (void)ga; (void)st;
  return cudaErrorInvalidValue;
}

template <typename T, int NDIM, int VB, int VPL>
static cudaError_t dense_one(const Problem& p, const SortPlan& sp, const void* go, float* gacc,
                             cudaStream_t st) {
  if constexpr (kAllowed<VB, VPL> && (VB != 8 || sizeof(T) == 2)) {
    const int64_t grid = p.B * p.H * int64_t{sp.ndl} * sp.dchunks;
    cudaError_t err = cudaFuncSetAttribute(msda_dense_kernel<T, NDIM, VB, VPL>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, sp.dsmem);
    if (err != cudaSuccess) return err;
    msda_dense_kernel<T, NDIM, VB, VPL>
        <<<dim3(static_cast<unsigned>(grid)), kThreads, static_cast<size_t>(sp.dsmem), st>>>(
            p, sp, static_cast<const T*>(go), gacc);
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gacc; (void)st;
  return cudaErrorInvalidValue;
}

template <typename T, int NDIM, int NT>
static cudaError_t dense_mma_one(const Problem& p, const SortPlan& sp, const void* go,
                                 float* gacc, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    const int64_t grid = p.B * p.H * int64_t{sp.nml} * sp.dchunks;
    cudaError_t err = cudaFuncSetAttribute(msda_dense_mma_kernel<T, NDIM, NT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           sp.dsmem_mma);
    if (err != cudaSuccess) return err;
    msda_dense_mma_kernel<T, NDIM, NT>
        <<<dim3(static_cast<unsigned>(grid)), kThreads, static_cast<size_t>(sp.dsmem_mma), st>>>(
            p, sp, static_cast<const T*>(go), gacc);
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gacc; (void)st;
  return cudaErrorInvalidValue;
}

template <typename T, int NDIM, int VB, int VPL>
static cudaError_t voxel_one(const Problem& p, const SortPlan& sp, const void* go, void* gv,
                             cudaStream_t st) {
  if constexpr (kAllowed<VB, VPL> && VB != 8) {
    const int64_t units = p.B * p.H * int64_t{sp.units_per_bh};
    cudaError_t err = cudaFuncSetAttribute(msda_voxel_kernel<T, NDIM, VB, VPL>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, sp.vsmem);
    if (err != cudaSuccess) return err;
    msda_voxel_kernel<T, NDIM, VB, VPL>
        <<<dim3(static_cast<unsigned>(units)), kThreads, static_cast<size_t>(sp.vsmem), st>>>(
            p, sp, static_cast<const T*>(go), static_cast<T*>(gv));
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gv; (void)st;
  return cudaErrorInvalidValue;
}

template <typename T, int NDIM, int NT>
static cudaError_t voxel_mma_one(const Problem& p, const SortPlan& sp, const void* go, void* gv,
                                 cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    const int64_t units = p.B * p.H * int64_t{sp.units_per_bh};
    cudaError_t err = cudaFuncSetAttribute(msda_voxel_mma_kernel<T, NDIM, NT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, sp.vsmem);
    if (err != cudaSuccess) return err;
    msda_voxel_mma_kernel<T, NDIM, NT>
        <<<dim3(static_cast<unsigned>(units)), kThreads, static_cast<size_t>(sp.vsmem), st>>>(
            p, sp, static_cast<const T*>(go), static_cast<T*>(gv));
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gv; (void)st;
  return cudaErrorInvalidValue;
}

template <typename T, int NDIM, int NT>
static cudaError_t voxel_tc_one(const Problem& p, const SortPlan& sp, const void* go, void* gv,
                                cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    const int64_t units = p.B * p.H * int64_t{sp.units_per_bh};
    cudaError_t err = cudaFuncSetAttribute(msda_voxel_tc_kernel<T, NDIM, NT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, sp.vsmem);
    if (err != cudaSuccess) return err;
    msda_voxel_tc_kernel<T, NDIM, NT>
        <<<dim3(static_cast<unsigned>(units)), kThreads, static_cast<size_t>(sp.vsmem), st>>>(
            p, sp, static_cast<const T*>(go), static_cast<T*>(gv));
    return cudaGetLastError();
  }
  (void)p; (void)sp; (void)go; (void)gv; (void)st;
  return cudaErrorInvalidValue;
}

// The forward shape: chunk bytes 16 (VPL 1, 2, 4) or 4 / 2 (VPL 1 or 8).
#define MSDA_FWD_SHAPE_SWITCH(vb, vpl, CALL)                                        \
  switch (vb * 16 + vpl) {                                                          \
    case 16 * 16 + 1: CALL(16, 1);                                                  \
    case 16 * 16 + 2: CALL(16, 2);                                                  \
    case 16 * 16 + 4: CALL(16, 4);                                                  \
    case 4 * 16 + 1: CALL(4, 1);                                                    \
    case 4 * 16 + 8: CALL(4, 8);                                                    \
    case 2 * 16 + 1: if constexpr (sizeof(T) == 2) { CALL(2, 1); } return cudaErrorInvalidValue; \
    case 2 * 16 + 8: if constexpr (sizeof(T) == 2) { CALL(2, 8); } return cudaErrorInvalidValue; \
    default: return cudaErrorInvalidValue;                                          \
  }

template <typename T, typename TS, int NDIM>
static cudaError_t sorted_chunk(const LaunchShape& ls, const LaunchShape& lsd, const Problem& p,
                                const SortPlan& sp, const void* go, float* gacc, void* gv,
                                void* gl, void* ga, cudaStream_t st) {
  cudaError_t err =
      cudaMemsetAsync(sp.cnt, 0, (static_cast<size_t>(sp.nkeys) + 1) * sizeof(int32_t), st);
  if (err != cudaSuccess) return err;
  {
    const int64_t grid = ls.grid;
#define MSDA_DOTS_CALL(VB, VPL) err = dots_one<T, TS, NDIM, VB, VPL>(p, sp, go, gl, ga, st, grid); break
    MSDA_FWD_SHAPE_SWITCH(ls.vb, ls.vpl, MSDA_DOTS_CALL)
#undef MSDA_DOTS_CALL
    if (err != cudaSuccess) return err;
  }
  const int32_t nblk = static_cast<int32_t>((int64_t{sp.nkeys} + kScanTile - 1) / kScanTile);
  msda_scan_reduce_kernel<<<nblk, kScanThreads, 0, st>>>(sp.cnt, sp.nkeys, sp.bsum);
  msda_scan_top_kernel<<<1, kScanThreads, 0, st>>>(sp.bsum, nblk);
  msda_scan_down_kernel<<<nblk, kScanThreads, 0, st>>>(sp.cnt, sp.nkeys, sp.bsum, nblk);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  const unsigned sblocks = static_cast<unsigned>((int64_t{sp.n} + kThreads - 1) / kThreads);
  msda_place_kernel<TS, NDIM><<<sblocks, kThreads, 0, st>>>(p, sp);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if (sp.nsl > 0) {
#define MSDA_SDOTS_CALL(VB, VPL) err = sdots_one<T, TS, NDIM, VB, VPL>(p, sp, go, gl, ga, st); break
    MSDA_FWD_SHAPE_SWITCH(ls.vb, ls.vpl, MSDA_SDOTS_CALL)
#undef MSDA_SDOTS_CALL
    if (err != cudaSuccess) return err;
  }
  if (sp.nml > 0) {
    switch (p.C) {
      case 16: err = dense_mma_one<T, NDIM, 2>(p, sp, go, gacc, st); break;
      case 32: err = dense_mma_one<T, NDIM, 4>(p, sp, go, gacc, st); break;
      case 64: err = dense_mma_one<T, NDIM, 8>(p, sp, go, gacc, st); break;
      default: return cudaErrorInvalidValue;
    }
    if (err != cudaSuccess) return err;
  }
  if (sp.ndl > 0) {
    switch (lsd.vb * 16 + lsd.vpl) {
      case 16 * 16 + 1: err = dense_one<T, NDIM, 16, 1>(p, sp, go, gacc, st); break;
      case 16 * 16 + 2: err = dense_one<T, NDIM, 16, 2>(p, sp, go, gacc, st); break;
      case 8 * 16 + 1: err = dense_one<T, NDIM, 8, 1>(p, sp, go, gacc, st); break;
      case 8 * 16 + 2: err = dense_one<T, NDIM, 8, 2>(p, sp, go, gacc, st); break;
      case 4 * 16 + 1: err = dense_one<T, NDIM, 4, 1>(p, sp, go, gacc, st); break;
      case 2 * 16 + 1:
        if constexpr (sizeof(T) == 2) { err = dense_one<T, NDIM, 2, 1>(p, sp, go, gacc, st); break; }
        return cudaErrorInvalidValue;
      default: return cudaErrorInvalidValue;
    }
    if (err != cudaSuccess) return err;
  }
  if (sp.nvl > 0 && sp.vmma == 2) {
    switch (p.C) {
      case 16: err = voxel_tc_one<T, NDIM, 2>(p, sp, go, gv, st); break;
      case 32: err = voxel_tc_one<T, NDIM, 4>(p, sp, go, gv, st); break;
      case 64: err = voxel_tc_one<T, NDIM, 8>(p, sp, go, gv, st); break;
      default: return cudaErrorInvalidValue;
    }
    if (err != cudaSuccess) return err;
  } else if (sp.nvl > 0 && sp.vmma) {
    switch (p.C) {
      case 16: err = voxel_mma_one<T, NDIM, 2>(p, sp, go, gv, st); break;
      case 32: err = voxel_mma_one<T, NDIM, 4>(p, sp, go, gv, st); break;
      case 64: err = voxel_mma_one<T, NDIM, 8>(p, sp, go, gv, st); break;
      default: return cudaErrorInvalidValue;
    }
    if (err != cudaSuccess) return err;
  } else if (sp.nvl > 0) {
#define MSDA_VOXEL_CALL(VB, VPL) err = voxel_one<T, NDIM, VB, VPL>(p, sp, go, gv, st); break
    MSDA_FWD_SHAPE_SWITCH(ls.vb, ls.vpl, MSDA_VOXEL_CALL)
#undef MSDA_VOXEL_CALL
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

// One chunk of the sorted backward: dots (+ histogram), scan, place, the
// sorted-order dots of the large sparse levels, the dense and voxel
// value-gradient kernels.  gacc receives the dense levels'
// value gradient (+=); the caller zero-fills it before and rounds it after.
template <typename T, typename TS>
cudaError_t launch_sorted_bwd(const LaunchShape& ls, const LaunchShape& lsd, const Problem& p,
                              const SortPlan& sp, const void* go, float* gacc, void* gv,
                              void* gl, void* ga, cudaStream_t st) {
  return ls.ndim == 2 ? sorted_chunk<T, TS, 2>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st)
                      : sorted_chunk<T, TS, 3>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st);
}

#define MSDA_DECLARE_SORTED(T, TS)                                                            \
  extern template cudaError_t launch_sorted_bwd<T, TS>(const LaunchShape&, const LaunchShape&, \
                                                       const Problem&, const SortPlan&,        \
                                                       const void*, float*, void*, void*,      \
                                                       void*, cudaStream_t);
#define MSDA_INSTANTIATE_SORTED(T, TS)                                                        \
  template cudaError_t launch_sorted_bwd<T, TS>(const LaunchShape&, const LaunchShape&,        \
                                                const Problem&, const SortPlan&, const void*,  \
                                                float*, void*, void*, void*, cudaStream_t);

}  // namespace msda
