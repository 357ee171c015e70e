// msda_binned_launch.cuh -- host-side launch sequence of the binned backward
// (counting sort of the samples into tiles, then the tile kernel).  Included
// by the msda_inst_*.cu files, one (value dtype, sampling dtype) pair each.
#pragma once

#include "msda_binned.cuh"

namespace msda {

struct BinLaunch {
  int ndim;
  int64_t nb;            // buckets = B * H * ntl
  int smem_main;         // dynamic shared memory of the tile kernel
  int fp32_value;        // value dtype is fp32: atomic levels accumulate in grad_value
};

// Exclusive scan of n int32 values: out[0..n) = prefix, out[n] = total;
// out2 (optional) receives a copy of out[0..n).  tmp holds ceil(n / 8192) ints.
inline cudaError_t scan_exclusive(const int32_t* in, int64_t n, int32_t* out, int32_t* out2,
                                  int32_t* tmp, cudaStream_t st) {
  const int64_t per_block = static_cast<int64_t>(kScanThreads) * kScanItems;
  const int64_t nblocks = (n + per_block - 1) / per_block;
  if (nblocks == 0) return cudaMemsetAsync(out, 0, sizeof(int32_t), st);
  msda_scan_reduce_kernel<<<static_cast<unsigned>(nblocks), kScanThreads, 0, st>>>(in, n, tmp);
  msda_scan_top_kernel<<<1, kScanThreads, 0, st>>>(tmp, nblocks);
  msda_scan_apply_kernel<<<static_cast<unsigned>(nblocks), kScanThreads, 0, st>>>(in, n, tmp,
                                                                                   out, out2);
  return cudaGetLastError();
}

template <typename T, typename TS>
cudaError_t launch_bwd_binned(const BinLaunch& bl, const Problem& p, const BinPlan& bp,
                              const BinBuffers& bb, const void* grad_out, void* grad_value,
                              void* grad_loc, void* grad_attn, cudaStream_t st) {
  cudaError_t err;
  const int64_t nb = bl.nb;
  // 1. zero the bucket counters, the work-item counter and the fp32
  //    accumulator of the atomic levels.
  if ((err = cudaMemsetAsync(bb.counts, 0, nb * sizeof(int32_t), st)) != cudaSuccess) return err;
  if ((err = cudaMemsetAsync(bb.item_counter, 0, sizeof(int32_t), st)) != cudaSuccess) return err;
  if (bp.atomic_mask) {
    if (bl.fp32_value) {
      // Accumulate straight into grad_value: zero the atomic levels' keys.
      for (int l = 0; l < p.L; ++l) {
        if (!((bp.atomic_mask >> l) & 1)) continue;
        const size_t row = static_cast<size_t>(p.H * p.C) * sizeof(float);
        int64_t nkey = static_cast<int64_t>(p.lv.size[l][0]) * p.lv.size[l][1] * p.lv.size[l][2];
        err = cudaMemset2DAsync(static_cast<float*>(grad_value) + p.lv.start[l] * p.H * p.C,
                                static_cast<size_t>(p.K) * row, 0, nkey * row,
                                static_cast<size_t>(p.B), st);
        if (err != cudaSuccess) return err;
      }
    } else {
      const size_t bytes = static_cast<size_t>(p.B * bp.acc_keys * p.H * p.C) * sizeof(float);
      if ((err = cudaMemsetAsync(bb.acc, 0, bytes, st)) != cudaSuccess) return err;
    }
  }
  // 2. counting sort of the sample records into buckets.
  const unsigned bin_grid = static_cast<unsigned>(p.B * p.H * bp.nchunk);
  const size_t bin_smem = static_cast<size_t>(bp.ntl) * sizeof(int32_t);
  auto count_k = bl.ndim == 2 ? msda_bin_kernel<TS, 2, false> : msda_bin_kernel<TS, 3, false>;
  auto fill_k = bl.ndim == 2 ? msda_bin_kernel<TS, 2, true> : msda_bin_kernel<TS, 3, true>;
  if (bin_smem * 2 > 48 * 1024) {
    if ((err = cudaFuncSetAttribute(count_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(bin_smem))) != cudaSuccess)
      return err;
    if ((err = cudaFuncSetAttribute(fill_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(bin_smem * 2))) != cudaSuccess)
      return err;
  }
  count_k<<<bin_grid, 512, bin_smem, st>>>(p, bp, bb);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if ((err = scan_exclusive(bb.counts, nb, bb.starts, bb.cursor, bb.scan_tmp, st)) != cudaSuccess)
    return err;
  fill_k<<<bin_grid, 512, bin_smem * 2, st>>>(p, bp, bb);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  // 3. work items (the cursor array is free again and holds the per-bucket counts).
  msda_items_kernel<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, st>>>(bb.counts, nb, bp,
                                                                               bb.cursor);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if ((err = scan_exclusive(bb.cursor, nb, bb.item_start, nullptr, bb.scan_tmp, st)) != cudaSuccess)
    return err;
  // 4. persistent tile kernel.
  auto main_k = bl.ndim == 2 ? msda_bwd_binned_kernel<T, TS, 2> : msda_bwd_binned_kernel<T, TS, 3>;
  if ((err = cudaFuncSetAttribute(main_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  bl.smem_main)) != cudaSuccess)
    return err;
  int dev = 0, nsm = 0, occ = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, main_k, kTileThreads,
                                                           bl.smem_main)) != cudaSuccess)
    return err;
  if (occ < 1) occ = 1;
  main_k<<<static_cast<unsigned>(nsm * occ), kTileThreads, bl.smem_main, st>>>(
      p, bp, bb, static_cast<const T*>(grad_out), static_cast<T*>(grad_value),
      static_cast<TS*>(grad_loc), static_cast<TS*>(grad_attn));
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  // 5. round the atomic levels' fp32 accumulator into grad_value.
  if (bp.atomic_mask && !bl.fp32_value) {
    const int64_t n = p.B * bp.acc_keys * p.H * p.C;
    int64_t blocks = (n + 255) / 256;
    if (blocks > nsm * 16) blocks = nsm * 16;
    msda_acc_cast_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        p, bp, bb.acc, static_cast<T*>(grad_value));
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

#define MSDA_DECLARE_BINNED(T, TS)                                                            \
  extern template cudaError_t launch_bwd_binned<T, TS>(const BinLaunch&, const Problem&,       \
                                                       const BinPlan&, const BinBuffers&,      \
                                                       const void*, void*, void*, void*,       \
                                                       cudaStream_t);
#define MSDA_INSTANTIATE_BINNED(T, TS)                                                        \
  template cudaError_t launch_bwd_binned<T, TS>(const BinLaunch&, const Problem&,              \
                                                const BinPlan&, const BinBuffers&, const void*, \
                                                void*, void*, void*, cudaStream_t);

}  // namespace msda
