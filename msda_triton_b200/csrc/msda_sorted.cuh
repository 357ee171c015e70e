// msda_sorted.cuh -- the cell-sorted MSDA backward.
//
// The value gradient of MSDA is a scatter: every sample adds a*w_c*grad_out
// into the 2^d corner rows around it.  Done per sample with vector
// reductions (red.global.add), its cost is set by the L2's reduction rate --
// measured on B200 at 47 G rows/s for 128-byte fp32 rows and 79 G rows/s for
// 64-byte bf16 rows, against 250 G rows/s for plain 64-byte row gathers.  This
// path groups the samples by the cell they fall in (a counting sort keyed by
// (b, h, level, cell)) and forms the value gradient without per-sample
// reductions:
//
//   sparse levels ("voxel" levels, few samples per cell): each value row's
//     gradient is GATHERED from the samples of the 2^d cells around it --
//     msda_voxel_kernel sums them in fp32 registers and stores the row once.
//     No reductions, no zero-fill, one rounding per element.
//   dense levels (many samples per cell): msda_dense_kernel walks the sorted
//     samples of each cell in segments and keeps the cell's 2^d corner
//     gradients in registers, flushing them with one fp32 vector reduction
//     per corner and segment instead of one per sample.
//
// grad_attn and grad_loc need no sort: msda_dots_kernel computes them in
// query order (the forward's gather plus the corner dot products), and
// counts the samples per cell on the way -- except on the large sparse
// levels, whose rows a query-order pass fetches from DRAM for every touch:
// msda_sdots_kernel takes those in sorted (cell) order.
//
// Pipeline for one chunk of batch entries (all on one stream):
//   msda_dots_kernel       grad_attn, grad_loc; rank = atomicAdd(count[key], 1)
//   msda_scan_*            counts -> exclusive bucket starts
//   msda_place_kernel      record (a, fractions, grad_out row, key) at start[key] + rank
//   msda_sdots_kernel      grad_attn, grad_loc of the large sparse levels, in sorted order
//   msda_sdots_finish_kernel  ... staged, then written out in query order
//   msda_dense_kernel      dense-level value gradient, per cell segment
//   msda_voxel_kernel      sparse-level value gradient, gathered per value row
//                          (msda_voxel_mma_kernel: the same on the tensor cores)
//
// Cells.  A sample at level l falls in the cell of its lower corner
// (i0x, i0y[, i0z]) with each i0 in [-1, size-1] (grid_sample's corner
// range for in-range and clamped locations); cell indices are i0 + 1, so the
// level has (W+1)(H+1)[(D+1)] cells plus one "dead" bucket for samples with
// no corner inside the level (locations far outside [0, 1] without the
// clamp, NaN).  Every (b, h, level) owns exactly Q*P consecutive sorted
// positions.  The value row at voxel (vx, vy, vz) is a corner of the cells
// with i0 in {v-1, v} on every axis.
//
// Reference kernel this replaces: _bwd_kernel (src/msda_triton/triton/
// msda_3d.py:291-653) and _bwd_kernel_2d (triton/msda_2d.py:263-510).
#pragma once

#include "msda_kernels.cuh"

namespace msda {

// n / d for 0 <= n < 2^31 as one 64-bit multiply and shift: with
// l = ceil(log2 d) and m = ceil(2^(31+l) / d), floor(n*m / 2^(31+l)) equals
// floor(n / d) because the rounding error n*(m*d - 2^(31+l)) / (d*2^(31+l))
// stays below 1/d.
struct FastDiv {
  uint32_t m;
  uint32_t shift;
};

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(n) * f.m) >> f.shift);
}

// Tile of the voxel kernels on one level: NZ voxel planes x NY rows x TX
// voxels (NZ = 1 for msda_voxel_kernel).
struct VoxTile {
  int32_t tx, ny, nz; // voxels per row segment, rows and planes per CTA
  int32_t ntx, nty;   // tiles along x and y
};

// One sample at its sorted position (32 bytes: one sector).
struct __align__(32) SRec {
  float a;        // attention weight
  float f[3];     // fractional offsets inside the cell
  uint32_t row;   // (b, q, h) row of grad_out
  int32_t key;    // bucket key
  uint32_t idx;   // sample index (b, q, h, l, p) inside the chunk
  uint32_t pass;  // bit a: the location's gradient passes the clamp on axis a
};

// Everything the sorted pipeline adds to Problem (one chunk of batch
// entries; the Problem's pointers are already offset to the chunk and its B
// is the chunk's batch count).
struct SortPlan {
  int32_t n;                       // samples in the chunk: B*Q*H*L*P
  int32_t nkeys;                   // bucket keys: B*H*seg_keys
  int32_t seg_keys;                // keys per (b, h): sum over levels of cells_l + 1
  int32_t lvl_base[kMaxLevels];    // first key of level l inside a (b, h) block
  int32_t cells[kMaxLevels][3];    // cell-grid extent per axis (size + 1; 1 for z in 2D)
  int32_t voxel_mask;              // levels whose value gradient msda_voxel_kernel gathers
  int32_t ndl;                     // dense levels on msda_dense_kernel (CUDA cores)
  int32_t dl_level[kMaxLevels];    // k-th such level
  int32_t dchunk;                  // sorted positions per msda_dense_kernel CTA
  int32_t dchunks;                 // msda_dense_kernel CTAs per (b, h, dense level)
  int32_t dlog2g, dnv;             // msda_dense_kernel lane group: 2^dlog2g lanes, dnv chunks per row
  FastDiv div_dnv;                 // / dnv
  int32_t dsmem;                   // msda_dense_kernel dynamic shared memory
  int32_t nml;                     // dense levels on msda_dense_mma_kernel (16-bit, C = 16/32/64)
  int32_t ml_level[kMaxLevels];    // k-th such level
  int32_t dsmem_mma;               // its dynamic shared memory
  int32_t nvl;                     // voxel levels
  int32_t vl_level[kMaxLevels];    // k-th voxel level
  VoxTile vl_tile[kMaxLevels];     // msda_voxel_kernel tile of the k-th voxel level
  int32_t vl_ubase[kMaxLevels + 1];// first voxel-kernel CTA of the k-th voxel level inside a (b, h) block
  int32_t units_per_bh;            // vl_ubase[nvl]
  int32_t vcap;                    // samples staged per round by msda_voxel_kernel
  int32_t vnv;                     // msda_voxel_kernel: VB-byte chunks per channel row
  FastDiv div_nv;                  // / vnv
  int32_t vsmem;                   // its dynamic shared memory
  int32_t vmma;                    // voxel levels on the tensor cores (16-bit, C = 16/32/64):
                                   // 1 msda_voxel_mma_kernel, 2 msda_voxel_tc_kernel
  FastDiv div_lp, div_p, div_h, div_l, div_q;
  int32_t sdots_mask;              // levels whose dot products msda_sdots_kernel takes in sorted order
  int32_t nsl;                     // such levels
  int32_t sl_level[kMaxLevels];    // k-th such level
  int32_t sd_per;                  // sorted positions per msda_sdots_kernel CTA
  int32_t sd_chunks;               // msda_sdots_kernel CTAs per (b, h, level)
  FastDiv div_cx[kMaxLevels], div_cy[kMaxLevels];  // / cells[l][0], / cells[l][1]
  int32_t* cnt;                    // nkeys + 1: counts, then exclusive starts
  int32_t* bsum;                   // scan block sums
  int32_t* pos;                    // n: each sample's rank inside its bucket
  SRec* srec;                      // n: the samples in sorted order
  float4* sd_stage;                // B*Q*H*nsl*P: msda_sdots_kernel's results in query order
};

// Bucket key of a resolved sample: the (b, h) block, the level's key range,
// then the cell (z-major, x fastest), or the level's dead bucket.
template <int NDIM>
__device__ __forceinline__ int32_t bucket_key(const Point<NDIM>& pt, const int32_t* sz,
                                              const int32_t* cells, int32_t base) {
  bool dead = false;
  int32_t c = 0;
  int32_t ncell = 1;
#pragma unroll
  for (int a = NDIM - 1; a >= 0; --a) {
    const int32_t i = pt.i0[a] + 1;
    dead |= static_cast<uint32_t>(i) > static_cast<uint32_t>(sz[a]);
    c = c * cells[a] + i;
    ncell *= cells[a];
  }
  return base + (dead ? ncell : c);
}

// Level geometry from the host-resolved table (the sorted path requires
// host shapes).
__device__ __forceinline__ LevelGeom level_geom_tab(const Problem& p, int l, int64_t key_bytes) {
  LevelGeom g;
  g.sz[0] = p.lv.size[l][0];
  g.sz[1] = p.lv.size[l][1];
  g.sz[2] = p.lv.size[l][2];
  g.start = p.lv.start[l];
  g.dx = key_bytes;
  g.dy = key_bytes * g.sz[0];
  g.dz = g.dy * g.sz[1];
  return g;
}

// Plain (shared-memory) loads of one chunk.
template <int VB> __device__ __forceinline__ Raw<VB> ld_shared_chunk(const void* p);
template <> __device__ __forceinline__ Raw<16> ld_shared_chunk<16>(const void* p) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  Raw<16> r; r.w[0] = v.x; r.w[1] = v.y; r.w[2] = v.z; r.w[3] = v.w; return r;
}
template <> __device__ __forceinline__ Raw<8> ld_shared_chunk<8>(const void* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  Raw<8> r; r.w[0] = v.x; r.w[1] = v.y; return r;
}
template <> __device__ __forceinline__ Raw<4> ld_shared_chunk<4>(const void* p) {
  Raw<4> r; r.w[0] = *reinterpret_cast<const unsigned int*>(p); return r;
}
template <> __device__ __forceinline__ Raw<2> ld_shared_chunk<2>(const void* p) {
  Raw<2> r; r.h = *reinterpret_cast<const unsigned short*>(p); return r;
}

// Asynchronous global -> shared copies (cp.async, sm_80+): a staging loop
// issues all of its copies before any completes, so a phase costs one memory
// round trip instead of one per loop iteration.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
template <int N>
__device__ __forceinline__ void cp_async(void* dst, const void* src) {
  static_assert(N == 4 || N == 8 || N == 16, "cp.async copies 4, 8 or 16 bytes");
  if constexpr (N == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "n"(N)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// Shared-memory accesses by 32-bit shared-window address.
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void sts_u16(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(static_cast<unsigned short>(v)) : "memory");
}
// One VB-byte chunk, asynchronously where cp.async has the width.
template <int VB>
__device__ __forceinline__ void stage_chunk(void* dst, const void* src) {
  if constexpr (VB >= 4) cp_async<VB>(dst, src);
  else st_chunk<VB>(dst, ld_chunk<VB>(src));
}

// A whole 32-byte record as one 256-bit access (ld/st .v8.b32, sm_100):
// one memory request per record instead of two.
__device__ __forceinline__ void st_rec(SRec* dst, const SRec& r) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&r);
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void ld_rec(const SRec* src, uint4& r0, uint4& r1) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r0.x), "=r"(r0.y), "=r"(r0.z), "=r"(r0.w), "=r"(r1.x), "=r"(r1.y),
                 "=r"(r1.z), "=r"(r1.w)
               : "l"(src));
}

// ------------------------------------------------------------------ dots
// grad_attn and grad_loc in query order, as the gather/scatter backward
// computes them (one lane group per (b, q, h) row, the row's grad_out chunk
// loaded once), without the value-gradient scatter.  Each sample's four
// results (d out/d attn, d out/d index per axis) are lane partials over the
// row's channel chunks; kDotBatch samples are reduced together by a
// transposed butterfly -- each step halves the values a lane keeps -- so a
// sample costs a few shuffles instead of a full butterfly of four values.
// The lane that ends with a sample's grad_attn also counts the sample into
// its bucket (the counting sort's histogram) and keeps its rank there.
//
// Levels in sp.sdots_mask (the large sparse ones, whose value rows do not
// stay in L2 between the scattered touches of a query-order pass) are only
// counted here; msda_sdots_kernel takes their dot products after the sort.
constexpr int kDotBatch = 2;

// Lane bookkeeping of the transposed reduction of NV = 4 * kDotBatch values
// over a lane group of G lanes.
struct DotLanes {
  unsigned gmask;  // the group's lanes
  int vbase;       // first of the values this lane keeps
  int nkeep;       // values kept
  bool writer;     // lanes above NV hold duplicates
};

__device__ __forceinline__ DotLanes dot_lanes(int G, int j, int lane) {
  constexpr int NV = kDotBatch * 4;
  DotLanes dl;
  dl.gmask = G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane & ~(G - 1)));
  int steps = 0;
  dl.vbase = 0;
#pragma unroll
  for (int s = 1, half = NV / 2; s < NV; s <<= 1, half >>= 1)
    if (s < G) {
      ++steps;
      if (j & s) dl.vbase += half;
    }
  dl.nkeep = NV >> steps;
  dl.writer = G <= NV || j < NV;
  return dl;
}

// v[4 i + comp] for sample i and comp (attn, x, y, z): each step halves the
// values a lane keeps; afterwards lane j holds the group sums of
// v[dl.vbase ... dl.vbase + dl.nkeep) in v[0 ... nkeep).
__device__ __forceinline__ void dot_reduce(float* v, int G, int j, const DotLanes& dl) {
  constexpr int NV = kDotBatch * 4;
#pragma unroll
  for (int s = 1, half = NV / 2; s < NV; s <<= 1, half >>= 1) {
    if (s < G) {
      const bool up = (j & s) != 0;
#pragma unroll
      for (int t = 0; t < NV / 2; ++t) {
        if (t < half) {
          const float send = up ? v[t] : v[t + half];
          const float keep = up ? v[t + half] : v[t];
          v[t] = keep + __shfl_xor_sync(dl.gmask, send, s);
        }
      }
    }
  }
  for (int s = NV; s < G; s <<= 1) v[0] += __shfl_xor_sync(dl.gmask, v[0], s);
}

// One sample's lane partials of d out/d attn and d out/d index per axis from
// its corner dot products D[c] = <grad_out row, corner row c> (lane partial),
// factored axis by axis: ex = the x-interpolated dots, dx = their
// x-differences.
template <int NDIM>
__device__ __forceinline__ void corner_dot_grads(const float* D, const float* f, float* out) {
  constexpr int NC = 1 << NDIM;
  const float fx = f[0], fy = f[1];
  const float gx0 = __fsub_rn(1.0f, fx), gy0 = __fsub_rn(1.0f, fy);
  float ex[NC / 2], dx[NC / 2];
#pragma unroll
  for (int t = 0; t < NC / 2; ++t) {
    ex[t] = fmaf(fx, D[2 * t + 1], gx0 * D[2 * t]);
    dx[t] = D[2 * t + 1] - D[2 * t];
  }
  if constexpr (NDIM == 2) {
    out[0] = fmaf(fy, ex[1], gy0 * ex[0]);
    out[1] = fmaf(fy, dx[1], gy0 * dx[0]);
    out[2] = ex[1] - ex[0];
    out[3] = 0.0f;
  } else {
    const float fz = f[2], gz0 = __fsub_rn(1.0f, fz);
    // t = by + 2 * bz
    const float ey0 = fmaf(fy, ex[1], gy0 * ex[0]);  // z = 0, y-interpolated
    const float ey1 = fmaf(fy, ex[3], gy0 * ex[2]);  // z = 1
    out[0] = fmaf(fz, ey1, gz0 * ey0);
    out[1] = fmaf(fz, fmaf(fy, dx[3], gy0 * dx[2]), gz0 * fmaf(fy, dx[1], gy0 * dx[0]));
    out[2] = fmaf(fz, ex[3] - ex[2], gz0 * (ex[1] - ex[0]));
    out[3] = ey1 - ey0;
  }
}

// The lane's kept results (dot_reduce) stored as grad_attn / grad_loc of
// their samples: batch slot i holds sample sidx[i] (kNoSample: none), its
// attention weight sa[i] and sinfo[i] = level | clamp-pass bits << 8.
constexpr uint32_t kNoSample = 0xffffffffu;

template <typename TS, int NDIM>
__device__ __forceinline__ void store_dot_results(const Problem& p, const float* v,
                                                  const DotLanes& dl, const uint32_t* sidx,
                                                  const float* sa, const int32_t* sinfo,
                                                  TS* grad_loc, TS* grad_attn) {
  constexpr int NV = kDotBatch * 4;
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    if (t < dl.nkeep) {
      const int idx = dl.vbase + t;
      const int slot = idx >> 2, comp = idx & 3;
      float a = 0.0f;
      uint32_t si = kNoSample;
      int32_t info = 0;
#pragma unroll
      for (int i = 0; i < kDotBatch; ++i)
        if (i == slot) { a = sa[i]; si = sidx[i]; info = sinfo[i]; }
      if (si == kNoSample) continue;
      if (comp == 0) {
        grad_attn[si] = Elem<TS>::from_f(v[t]);
      } else if (comp - 1 < NDIM) {
        const int ax = comp - 1, ls = info & 0xff;
        const float val = ((info >> (8 + ax)) & 1)
                              ? a * v[t] * static_cast<float>(p.lv.size[ls][ax]) : 0.0f;
        grad_loc[static_cast<int64_t>(si) * NDIM + ax] = Elem<TS>::from_f(val);
      }
    }
  }
}

// msda_sdots_kernel's variant of store_dot_results: the results land in the
// (row, sorted-dots level, point) slot of sp.sd_stage as fp32 (grad_attn,
// grad_loc per axis), which msda_sdots_finish_kernel then writes out in query
// order.  Scattered 2-byte stores straight into grad_attn / grad_loc would
// each touch a line the query-order pass filled long before: a DRAM
// read-modify-write per store.
template <int NDIM>
__device__ __forceinline__ void stage_dot_results(const Problem& p, const SortPlan& sp,
                                                  const float* v, const DotLanes& dl,
                                                  const uint32_t* sidx, const float* sa,
                                                  const int32_t* sinfo, int li) {
  constexpr int NV = kDotBatch * 4;
#pragma unroll
  for (int t = 0; t < NV; ++t) {
    if (t < dl.nkeep) {
      const int idx = dl.vbase + t;
      const int slot = idx >> 2, comp = idx & 3;
      float a = 0.0f;
      uint32_t si = kNoSample;
      int32_t info = 0;
#pragma unroll
      for (int i = 0; i < kDotBatch; ++i)
        if (i == slot) { a = sa[i]; si = sidx[i]; info = sinfo[i]; }
      if (si == kNoSample || comp > NDIM) continue;
      const int ls = info & 0xff;
      float val = v[t];
      if (comp > 0) {
        const int ax = comp - 1;
        val = ((info >> (8 + ax)) & 1) ? a * val * static_cast<float>(p.lv.size[ls][ax]) : 0.0f;
      }
      const uint32_t row = fdiv(si, sp.div_lp);
      const uint32_t pp = si - row * static_cast<uint32_t>(p.L * p.P) -
                          static_cast<uint32_t>(ls) * static_cast<uint32_t>(p.P);
      const int64_t e = (static_cast<int64_t>(row) * sp.nsl + li) * p.P + pp;
      reinterpret_cast<float*>(sp.sd_stage + e)[comp] = val;
    }
  }
}

template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads, 4)
    msda_dots_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                     TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;
  constexpr int NV = kDotBatch * 4;
  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  uint64_t r = tid >> p.log2g;
  const int G = 1 << p.log2g;
  const int j = static_cast<int>(tid & static_cast<uint64_t>(G - 1));
  const int lane = static_cast<int>(threadIdx.x & 31u);
  // rows past the end stay (on row 0, storing nothing) for the group shuffles
  const bool active = r < static_cast<uint64_t>(p.B * p.Q * p.H);
  if (!active) r = 0;
  const RowCoord rc = decode_row(static_cast<uint32_t>(r), p);
  const int64_t row = (rc.b * p.Q + rc.q) * p.H + rc.h;
  const int64_t key_bytes = key_stride(p) * static_cast<int64_t>(sizeof(T));
  const char* vbase = static_cast<const char*>(p.value) +
                      bh_base(p, rc.b, rc.h, p.K) * static_cast<int64_t>(sizeof(T));
  const int LP = static_cast<int>(p.L * p.P);
  const TS* lrow = static_cast<const TS*>(p.loc) + row * LP * NDIM;
  const TS* arow = static_cast<const TS*>(p.attn) + row * LP;
  const int32_t kbh = (static_cast<int32_t>(rc.b) * static_cast<int32_t>(p.H) +
                       static_cast<int32_t>(rc.h)) * sp.seg_keys;

  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) has[v] = j + v * G < p.nv;
  Raw<VB> gor[VPL];  // the row's grad_out chunks
  {
    const char* gorow = reinterpret_cast<const char*>(grad_out) +
                        row * p.C * static_cast<int64_t>(sizeof(T));
#pragma unroll
    for (int v = 0; v < VPL; ++v)
      gor[v] = has[v] ? ld_chunk<VB>(gorow + (j + v * G) * VB) : raw_zero<VB>();
  }
  const DotLanes dl = dot_lanes(G, j, lane);

  // Rounds of G samples: lane j resolves sample r0 + j (and takes its rank
  // in its bucket), then the group walks the round's samples kDotBatch at a
  // time with the resolved samples broadcast from their lanes.
  for (int r0 = 0; r0 < LP; r0 += G) {
    SampleMeta mine;
    mine.key0 = 0;
    mine.info = kMetaSkip;
    mine.f[0] = mine.f[1] = mine.f[2] = 0.0f;
    mine.a = 0.0f;
    int32_t rank = -1;
    const int sj = r0 + j;
    if (sj < LP) {
      const int l = static_cast<int>(fdiv(static_cast<uint32_t>(sj), sp.div_p));
      const LevelGeom g = level_geom_tab(p, l, key_bytes);
      const Point<NDIM> pt = load_point<TS, NDIM>(lrow + sj * NDIM, g.sz, p);
      mine = make_meta<NDIM>(pt, g, Elem<TS>::to_f(arow[sj]), l);
      if ((sp.sdots_mask >> l) & 1) mine.info |= kMetaSkip;
      if (active)
        rank = atomicAdd(sp.cnt + bucket_key<NDIM>(pt, g.sz, sp.cells[l], kbh + sp.lvl_base[l]),
                         1);
    }
    const int nr = LP - r0 < G ? LP - r0 : G;
    // a round wholly inside levels taken in sorted order has no dot products
    // here (uniform across the warp: every row has the same level layout)
    bool skip_round = true;
    {
      const int lf = static_cast<int>(fdiv(static_cast<uint32_t>(r0), sp.div_p));
      const int ll = static_cast<int>(fdiv(static_cast<uint32_t>(r0 + nr - 1), sp.div_p));
      for (int lv = lf; lv <= ll; ++lv) skip_round = skip_round && ((sp.sdots_mask >> lv) & 1);
    }
    if (skip_round) {
      if (rank >= 0) sp.pos[row * LP + sj] = rank;
      continue;
    }
    for (int t0 = 0; t0 < nr; t0 += kDotBatch) {
      float v[NV];
      float sa[kDotBatch];
      uint32_t sidx[kDotBatch];
      int32_t sinfo[kDotBatch];
#pragma unroll
      for (int i = 0; i < kDotBatch; ++i) {
        v[4 * i] = v[4 * i + 1] = v[4 * i + 2] = v[4 * i + 3] = 0.0f;
        sa[i] = 0.0f;
        sidx[i] = kNoSample;
        sinfo[i] = 0;
        const int t = t0 + i;
        if (t < nr) {
          const SampleMeta m = shfl_meta<NDIM>(mine, t, G);
          if (!(m.info & kMetaSkip)) {
            const int l = static_cast<int>((m.info >> 12) & 0xfu);
            const LevelGeom g = level_geom_tab(p, l, key_bytes);
            Raw<VB> raw[NC][VPL];
            gather_meta_corners<T, NDIM, VB, VPL>(p, m, g, vbase, key_bytes, j * VB, G, has, raw);
            float D[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
              float dot = 0.0f;
#pragma unroll
              for (int vv = 0; vv < VPL; ++vv) dot = DotChunk<T, VB>::fma(gor[vv], raw[c][vv], dot);
              D[c] = dot;
            }
            corner_dot_grads<NDIM>(D, m.f, v + 4 * i);
            sa[i] = m.a;
            sinfo[i] = l | static_cast<int32_t>(((m.info >> 8) & 7u) << 8);
            sidx[i] = static_cast<uint32_t>(row * LP + r0 + t);
          }
        }
      }
      dot_reduce(v, G, j, dl);
      if (active && dl.writer)
        store_dot_results<TS, NDIM>(p, v, dl, sidx, sa, sinfo, grad_loc, grad_attn);
    }
    if (rank >= 0) sp.pos[row * LP + sj] = rank;
  }
}

// ------------------------------------------------------------------ sdots
// grad_attn and grad_loc of the levels in sp.sdots_mask, in sorted order: a
// lane group per record, kDotBatch records at a time, with the dot products
// and reduction of msda_dots_kernel.  The records of a (b, h, level) run
// through the level's cells z-major, so the value rows a CTA touches lie in
// a few consecutive planes and stay in L2; consecutive CTAs take the same
// stretch of positions of the eight heads (CTA index: head fastest), whose
// rows share the value lines.  The sample's grad_out row is gathered per
// record (grad_out of a batch entry is a few tens of MB and stays in L2).
constexpr int kSdotsPer = 256;  // default sorted positions per msda_sdots_kernel CTA (one round)

template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads, 4)
    msda_sdots_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                      TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;
  constexpr int NV = kDotBatch * 4;
  // CTA -> (b, level, head group, stretch, head in group), fastest last:
  // the heads of a group (p.hg: those whose rows share 128-byte value lines;
  // one head for a head-major value) walk the same stretch of positions
  // together, and one group's value lines and grad_out rows (a quarter of
  // the batch entry's for groups of 2 of 8 heads) stay in L2.
  uint32_t u = blockIdx.x;
  const uint32_t nch = static_cast<uint32_t>(sp.sd_chunks);
  const uint32_t hgs = p.head_major ? 1u : static_cast<uint32_t>(p.hg);
  const uint32_t ngrp = static_cast<uint32_t>(p.H) / hgs;
  const uint32_t hi = u % hgs;
  u /= hgs;
  const int32_t k = static_cast<int32_t>(u % nch);
  u /= nch;
  const int32_t h = static_cast<int32_t>((u % ngrp) * hgs + hi);
  u /= ngrp;
  const int32_t li = static_cast<int32_t>(u % static_cast<uint32_t>(sp.nsl));
  const int64_t b = u / static_cast<uint32_t>(sp.nsl);
  const int l = sp.sl_level[li];
  const int64_t QP = p.Q * p.P;
  const int64_t bh = b * p.H + h;
  const SRec* recs = sp.srec + (bh * p.L + l) * QP;  // the (b, h, l) block of positions
  const int64_t per = sp.sd_per;
  const int64_t q_end = int64_t{k + 1} * per < QP ? int64_t{k + 1} * per : QP;

  const int G = 1 << p.log2g;
  const int j = static_cast<int>(threadIdx.x) & (G - 1);
  const int grp = static_cast<int>(threadIdx.x) >> p.log2g;
  const int groups = kThreads >> p.log2g;
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const DotLanes dl = dot_lanes(G, j, lane);
  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) has[v] = j + v * G < p.nv;

  const int64_t e = static_cast<int64_t>(sizeof(T));
  const int64_t key_bytes = key_stride(p) * e;
  const char* vbase = static_cast<const char*>(p.value) + bh_base(p, b, h, p.K) * e;
  const LevelGeom g = level_geom_tab(p, l, key_bytes);
  const int32_t kb = static_cast<int32_t>(bh) * sp.seg_keys + sp.lvl_base[l];
  const uint32_t ncell = static_cast<uint32_t>(sp.cells[l][0]) *
                         static_cast<uint32_t>(sp.cells[l][1]) *
                         static_cast<uint32_t>(sp.cells[l][2]);

  // Rounds (CTA-uniform, so every lane of a warp takes every shuffle): each
  // group takes G consecutive records; lane j decodes record q0 + j, then the
  // group walks them kDotBatch at a time.
  for (int64_t qr = int64_t{k} * per; qr < q_end; qr += int64_t{groups} * G) {
    const int64_t q0 = qr + int64_t{grp} * G;
    SampleMeta mine;
    mine.key0 = 0;
    mine.info = kMetaSkip;
    mine.f[0] = mine.f[1] = mine.f[2] = 0.0f;
    mine.a = 0.0f;
    uint32_t my_row = 0, my_idx = kNoSample;
    if (q0 + j < q_end) {
      uint4 r0, r1;
      ld_rec(recs + q0 + j, r0, r1);
      // r0 = (a, f0, f1, f2), r1 = (row, key, idx, pass)
      const uint32_t c = static_cast<uint32_t>(static_cast<int32_t>(r1.y) - kb);
      Point<NDIM> pt;
      pt.f[0] = __uint_as_float(r0.y);
      pt.f[1] = __uint_as_float(r0.z);
      pt.f[2] = __uint_as_float(r0.w);
      const uint32_t t = fdiv(c, sp.div_cx[l]);
      pt.i0[0] = static_cast<int32_t>(c - t * static_cast<uint32_t>(sp.cells[l][0])) - 1;
      if constexpr (NDIM == 3) {
        const uint32_t z = fdiv(t, sp.div_cy[l]);
        pt.i0[1] = static_cast<int32_t>(t - z * static_cast<uint32_t>(sp.cells[l][1])) - 1;
        pt.i0[2] = static_cast<int32_t>(z) - 1;
      } else {
        pt.i0[1] = static_cast<int32_t>(t) - 1;
        pt.i0[2] = 0;
      }
      // the level's dead bucket: no corner inside the level
      if (c >= ncell) pt.i0[0] = pt.i0[1] = pt.i0[2] = -2;
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) pt.pass[ax] = (r1.w >> ax) & 1u;
      mine = make_meta<NDIM>(pt, g, __uint_as_float(r0.x), l);
      my_row = r1.x;
      my_idx = r1.z;
    }
    const int64_t left = q_end - q0;
    const int nr = left <= 0 ? 0 : (left < G ? static_cast<int>(left) : G);
    for (int t0 = 0; t0 < G; t0 += kDotBatch) {
      float v[NV];
      float sa[kDotBatch];
      uint32_t sidx[kDotBatch];
      int32_t sinfo[kDotBatch];
#pragma unroll
      for (int i = 0; i < kDotBatch; ++i) {
        v[4 * i] = v[4 * i + 1] = v[4 * i + 2] = v[4 * i + 3] = 0.0f;
        sa[i] = 0.0f;
        sidx[i] = kNoSample;
        sinfo[i] = 0;
        const int t = t0 + i;
        const SampleMeta m = shfl_meta<NDIM>(mine, t, G);
        const uint32_t grow = __shfl_sync(0xffffffffu, my_row, t, G);
        const uint32_t gidx = __shfl_sync(0xffffffffu, my_idx, t, G);
        if (t < nr) {
          Raw<VB> gor[VPL];
          {
            const char* gorow = reinterpret_cast<const char*>(grad_out) +
                                static_cast<int64_t>(grow) * p.C * e;
#pragma unroll
            for (int vv = 0; vv < VPL; ++vv)
              gor[vv] = has[vv] ? ld_chunk<VB>(gorow + (j + vv * G) * VB) : raw_zero<VB>();
          }
          Raw<VB> raw[NC][VPL];
          gather_meta_corners<T, NDIM, VB, VPL>(p, m, g, vbase, key_bytes, j * VB, G, has, raw);
          float D[NC];
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            float dot = 0.0f;
#pragma unroll
            for (int vv = 0; vv < VPL; ++vv) dot = DotChunk<T, VB>::fma(gor[vv], raw[c][vv], dot);
            D[c] = dot;
          }
          corner_dot_grads<NDIM>(D, m.f, v + 4 * i);
          sa[i] = m.a;
          sinfo[i] = l | static_cast<int32_t>(((m.info >> 8) & 7u) << 8);
          sidx[i] = gidx;
        }
      }
      dot_reduce(v, G, j, dl);
      if (dl.writer) stage_dot_results<NDIM>(p, sp, v, dl, sidx, sa, sinfo, li);
    }
  }
}

// The staged sorted-order results written to grad_attn / grad_loc, one
// thread per (row, sorted-dots level, point), in query order.
template <typename TS, int NDIM>
__global__ void __launch_bounds__(kThreads)
    msda_sdots_finish_kernel(const Problem p, const SortPlan sp, TS* __restrict__ grad_loc,
                             TS* __restrict__ grad_attn) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t total = p.B * p.Q * p.H * sp.nsl * p.P;
  if (e >= total) return;
  const int64_t t = e / p.P;
  const int64_t pp = e - t * p.P;
  const int64_t row = t / sp.nsl;
  const int li = static_cast<int>(t - row * sp.nsl);
  const int64_t si = row * p.L * p.P + static_cast<int64_t>(sp.sl_level[li]) * p.P + pp;
  const float4 r = sp.sd_stage[e];
  grad_attn[si] = Elem<TS>::from_f(r.x);
  grad_loc[si * NDIM] = Elem<TS>::from_f(r.y);
  grad_loc[si * NDIM + 1] = Elem<TS>::from_f(r.z);
  if constexpr (NDIM == 3) grad_loc[si * NDIM + 2] = Elem<TS>::from_f(r.w);
}

// ------------------------------------------------------------------ place
// One thread per sample: its record at start[key] + rank.
template <typename TS, int NDIM>
// Threads run over the samples head by head -- (b, h, q, l, p), samples of
// a row fastest -- so the records of a stretch of the grid land in the
// sorted blocks of one (b, h) (a few tens of MB, resident in L2) and their
// lines are completed in L2 instead of each 32-byte store costing DRAM a
// read-modify-write.
__global__ void __launch_bounds__(kThreads) msda_place_kernel(const Problem p, const SortPlan sp) {
  const uint32_t t = blockIdx.x * kThreads + threadIdx.x;
  if (t >= static_cast<uint32_t>(sp.n)) return;
  const uint32_t LP = static_cast<uint32_t>(p.L * p.P);
  const uint32_t r0 = fdiv(t, sp.div_lp);      // (b * H + h) * Q + q
  const uint32_t i = t - r0 * LP;              // l * P + p
  const uint32_t bh = fdiv(r0, sp.div_q);
  const uint32_t q = r0 - bh * static_cast<uint32_t>(p.Q);
  const uint32_t b = fdiv(bh, sp.div_h);
  const int32_t h = static_cast<int32_t>(bh - b * static_cast<uint32_t>(p.H));
  const int32_t l = static_cast<int32_t>(fdiv(i, sp.div_p));
  const uint32_t row = (b * static_cast<uint32_t>(p.Q) + q) * static_cast<uint32_t>(p.H) +
                       static_cast<uint32_t>(h);  // (b * Q + q) * H + h
  const uint32_t s = row * LP + i;                // the sample index
  const Point<NDIM> pt = load_point<TS, NDIM>(
      static_cast<const TS*>(p.loc) + static_cast<int64_t>(s) * NDIM, p.lv.size[l], p);
  SRec rec;
  rec.a = Elem<TS>::to_f(static_cast<const TS*>(p.attn)[s]);
  rec.f[0] = pt.f[0];
  rec.f[1] = pt.f[1];
  rec.f[2] = NDIM == 3 ? pt.f[2] : 0.0f;
  rec.row = row;
  rec.key = bucket_key<NDIM>(pt, p.lv.size[l], sp.cells[l],
                             (static_cast<int32_t>(b) * static_cast<int32_t>(p.H) + h) *
                                 sp.seg_keys + sp.lvl_base[l]);
  rec.idx = s;
  rec.pass = 0u;
#pragma unroll
  for (int ax = 0; ax < NDIM; ++ax) rec.pass |= pt.pass[ax] ? (1u << ax) : 0u;
  const int32_t at = __ldg(sp.cnt + rec.key) + sp.pos[s];
  st_rec(sp.srec + at, rec);
}

// ------------------------------------------------------------------ scan
// Exclusive scan of n int32 counts in place, with data[n] = total, in three
// launches: per-tile sums, a single-CTA scan of the tile sums, and the tiles'
// own scans offset by their tile's prefix.
constexpr int kScanThreads = 256;
constexpr int kScanPer = 16;
constexpr int kScanTile = kScanThreads * kScanPer;

__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t* warp_tot,
                                                        int32_t& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  if (w == 0) {
    int32_t t = lane < (kScanThreads / 32) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < (kScanThreads / 32)) warp_tot[lane] = t;  // inclusive warp prefixes
  }
  __syncthreads();
  total = warp_tot[kScanThreads / 32 - 1];
  const int32_t before = w > 0 ? warp_tot[w - 1] : 0;
  const int32_t r = before + x - v;
  __syncthreads();
  return r;
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_reduce_kernel(const int32_t* __restrict__ data, int64_t n, int32_t* __restrict__ bsum) {
  __shared__ int32_t wt[kScanThreads / 32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  int32_t sum = 0;
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int64_t k = base + i * kScanThreads + threadIdx.x;
    if (k < n) sum += data[k];
  }
  int32_t total;
  block_exclusive_scan(sum, wt, total);
  if (threadIdx.x == 0) bsum[blockIdx.x] = total;
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_top_kernel(int32_t* __restrict__ bsum, int32_t nblk) {
  __shared__ int32_t wt[kScanThreads / 32];
  int32_t carry = 0;
  for (int32_t base = 0; base < nblk; base += kScanThreads) {
    const int32_t k = base + static_cast<int32_t>(threadIdx.x);
    const int32_t v = k < nblk ? bsum[k] : 0;
    int32_t total;
    const int32_t ex = block_exclusive_scan(v, wt, total);
    if (k < nblk) bsum[k] = carry + ex;
    carry += total;
  }
  if (threadIdx.x == 0) bsum[nblk] = carry;
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_down_kernel(int32_t* __restrict__ data, int64_t n, const int32_t* __restrict__ bsum,
                          int32_t nblk) {
  __shared__ int32_t wt[kScanThreads / 32];
  // each thread scans kScanPer consecutive counts: four 16-byte loads and
  // stores when the tile is whole (tiles start 16 KB apart in a 256-byte
  // aligned buffer)
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  const int64_t e0 = base + static_cast<int64_t>(threadIdx.x) * kScanPer;
  const bool whole = base + kScanTile <= n;
  int32_t loc[kScanPer];
  if (whole) {
    const int4* src = reinterpret_cast<const int4*>(data + e0);
#pragma unroll
    for (int q = 0; q < kScanPer / 4; ++q) {
      const int4 v = src[q];
      loc[4 * q] = v.x; loc[4 * q + 1] = v.y; loc[4 * q + 2] = v.z; loc[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kScanPer; ++i) loc[i] = e0 + i < n ? data[e0 + i] : 0;
  }
  int32_t sum = 0;
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) sum += loc[i];
  int32_t total;
  int32_t run = block_exclusive_scan(sum, wt, total) + bsum[blockIdx.x];
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int32_t c = loc[i];
    loc[i] = run;
    run += c;
  }
  if (whole) {
    int4* dst = reinterpret_cast<int4*>(data + e0);
#pragma unroll
    for (int q = 0; q < kScanPer / 4; ++q)
      dst[q] = make_int4(loc[4 * q], loc[4 * q + 1], loc[4 * q + 2], loc[4 * q + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < kScanPer; ++i)
      if (e0 + i < n) data[e0 + i] = loc[i];
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) data[n] = bsum[nblk];
}


// ------------------------------------------------------------------ dense levels
// Value gradient of the dense levels.  One CTA per sp.dchunk sorted positions
// of one (b, h, dense level) -- each owns exactly Q*P consecutive positions.
// The CTA stages the positions' records and their grad_out rows in shared
// memory (cp.async: two memory round trips), cuts the positions into
// segments of one cell, at most kSegMax long, and replaces each record by
// its 2^d corner weights a * w (computed once per sample, not once per lane).
// Each segment goes to a lane group: per sample a * w_corner * grad_out is
// added to the cell's 2^d corner gradients in fp32 registers, flushed with
// one vector reduction per corner.
constexpr int kSegMax = 16;

// Rows of at most 32 fp32 accumulators per lane are held to 4 CTAs per SM
// (64 registers); wider ones keep the registers they need.
template <typename T, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads,
                                  ((1 << NDIM) * VPL * Chunk<T, VB>::EPV <= 32) ? 4 : 1)
    msda_dense_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                      float* __restrict__ gacc) {
  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;
  extern __shared__ __align__(16) unsigned char dsm[];
  const int chunkn = sp.dchunk;
  SRec* rec_s = reinterpret_cast<SRec*>(dsm);                              // chunkn
  const int64_t row_bytes = p.C * static_cast<int64_t>(sizeof(T));
  const int rowb = static_cast<int>(row_bytes);
  unsigned char* go_s = dsm + static_cast<size_t>(chunkn) * sizeof(SRec);  // chunkn * rowb
  int32_t* seg = reinterpret_cast<int32_t*>(go_s + static_cast<size_t>(chunkn) * rowb);
  int32_t* segc = seg + chunkn + 1;  // the cell (level-relative key) of each segment
  __shared__ int32_t warp_tot[kThreads / 32];

  const uint32_t u = blockIdx.x;
  const uint32_t chunk = u % static_cast<uint32_t>(sp.dchunks);
  const uint32_t r1 = u / static_cast<uint32_t>(sp.dchunks);
  const int kd = static_cast<int>(r1 % static_cast<uint32_t>(sp.ndl));
  const uint32_t bh = r1 / static_cast<uint32_t>(sp.ndl);
  const int l = sp.dl_level[kd];
  const int64_t qp = p.Q * p.P;
  const int64_t base = (static_cast<int64_t>(bh) * p.L + l) * qp + int64_t{chunk} * chunkn;
  const int cnt = static_cast<int>(min(static_cast<int64_t>(chunkn), qp - int64_t{chunk} * chunkn));
  const int32_t kl = static_cast<int32_t>(bh) * sp.seg_keys + sp.lvl_base[l];
  // records, then the grad_out rows they name
  for (int idx = threadIdx.x; idx < cnt * 2; idx += kThreads)
    cp_async<16>(reinterpret_cast<char*>(rec_s) + idx * 16,
                 reinterpret_cast<const char*>(sp.srec + base) + idx * 16);
  cp_async_wait_all();
  __syncthreads();
  const int nv = sp.dnv;
  for (int idx = threadIdx.x; idx < cnt * nv; idx += kThreads) {
    const int t = static_cast<int>(fdiv(static_cast<uint32_t>(idx), sp.div_dnv));
    const int c = idx - t * nv;
    stage_chunk<VB>(go_s + static_cast<size_t>(t) * rowb + c * VB,
                    reinterpret_cast<const char*>(grad_out) +
                        static_cast<int64_t>(rec_s[t].row) * row_bytes + c * VB);
  }
  {
    const int t0 = 2 * threadIdx.x;
    bool h0 = false, h1 = false;
    if (t0 < cnt) h0 = (t0 % kSegMax == 0) || rec_s[t0].key != rec_s[t0 - 1].key;
    if (t0 + 1 < cnt) h1 = ((t0 + 1) % kSegMax == 0) || rec_s[t0 + 1].key != rec_s[t0].key;
    int32_t total;
    const int32_t off = block_exclusive_scan(static_cast<int32_t>(h0) + static_cast<int32_t>(h1),
                                             warp_tot, total);
    if (h0) {
      seg[off] = t0;
      segc[off] = rec_s[t0].key - kl;
    }
    if (h1) {
      seg[off + (h0 ? 1 : 0)] = t0 + 1;
      segc[off + (h0 ? 1 : 0)] = rec_s[t0 + 1].key - kl;
    }
    if (threadIdx.x == 0) seg[total] = cnt;
    cp_async_wait_all();
    __syncthreads();
    if (threadIdx.x == 0) warp_tot[0] = total;
    // every grad_out copy has been issued and every key read: the records
    // become their corner weights a * w (the reference's product order)
    for (int t = threadIdx.x; t < cnt; t += kThreads) {
      const float4 af = *reinterpret_cast<const float4*>(rec_s + t);  // a, f0, f1, f2
      float wt[3][2];
      const float f[3] = {af.y, af.z, af.w};
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        if (ax < NDIM) { wt[ax][0] = __fsub_rn(1.0f, f[ax]); wt[ax][1] = f[ax]; }
        else { wt[ax][0] = 1.0f; wt[ax][1] = 0.0f; }
      }
      float aw[8];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        float w = __fmul_rn(wt[0][cc & 1], wt[1][(cc >> 1) & 1]);
        if (NDIM == 3) w = __fmul_rn(w, wt[2][(cc >> 2) & 1]);
        aw[cc] = cc < NC ? af.x * w : 0.0f;
      }
      float4* dst = reinterpret_cast<float4*>(rec_s + t);
      dst[0] = make_float4(aw[0], aw[1], aw[2], aw[3]);
      if (NDIM == 3) dst[1] = make_float4(aw[4], aw[5], aw[6], aw[7]);
    }
    __syncthreads();
  }
  const int nseg = warp_tot[0];

  const int G = 1 << sp.dlog2g;
  const int ng = kThreads >> sp.dlog2g;
  const int grp = static_cast<int>(threadIdx.x) >> sp.dlog2g;
  const int j = static_cast<int>(threadIdx.x) & (G - 1);
  const int32_t cx = sp.cells[l][0], cy = sp.cells[l][1];
  const int32_t ncell = cx * cy * sp.cells[l][2];
  const int32_t sz0 = p.lv.size[l][0], sz1 = p.lv.size[l][1], sz2 = p.lv.size[l][2];
  const int32_t b = static_cast<int32_t>(bh / static_cast<uint32_t>(p.H));
  const int32_t h = static_cast<int32_t>(bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(p.H));
  const int64_t kshift = p.acc_compact ? p.acc_start[l] : p.lv.start[l];
  float* gbase = gacc + bh_base(p, b, h, p.acc_keys) + kshift * key_stride(p) + j * EPV;
  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) has[v] = (j + v * G < nv);

  for (int sg = grp; sg < nseg; sg += ng) {
    const int ta = seg[sg], tb = seg[sg + 1];
    const int32_t c = segc[sg];
    if (c >= ncell) continue;  // the dead bucket: no corner inside the level
    // the cell's lower corner and which of its corners lie inside the level
    const uint32_t cyz = fdiv(static_cast<uint32_t>(c), sp.div_cx[l]);
    const uint32_t czz = fdiv(cyz, sp.div_cy[l]);
    const int32_t ix = c - static_cast<int32_t>(cyz) * cx - 1;
    const int32_t iy = static_cast<int32_t>(cyz - czz * static_cast<uint32_t>(cy)) - 1;
    const int32_t iz = NDIM == 3 ? static_cast<int32_t>(czz) - 1 : 0;
    uint32_t vbits = 0;
#pragma unroll
    for (int cc = 0; cc < NC; ++cc) {
      const int32_t x = ix + (cc & 1), y = iy + ((cc >> 1) & 1), z = iz + ((cc >> 2) & 1);
      const bool ok = static_cast<uint32_t>(x) < static_cast<uint32_t>(sz0) &&
                      static_cast<uint32_t>(y) < static_cast<uint32_t>(sz1) &&
                      (NDIM == 2 || static_cast<uint32_t>(z) < static_cast<uint32_t>(sz2));
      vbits |= ok ? (1u << cc) : 0u;
    }
    float acc[NC][VPL][EPV];
#pragma unroll
    for (int cc = 0; cc < NC; ++cc)
#pragma unroll
      for (int v = 0; v < VPL; ++v)
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[cc][v][e] = 0.0f;
    for (int t = ta; t < tb; ++t) {
      float go[VPL][EPV];
      const unsigned char* gq = go_s + static_cast<size_t>(t) * rowb + j * VB;
#pragma unroll
      for (int v = 0; v < VPL; ++v)
        CK::unpack(has[v] ? ld_shared_chunk<VB>(gq + v * G * VB) : raw_zero<VB>(), go[v]);
      const float4 w03 = *reinterpret_cast<const float4*>(rec_s + t);
      float aw[8] = {w03.x, w03.y, w03.z, w03.w, 0.0f, 0.0f, 0.0f, 0.0f};
      if constexpr (NDIM == 3) {
        const float4 w47 = *(reinterpret_cast<const float4*>(rec_s + t) + 1);
        aw[4] = w47.x; aw[5] = w47.y; aw[6] = w47.z; aw[7] = w47.w;
      }
#pragma unroll
      for (int cc = 0; cc < NC; ++cc) {
#pragma unroll
        for (int v = 0; v < VPL; ++v)
#pragma unroll
          for (int e = 0; e < EPV; ++e) acc[cc][v][e] = fmaf(aw[cc], go[v][e], acc[cc][v][e]);
      }
    }
    const int32_t k0 = (iz * sz1 + iy) * sz0 + ix;
#pragma unroll
    for (int cc = 0; cc < NC; ++cc) {
      if (!((vbits >> cc) & 1u)) continue;
      const int32_t k = k0 + (cc & 1) + ((cc >> 1) & 1) * sz0 + ((cc >> 2) & 1) * sz0 * sz1;
      float* dst = gbase + static_cast<int64_t>(k) * key_stride(p);
#pragma unroll
      for (int v = 0; v < VPL; ++v)
        if (has[v]) red_add_f32<EPV>(dst + v * G * EPV, acc[cc][v]);
    }
  }
}

// ------------------------------------------------------------------ dense levels, tensor cores
// The same value gradient for 16-bit values (C a multiple of 16 bytes' worth
// of channels, C/8 = NT n-tiles of 8 channels) on the tensor cores.  Within
// one cell the gradient of its corners is a small product:
//   G[corner][ch] = sum over the cell's samples s of W[s][corner] * go[s][ch]
// with W = a * w_corner.  A warp takes one cell run (all its samples inside
// the CTA's positions, not capped) and walks it 16 samples at a time with
// mma.sync m16n8k16 (rows: corners, K: samples, N: channels): grad_out rows
// come from shared memory with ldmatrix.trans, the weights as two 16-bit
// halves W = W_hi + W_lo (two products per tile, fp32 accumulation), which
// keeps the weight's error near 2^-16 of W.  The corners are flushed with one
// fp32 vector reduction per lane, corner and n-tile, once per cell run.
template <typename T> struct MmaT;
template <> struct MmaT<__nv_bfloat16> {
  static __device__ __forceinline__ uint16_t bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ float value(uint16_t b) {
    return __bfloat162float(__ushort_as_bfloat16(b));
  }
  static __device__ __forceinline__ void mma(float* d, uint32_t a0, uint32_t a2, uint32_t b0,
                                             uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
  // all four A registers (rows 0-15)
  static __device__ __forceinline__ void mma4(float* d, const uint32_t* a, uint32_t b0,
                                              uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // two values rounded to the 16-bit type, the first in the low half
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};
template <> struct MmaT<__half> {
  static __device__ __forceinline__ uint16_t bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
  }
  static __device__ __forceinline__ float value(uint16_t b) {
    return __half2float(__ushort_as_half(b));
  }
  static __device__ __forceinline__ void mma(float* d, uint32_t a0, uint32_t a2, uint32_t b0,
                                             uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
  // all four A registers (rows 0-15)
  static __device__ __forceinline__ void mma4(float* d, const uint32_t* a, uint32_t b0,
                                              uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // two values rounded to the 16-bit type, the first in the low half
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Row stride (16-bit values) of the corner-weight table in shared memory:
// the CTA's positions (at most 2 * kThreads) plus 8 halves of padding (a
// 4-bank shift per row) and 8 of slack for the last row's paired loads.
constexpr int kWStride = 2 * kThreads + 8;
constexpr int kWBytes = (16 * kWStride + 8) * 2;

template <typename T, int NDIM, int NT>
__global__ void __launch_bounds__(kThreads, 4)
    msda_dense_mma_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                          float* __restrict__ gacc) {
  constexpr int NC = 1 << NDIM;
  constexpr int ROWB = NT * 16;  // grad_out row bytes (C 16-bit channels)
  extern __shared__ __align__(16) unsigned char dsm[];
  const int chunkn = sp.dchunk;
  // the records (chunkn * 32 bytes), later the corner-weight table (kWBytes)
  SRec* rec_s = reinterpret_cast<SRec*>(dsm);
  const size_t area0 = (max(static_cast<size_t>(chunkn) * sizeof(SRec),
                            static_cast<size_t>(kWBytes)) + 15) & ~size_t{15};
  unsigned char* go_s = dsm + area0;                                       // chunkn * ROWB
  int32_t* seg = reinterpret_cast<int32_t*>(go_s + static_cast<size_t>(chunkn) * ROWB);
  int32_t* segc = seg + chunkn + 1;
  // 16 zero bytes: the ldmatrix row of samples outside a run
  unsigned char* zrow = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(segc + chunkn) + 15) & ~uintptr_t{15});
  __shared__ int32_t warp_tot[kThreads / 32];

  const uint32_t u = blockIdx.x;
  const uint32_t chunk = u % static_cast<uint32_t>(sp.dchunks);
  const uint32_t r1 = u / static_cast<uint32_t>(sp.dchunks);
  const int kd = static_cast<int>(r1 % static_cast<uint32_t>(sp.nml));
  const uint32_t bh = r1 / static_cast<uint32_t>(sp.nml);
  const int l = sp.ml_level[kd];
  const int64_t qp = p.Q * p.P;
  const int64_t base = (static_cast<int64_t>(bh) * p.L + l) * qp + int64_t{chunk} * chunkn;
  const int cnt = static_cast<int>(min(static_cast<int64_t>(chunkn), qp - int64_t{chunk} * chunkn));
  const int32_t kl = static_cast<int32_t>(bh) * sp.seg_keys + sp.lvl_base[l];
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(zrow)[threadIdx.x] = 0u;
  // records, then the grad_out rows they name
  for (int idx = threadIdx.x; idx < cnt * 2; idx += kThreads)
    cp_async<16>(reinterpret_cast<char*>(rec_s) + idx * 16,
                 reinterpret_cast<const char*>(sp.srec + base) + idx * 16);
  cp_async_wait_all();
  __syncthreads();
  for (int idx = threadIdx.x; idx < cnt * NT; idx += kThreads) {
    const int t = idx / NT;
    const int c = idx - t * NT;
    cp_async<16>(go_s + static_cast<size_t>(t) * ROWB + c * 16,
                 reinterpret_cast<const char*>(grad_out) +
                     static_cast<int64_t>(rec_s[t].row) * ROWB + c * 16);
  }
  {
    // runs of one cell (no length cap)
    const int t0 = 2 * threadIdx.x;
    bool h0 = false, h1 = false;
    if (t0 < cnt) h0 = t0 == 0 || rec_s[t0].key != rec_s[t0 - 1].key;
    if (t0 + 1 < cnt) h1 = rec_s[t0 + 1].key != rec_s[t0].key;
    int32_t total;
    const int32_t off = block_exclusive_scan(static_cast<int32_t>(h0) + static_cast<int32_t>(h1),
                                             warp_tot, total);
    if (h0) {
      seg[off] = t0;
      segc[off] = rec_s[t0].key - kl;
    }
    if (h1) {
      seg[off + (h0 ? 1 : 0)] = t0 + 1;
      segc[off + (h0 ? 1 : 0)] = rec_s[t0 + 1].key - kl;
    }
    if (threadIdx.x == 0) seg[total] = cnt;
    cp_async_wait_all();
    __syncthreads();
    if (threadIdx.x == 0) warp_tot[0] = total;
    // every grad_out copy issued and every key read: the record area becomes
    // the corner weights, 16 rows of 16-bit values (rows 0-7: high halves of
    // corners 0-7, rows 8-15: low halves) of kWStride samples each; the row
    // padding makes the A-fragment loads of a warp hit 32 distinct banks.
    // Each thread first takes its (at most two) records into registers.
    float4 af[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = threadIdx.x + i * kThreads;
      af[i] = t < cnt ? *reinterpret_cast<const float4*>(rec_s + t) : make_float4(0, 0, 0, 0);
    }
    __syncthreads();
    uint16_t* wts_w = reinterpret_cast<uint16_t*>(rec_s);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = threadIdx.x + i * kThreads;
      if (t >= cnt) continue;
      float wt[3][2];
      const float f[3] = {af[i].y, af[i].z, af[i].w};
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        if (ax < NDIM) { wt[ax][0] = __fsub_rn(1.0f, f[ax]); wt[ax][1] = f[ax]; }
        else { wt[ax][0] = 1.0f; wt[ax][1] = 0.0f; }
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        float w = __fmul_rn(wt[0][cc & 1], wt[1][(cc >> 1) & 1]);
        if (NDIM == 3) w = __fmul_rn(w, wt[2][(cc >> 2) & 1]);
        const float aw = cc < NC ? af[i].x * w : 0.0f;
        const uint16_t bh16 = MmaT<T>::bits(aw);
        wts_w[cc * kWStride + t] = bh16;
        wts_w[(8 + cc) * kWStride + t] = MmaT<T>::bits(aw - MmaT<T>::value(bh16));
      }
    }
    __syncthreads();
  }
  const int nseg = warp_tot[0];

  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int g = lane >> 2, t4 = lane & 3;
  const int32_t cx = sp.cells[l][0], cy = sp.cells[l][1];
  const int32_t ncell = cx * cy * sp.cells[l][2];
  const int32_t sz0 = p.lv.size[l][0], sz1 = p.lv.size[l][1], sz2 = p.lv.size[l][2];
  const int32_t b = static_cast<int32_t>(bh / static_cast<uint32_t>(p.H));
  const int32_t h = static_cast<int32_t>(bh - static_cast<uint32_t>(b) * static_cast<uint32_t>(p.H));
  const int64_t kshift = p.acc_compact ? p.acc_start[l] : p.lv.start[l];
  const int64_t ks = key_stride(p);
  float* gbase = gacc + bh_base(p, b, h, p.acc_keys) + kshift * ks + 2 * t4;
  // 32-bit shared addresses: this lane's row of the corner-weight table
  // [16][kWStride] (high halves; the low halves 8 rows further), the
  // grad_out rows and the zero row
  const uint32_t wts_a = smem_addr(rec_s) + g * kWStride * 2;
  const uint32_t go_a = smem_addr(go_s), zrow_a = smem_addr(zrow);
  // this lane's ldmatrix row: sample kr of the 16-sample step, n-tile offset jo
  const int kr = (lane & 7) + ((lane >> 3) & 1) * 8;
  const int jo = lane >> 4;

  for (int sg = warp; sg < nseg; sg += kThreads / 32) {
    const int ta = seg[sg], tb = seg[sg + 1];
    const int32_t c = segc[sg];
    if (c >= ncell) continue;  // the dead bucket: no corner inside the level
    const uint32_t cyz = fdiv(static_cast<uint32_t>(c), sp.div_cx[l]);
    const uint32_t czz = fdiv(cyz, sp.div_cy[l]);
    const int32_t ix = c - static_cast<int32_t>(cyz) * cx - 1;
    const int32_t iy = static_cast<int32_t>(cyz - czz * static_cast<uint32_t>(cy)) - 1;
    const int32_t iz = NDIM == 3 ? static_cast<int32_t>(czz) - 1 : 0;
    float d[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.0f;
    // 16-sample steps from an even position (32-bit weight pairs); samples
    // outside the run [ta, tb) get weight 0 and the zero grad_out row
    for (int k0 = ta & ~1; k0 < tb; k0 += 16) {
      uint32_t ah0 = 0u, ah2 = 0u, al0 = 0u, al2 = 0u;
      if (g < NC) {
        const int s0 = k0 + 2 * t4;
        uint32_t w[2][2];  // [step half][hi / lo]
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int s = s0 + 8 * e;  // even: samples s, s + 1
          const uint32_t keep = (s >= ta && s < tb ? 0x0000ffffu : 0u) |
                                (s + 1 >= ta && s + 1 < tb ? 0xffff0000u : 0u);
          const bool any = keep != 0u;
          w[e][0] = any ? lds_u32(wts_a + s * 2) & keep : 0u;
          w[e][1] = any ? lds_u32(wts_a + (8 * kWStride + s) * 2) & keep : 0u;
        }
        ah0 = w[0][0];
        ah2 = w[1][0];
        al0 = w[0][1];
        al2 = w[1][1];
      }
      const int sr = k0 + kr;
      const bool rin = sr >= ta && sr < tb;
      const uint32_t rowa = go_a + static_cast<uint32_t>(rin ? sr : 0) * ROWB;
      // every n-tile's high-half product before the low halves, so that the
      // two products into one accumulator are NT instructions apart (C = 64:
      // per pair of n-tiles, within the register bound)
      constexpr int NP = NT <= 4 ? NT / 2 : 1;  // n-tile pairs per pass
#pragma unroll
      for (int jb = 0; jb < NT / 2; jb += NP) {
        uint32_t bq[NP][4];
#pragma unroll
        for (int jp = 0; jp < NP; ++jp)
          ldmatrix_x4_trans(rin ? rowa + (2 * (jb + jp) + jo) * 16 : zrow_a, bq[jp][0], bq[jp][1],
                            bq[jp][2], bq[jp][3]);
#pragma unroll
        for (int jp = 0; jp < NP; ++jp) {
          MmaT<T>::mma(d[2 * (jb + jp)], ah0, ah2, bq[jp][0], bq[jp][1]);
          MmaT<T>::mma(d[2 * (jb + jp) + 1], ah0, ah2, bq[jp][2], bq[jp][3]);
        }
#pragma unroll
        for (int jp = 0; jp < NP; ++jp) {
          MmaT<T>::mma(d[2 * (jb + jp)], al0, al2, bq[jp][0], bq[jp][1]);
          MmaT<T>::mma(d[2 * (jb + jp) + 1], al0, al2, bq[jp][2], bq[jp][3]);
        }
      }
    }
    if (g < NC) {
      const int x = ix + (g & 1), y = iy + ((g >> 1) & 1), z = iz + ((g >> 2) & 1);
      const bool ok = static_cast<uint32_t>(x) < static_cast<uint32_t>(sz0) &&
                      static_cast<uint32_t>(y) < static_cast<uint32_t>(sz1) &&
                      (NDIM == 2 || static_cast<uint32_t>(z) < static_cast<uint32_t>(sz2));
      if (ok) {
        const int32_t k = (z * sz1 + y) * sz0 + x;
        float* dst = gbase + static_cast<int64_t>(k) * ks;
#pragma unroll
        for (int j = 0; j < NT; ++j) red_add_f32<2>(dst + 8 * j, d[j]);
      }
    }
  }
}

// ------------------------------------------------------------------ voxel gather
// Value gradient of the sparse levels.  One CTA per tile of NY voxel rows x TX
// voxels at one (b, h, level, z); one warp per 32-voxel segment of a row.
// Voxel (x, y, z) is a corner of the cells with lower corner (x-1 or x, y-1
// or y, z-1 or z), so the tile's samples lie in the cell rows (y', z') =
// (y0-1 .. y0+NY-1, z-1 .. z), each row's cells x0-1 .. x0+TX-1 being one
// contiguous range of the sorted records.  The CTA stages, in rounds of
// sp.vcap samples (cp.async: three memory round trips): the range bounds, the
// records -- turned into their four (bx, by) corner weights a * w (the
// reference's product order) and their cell's x offset -- and their grad_out
// rows.  Each voxel row is stored once: no reductions, no zero-fill.

// The voxel-kernel unit: (b, h, voxel level, z, y tile, x tile) and its cell rows.
struct VoxUnit {
  uint32_t bh;
  int32_t b, h, l;
  VoxTile vt;
  int32_t W, Hs;       // level size along x and y
  int32_t x0, y0, vz;  // the tile's first voxel (vz: its first plane)
  int32_t cxn, cyn;    // cells along x and y
  int32_t kb;          // the level's first bucket key inside the (b, h) block
  int32_t nyr, ncr;    // cell rows per z, cell rows
  int32_t cw;          // range bounds per cell row
};

template <int NDIM>
__device__ __forceinline__ VoxUnit voxel_unit(const Problem& p, const SortPlan& sp) {
  VoxUnit U;
  const uint32_t u = blockIdx.x;
  U.bh = u / static_cast<uint32_t>(sp.units_per_bh);
  uint32_t rem = u - U.bh * static_cast<uint32_t>(sp.units_per_bh);
  int k = 0;
  while (k + 1 < sp.nvl && rem >= static_cast<uint32_t>(sp.vl_ubase[k + 1])) ++k;
  rem -= static_cast<uint32_t>(sp.vl_ubase[k]);
  U.l = sp.vl_level[k];
  U.vt = sp.vl_tile[k];
  U.W = p.lv.size[U.l][0];
  U.Hs = p.lv.size[U.l][1];
  const uint32_t xt = rem % static_cast<uint32_t>(U.vt.ntx);
  const uint32_t r2 = rem / static_cast<uint32_t>(U.vt.ntx);
  const uint32_t yt = r2 % static_cast<uint32_t>(U.vt.nty);
  U.vz = static_cast<int32_t>(r2 / static_cast<uint32_t>(U.vt.nty)) * U.vt.nz;
  U.x0 = static_cast<int32_t>(xt) * U.vt.tx;
  U.y0 = static_cast<int32_t>(yt) * U.vt.ny;
  U.b = static_cast<int32_t>(U.bh / static_cast<uint32_t>(p.H));
  U.h = static_cast<int32_t>(U.bh - static_cast<uint32_t>(U.b) * static_cast<uint32_t>(p.H));
  U.cxn = sp.cells[U.l][0];
  U.cyn = sp.cells[U.l][1];
  U.kb = static_cast<int32_t>(U.bh) * sp.seg_keys + sp.lvl_base[U.l];
  U.nyr = U.vt.ny + 1;
  U.ncr = (NDIM == 3 ? 2 : 1) * U.nyr;
  U.cw = U.vt.tx + 2;
  return U;
}

// The unit's range bounds, cnt_s[cr][c] = start of cell x0-1+c of cell row cr
// (cr = dz * nyr + row, the row's lower corner y0-1+row at z - dz), and the
// cell rows' offsets in the staged order, off_s[0..ncr].  Returns the unit's
// sample count.  Ends with the CTA synchronised.
template <int NDIM>
__device__ __forceinline__ int32_t voxel_bounds(const SortPlan& sp, const VoxUnit& U,
                                                int32_t* cnt_s, int32_t* off_s) {
  for (int cr = 0; cr < U.ncr; ++cr) {
    const int dz = (NDIM == 3 && cr >= U.nyr) ? 1 : 0;
    const int32_t yc = U.y0 - 1 + (cr - dz * U.nyr);  // the cell row's i0y
    const int32_t zc = NDIM == 3 ? U.vz - dz : -1;
    const int32_t krow = U.kb + ((zc + 1) * U.cyn + (yc + 1)) * U.cxn;
    for (int c = threadIdx.x; c < U.cw; c += kThreads) {
      if (yc <= U.Hs - 1)  // past the row end: its end bound
        cp_async<4>(cnt_s + cr * U.cw + c, sp.cnt + krow + min(U.x0 + c, U.cxn));
      else
        cnt_s[cr * U.cw + c] = 0;  // rows outside the level are empty
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t o = 0;
    for (int cr = 0; cr < U.ncr; ++cr) {
      off_s[cr] = o;
      o += cnt_s[cr * U.cw + U.cw - 1] - cnt_s[cr * U.cw];
    }
    off_s[U.ncr] = o;
  }
  __syncthreads();
  return off_s[U.ncr];
}

// First staging phase of a round: the records of staged positions q0 ..
// q0+nr-1 (cp.async) and each one's cell row in lo_s.
__device__ __forceinline__ void voxel_stage_records(const SortPlan& sp, const VoxUnit& U,
                                                    int32_t q0, int nr, SRec* rec_s,
                                                    int32_t* lo_s, const int32_t* cnt_s,
                                                    const int32_t* off_s) {
  for (int q = threadIdx.x; q < nr; q += kThreads) {
    const int32_t qq = q0 + q;
    int lo = 0, hi = U.ncr;  // cell row: off_s[lo] <= qq < off_s[lo + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (off_s[mid] <= qq) lo = mid; else hi = mid;
    }
    lo_s[q] = lo;
    const SRec* src = sp.srec + cnt_s[lo * U.cw] + (qq - off_s[lo]);
    cp_async<16>(reinterpret_cast<char*>(rec_s + q), src);
    cp_async<16>(reinterpret_cast<char*>(rec_s + q) + 16, reinterpret_cast<const char*>(src) + 16);
  }
}

// A staged record of cell row cr: its four (bx, by) corner weights a * w at
// the unit's z plane -- (bx, by) = (0, 0), (0, 1), (1, 0), (1, 1) -- and its
// cell's x offset in the tile (cell i0x = x0 + offset - 1).
template <int NDIM>
__device__ __forceinline__ float4 voxel_weights(const SRec& rec, int cr, const VoxUnit& U,
                                                int32_t& xoff) {
  const int dz = (NDIM == 3 && cr >= U.nyr) ? 1 : 0;
  const int32_t yc = U.y0 - 1 + (cr - dz * U.nyr);
  const int32_t zc = NDIM == 3 ? U.vz - dz : -1;
  xoff = rec.key - (U.kb + ((zc + 1) * U.cyn + (yc + 1)) * U.cxn) - U.x0;
  const float wx0 = __fsub_rn(1.0f, rec.f[0]), wx1 = rec.f[0];
  const float wy0 = __fsub_rn(1.0f, rec.f[1]), wy1 = rec.f[1];
  float w00 = __fmul_rn(wx0, wy0), w01 = __fmul_rn(wx0, wy1);
  float w10 = __fmul_rn(wx1, wy0), w11 = __fmul_rn(wx1, wy1);
  if (NDIM == 3) {
    const float wz = dz ? rec.f[2] : __fsub_rn(1.0f, rec.f[2]);
    w00 = __fmul_rn(w00, wz); w01 = __fmul_rn(w01, wz);
    w10 = __fmul_rn(w10, wz); w11 = __fmul_rn(w11, wz);
  }
  return make_float4(rec.a * w00, rec.a * w01, rec.a * w10, rec.a * w11);
}

// msda_voxel_kernel: a warp per 32-voxel row segment, lanes over channels.
// A warp walks, for each of the 2^(d-1) cell rows its voxel row touches, the
// samples of the 33 cells around its segment, every lane adding its
// channel's a * w * grad_out to the sample's two x-corners in a warp-private
// fp32 accumulator in shared memory (the lanes of a row hit 32 distinct
// banks).  The work follows the number of samples, not the busiest voxel.
template <typename T, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads)
    msda_voxel_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                      T* __restrict__ grad_value) {
  extern __shared__ __align__(16) unsigned char vsm[];
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int64_t row_bytes = p.C * static_cast<int64_t>(sizeof(T));
  const int rowb = static_cast<int>(row_bytes);
  const int nv = sp.vnv;  // VB-byte chunks per row (staging)
  const VoxUnit U = voxel_unit<NDIM>(p, sp);
  const int32_t W = U.W, Hs = U.Hs, x0 = U.x0, y0 = U.y0, vz = U.vz;
  const int nyr = U.nyr, cw = U.cw;

  float* acc_s = reinterpret_cast<float*>(vsm);                       // warps x 32 voxels x 32 lanes
  SRec* rec_s = reinterpret_cast<SRec*>(vsm + (kThreads / 32) * 32 * 32 * sizeof(float));  // vcap
  unsigned char* go_s = reinterpret_cast<unsigned char*>(rec_s + sp.vcap);               // vcap * rowb
  int32_t* lo_s = reinterpret_cast<int32_t*>(go_s + static_cast<size_t>(sp.vcap) * rowb);
  int32_t* cnt_s = lo_s + sp.vcap;                                    // ncr * cw
  int32_t* off_s = cnt_s + U.ncr * cw;                                // ncr + 1
  const int32_t total = voxel_bounds<NDIM>(sp, U, cnt_s, off_s);

  // this warp's 32-voxel segment
  const int segs = (U.vt.tx + 31) / 32;
  const int ry = warp / segs, sgi = warp - ry * segs;
  const int32_t xw = x0 + sgi * 32;  // first voxel of the segment
  const bool wactive = ry < U.vt.ny && y0 + ry < Hs && xw < W;
  float* acc = acc_s + warp * 32 * 32;

  const int ncb = (static_cast<int>(p.C) + 31) / 32;  // 32-channel blocks
  for (int cb = 0; cb < ncb; ++cb) {
    const int ch = cb * 32 + lane;
    const bool lact = ch < p.C;
#pragma unroll
    for (int v = lane; v < 32 * 32 / 4; v += 32)
      reinterpret_cast<float4*>(acc)[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    __syncwarp();
    for (int32_t q0 = 0; q0 < total; q0 += sp.vcap) {
      const int nr = min(sp.vcap, total - q0);
      if (cb == 0 || total > sp.vcap) {
        // stage the round: records, then per record its four (bx, by) corner
        // weights in place of (a, f), its cell's x offset and its grad_out row
        if (q0 > 0 || cb > 0) __syncthreads();
        voxel_stage_records(sp, U, q0, nr, rec_s, lo_s, cnt_s, off_s);
        cp_async_wait_all();
        __syncthreads();
        for (int q = threadIdx.x; q < nr; q += kThreads) {
          const SRec rec = rec_s[q];
          int32_t xoff;
          *reinterpret_cast<float4*>(rec_s + q) = voxel_weights<NDIM>(rec, lo_s[q], U, xoff);
          lo_s[q] = xoff;
          for (int c = 0; c < nv; ++c)
            stage_chunk<VB>(go_s + static_cast<size_t>(q) * rowb + c * VB,
                            reinterpret_cast<const char*>(grad_out) +
                                static_cast<int64_t>(rec.row) * row_bytes + c * VB);
        }
        cp_async_wait_all();
        __syncthreads();
      }
      if (wactive) {
#pragma unroll
        for (int dz = 0; dz < (NDIM == 3 ? 2 : 1); ++dz) {
#pragma unroll
          for (int dy = 0; dy < 2; ++dy) {
            const int cr = dz * nyr + (ry - dy + 1);
            const int32_t* crp = cnt_s + cr * cw;
            const int32_t slot0 = off_s[cr] - crp[0] - q0;  // position -> round slot
            const int c0 = sgi * 32;                        // cells c0 .. c0+32 touch the segment
            const int32_t qa = max(crp[c0] + slot0, 0);
            const int32_t qb = min(crp[min(c0 + 33, cw - 1)] + slot0, nr);
            for (int32_t q = qa; q < qb; ++q) {
              const float4 w4 = *reinterpret_cast<const float4*>(rec_s + q);
              const int vlo = lo_s[q] - 1 - sgi * 32;  // the cell's lower-x voxel in the segment
              const float g = lact ? Elem<T>::to_f(reinterpret_cast<const T*>(
                                         go_s + static_cast<size_t>(q) * rowb)[ch])
                                   : 0.0f;
              if (static_cast<unsigned>(vlo) < 32u)
                acc[vlo * 32 + lane] = fmaf(dy ? w4.y : w4.x, g, acc[vlo * 32 + lane]);
              if (static_cast<unsigned>(vlo + 1) < 32u)
                acc[(vlo + 1) * 32 + lane] = fmaf(dy ? w4.w : w4.z, g, acc[(vlo + 1) * 32 + lane]);
            }
          }
        }
      }
    }
    if (wactive) {
      const int32_t y = y0 + ry;
      const int64_t key0 = static_cast<int64_t>(p.lv.start[U.l]) + (static_cast<int64_t>(vz) * Hs + y) * W;
      const int64_t ks = key_stride(p);
      const int nvox = min(32, W - xw);
      if (p.C % 32 == 0) {
        // whole 32-channel blocks: lanes as (voxel, 8-channel chunk), one
        // 8-element vector store per lane and voxel
        __syncwarp();
        const int vv = lane >> 2, qq = lane & 3;
        T* gvb = grad_value + bh_base(p, U.b, U.h, p.K) + cb * 32 + qq * 8;
#pragma unroll
        for (int pass = 0; pass < 4; ++pass) {
          const int v = pass * 8 + vv;
          if (v < nvox) {
            const float4 a0 = *reinterpret_cast<const float4*>(acc + v * 32 + qq * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(acc + v * 32 + qq * 8 + 4);
            struct alignas(16) Oct { T e[8]; } o;
            o.e[0] = Elem<T>::from_f(a0.x); o.e[1] = Elem<T>::from_f(a0.y);
            o.e[2] = Elem<T>::from_f(a0.z); o.e[3] = Elem<T>::from_f(a0.w);
            o.e[4] = Elem<T>::from_f(a1.x); o.e[5] = Elem<T>::from_f(a1.y);
            o.e[6] = Elem<T>::from_f(a1.z); o.e[7] = Elem<T>::from_f(a1.w);
            *reinterpret_cast<Oct*>(gvb + (key0 + xw + v) * ks) = o;
          }
        }
      } else if (lact) {
        T* gvb = grad_value + bh_base(p, U.b, U.h, p.K) + ch;
        for (int v = 0; v < nvox; ++v)
          gvb[(key0 + xw + v) * ks] = Elem<T>::from_f(acc[v * 32 + lane]);
      }
    }
    if (cb + 1 < ncb) __syncwarp();
  }
}

// ------------------------------------------------------------------ voxel levels, tensor cores
// The same value gradient for 16-bit values with C = 8 * NT channels (NT 2,
// 4 or 8) as small products on the tensor cores.  A 32-voxel row segment
// gets
//   G[v][ch] = sum over the samples s of its 2^(d-1) cell rows of A[v][s] * go[s][ch]
// with A[v][s] = a * w of sample s's corner at voxel v: two entries per
// sample (its lower and upper x-corner in this row), zero elsewhere.  A warp
// walks the concatenated samples of a segment's cell rows 16 at a time with
// mma.sync m16n8k16 (rows: the segment's 32 voxels as two m-tiles, K:
// samples, N: channels).  Each step writes the 16 samples' two weights -- as
// two 16-bit halves W = W_hi + W_lo, as msda_dense_mma_kernel does -- into a
// zeroed 32 x 16 tile per half in shared memory, loads the A fragments with
// ldmatrix and clears what it wrote; the grad_out rows come with
// ldmatrix.trans from the staged rows.  Samples past the step's end read the
// zero row.  The fp32 accumulators are rounded once, staged through shared
// memory with stmatrix and stored as whole 16-byte chunks.  A sample whose
// grad_out row holds an Inf or NaN spreads NaN over its whole segment (0 *
// Inf in the product), where the reference's per-corner scatter confines it
// to the sample's corners.
//
// Tile: NZ voxel planes (2 in 3D) x NY rows x TX voxels per CTA, staged
// once for all its segments (each warp takes every eighth): the cell planes
// z0-1 .. z0+NZ-1 x cell rows y0-1 .. y0+NY-1, so a sample is staged by
// (NZ+1)/NZ x (NY+1)/NY CTAs on average.  Per staged sample the CTA keeps
// its 2^d corner weights as 16-bit halves (word (bz*2 + by)*2 + half: the
// (bx 0, bx 1) pair), its cell's x offset and its grad_out row (16-byte
// chunks XOR-swizzled by slot so that eight consecutive slots hit distinct
// banks).  Of the range bounds only those at segment edges are loaded.

// Bytes of a warp's area: its two A tiles (32 rows of 32 bytes each) or,
// after a segment's last step, its 32 output rows of 16 * nt bytes.
__host__ __device__ constexpr int vm_warp_bytes(int nt) {
  return 2 * 32 * 32 > 32 * 16 * nt ? 2 * 32 * 32 : 32 * 16 * nt;
}
// Entries of a warp's slot list (a chunk of a segment's samples).
constexpr int kVmList = 64;
// Range bounds per cell row of a tile with segs 32-voxel segments: two per
// segment (the first and past-the-last cell touching it).
__host__ __device__ constexpr int vm_bounds_per_row(int segs) { return 2 * segs; }

// Position of 16-byte chunk c in row r of a 16 * NT-byte row array: c XOR a
// function of r that puts chunk c of eight consecutive rows into eight
// distinct 16-byte bank groups.
template <int NT>
__device__ __forceinline__ int vm_swz(int c, int r) {
  return c ^ ((r / (8 / NT)) % NT);
}
// 16-bit element (row v, column j) of a 32 x 16 A tile with 32-byte rows:
// the two 8-column halves of rows 4-7 of every 8 swap places, which keeps
// ldmatrix's eight row reads in distinct bank groups.
__device__ __forceinline__ int vm_at(int v, int j) {
  return v * 16 + ((((j >> 3) ^ (v >> 2)) & 1) << 3) + (j & 7);
}

__device__ __forceinline__ void ldmatrix_x4_m(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldmatrix_x4_trans_m(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                    uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2,
                                            uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr),
               "r"(r0), "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}

// The staged form of one record for the tensor-core voxel kernel: its
// corner weights a * w (the reference's product order, w = wx * wy [* wz])
// as 16-bit halves in wt (2^(d-1) * 2 words), its cell's x offset.
template <typename T, int NDIM>
__device__ __forceinline__ void vm_stage_weights(const uint4& r0, uint32_t* wt) {
  const float a = __uint_as_float(r0.x);
  const float fx = __uint_as_float(r0.y), fy = __uint_as_float(r0.z), fz = __uint_as_float(r0.w);
  const float wx[2] = {__fsub_rn(1.0f, fx), fx};
  const float wy[2] = {__fsub_rn(1.0f, fy), fy};
  const float wz[2] = {__fsub_rn(1.0f, fz), fz};
#pragma unroll
  for (int bz = 0; bz < (NDIM == 3 ? 2 : 1); ++bz)
#pragma unroll
    for (int by = 0; by < 2; ++by) {
      uint32_t hi = 0u, lo = 0u;
#pragma unroll
      for (int bx = 0; bx < 2; ++bx) {
        float w = __fmul_rn(wx[bx], wy[by]);
        if (NDIM == 3) w = __fmul_rn(w, wz[bz]);
        const float aw = a * w;
        const uint16_t h16 = MmaT<T>::bits(aw);
        hi |= static_cast<uint32_t>(h16) << (16 * bx);
        lo |= static_cast<uint32_t>(MmaT<T>::bits(aw - MmaT<T>::value(h16))) << (16 * bx);
      }
      wt[(bz * 2 + by) * 2] = hi;
      wt[(bz * 2 + by) * 2 + 1] = lo;
    }
}

template <typename T, int NDIM, int NT>
__global__ void __launch_bounds__(kThreads, NT > 4 ? 2 : 3)
    msda_voxel_mma_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                          T* __restrict__ grad_value) {
  constexpr int ROWB = 16 * NT;                 // grad_out row bytes
  constexpr int WB = vm_warp_bytes(NT);
  constexpr int NR = NDIM == 3 ? 4 : 2;         // cell rows per voxel row
  constexpr int NWW = NR * 2;                   // weight words per staged sample
  constexpr int NW = kThreads / 32;
  extern __shared__ __align__(16) unsigned char vsm[];
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const VoxUnit U = voxel_unit<NDIM>(p, sp);
  const int nzp = NDIM == 3 ? U.vt.nz : 1;      // voxel planes of the tile
  const int D = NDIM == 3 ? p.lv.size[U.l][2] : 1;
  const int segs = (U.vt.tx + 31) / 32;         // segments per voxel row
  const int nb = vm_bounds_per_row(segs);       // range bounds per cell row
  const int nyr = U.vt.ny + 1;
  const int ncr = (NDIM == 3 ? nzp + 1 : 1) * nyr;  // cell rows (iz, iy), iz slowest

  unsigned char* zrow = vsm;                    // 16 zero bytes (32 reserved)
  unsigned char* wa_s = vsm + 32;               // warps x WB
  uint32_t* wt_s = reinterpret_cast<uint32_t*>(wa_s + NW * WB);                  // vcap x NWW
  unsigned char* go_s = reinterpret_cast<unsigned char*>(wt_s + static_cast<size_t>(sp.vcap) * NWW);
  int32_t* lo_s = reinterpret_cast<int32_t*>(go_s + static_cast<size_t>(sp.vcap) * ROWB);  // vcap
  uint16_t* lst_s = reinterpret_cast<uint16_t*>(lo_s + sp.vcap);                 // warps x kVmList
  int32_t* rng_s = reinterpret_cast<int32_t*>(lst_s + NW * kVmList);             // warps x 2 NR
  int32_t* bnd_s = rng_s + NW * 2 * NR;                                         // ncr x nb
  int32_t* off_s = bnd_s + ncr * nb;                                            // ncr + 1
  {
    // the layout inside the launch's dynamic shared memory, or no access at
    // all (checked build: bit 8 of the check word)
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if (static_cast<size_t>(reinterpret_cast<unsigned char*>(off_s + ncr + 1) - vsm) > dyn) {
#ifdef MSDA_CHECKED
      if (threadIdx.x == 0) atomicOr(p.check_flag, 8u);
#endif
      return;
    }
  }
  for (int i = threadIdx.x; i < (32 + NW * WB) / 16; i += kThreads)
    reinterpret_cast<uint4*>(vsm)[i] = make_uint4(0u, 0u, 0u, 0u);

  // range bounds at the segment edges: bnd_s[cr][2s] = start of cell 32s,
  // bnd_s[cr][2s+1] = start of cell min(32s+33, TX+1) (the end of the cells
  // touching segment s; for the last segment the row's end) of cell row cr =
  // iz * nyr + iy, whose cells have lower corner (y0-1+iy, z0-1+iz)
  for (int i = threadIdx.x; i < ncr * nb; i += kThreads) {
    const int cr = i / nb, e = i - cr * nb;
    const int iz = cr / nyr, iy = cr - iz * nyr;
    const int32_t yc = U.y0 - 1 + iy, zc = NDIM == 3 ? U.vz - 1 + iz : -1;
    const int c = (e & 1) ? min(32 * (e >> 1) + 33, U.cw - 1) : 32 * (e >> 1);
    if (yc <= U.Hs - 1 && zc <= D - 1)
      cp_async<4>(bnd_s + i, sp.cnt + U.kb + ((zc + 1) * U.cyn + (yc + 1)) * U.cxn +
                                 min(U.x0 + c, U.cxn));
    else
      bnd_s[i] = 0;  // rows outside the level are empty
  }
  cp_async_wait_all();
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t o = 0;
    for (int cr = 0; cr < ncr; ++cr) {
      off_s[cr] = o;
      o += bnd_s[cr * nb + nb - 1] - bnd_s[cr * nb];
    }
    off_s[ncr] = o;
  }
  __syncthreads();
  const int32_t total = off_s[ncr];
  const bool one_round = total <= sp.vcap;

  uint16_t* at = reinterpret_cast<uint16_t*>(wa_s + warp * WB);  // [half][32 x 16]
  const int j = lane & 15, hl = lane >> 4;      // this lane's sample of a step, its half
  // ldmatrix: this lane's A row and column block (half 0, m-tile 0); B n-tile offset
  const int ar = (lane & 7) + ((lane >> 3) & 1) * 8;
  const uint32_t a_addr = smem_addr(at + vm_at(ar, (lane >> 4) * 8));
  const int jo = lane >> 4;
  uint16_t* lst = lst_s + warp * kVmList;
  int32_t* rng = rng_s + warp * 2 * NR;
  const int nseg = segs * U.vt.ny * nzp;
  // 32-bit shared addresses of the step's accesses: this lane's list entry,
  // the x offsets, its weight half, the grad_out rows, the zero row and its
  // A-tile column (row v at + v * 32, the 8-column halves of rows 4-7 of
  // every 8 swapped: see vm_at)
  const uint32_t lst_a = smem_addr(lst) + j * 2;
  const uint32_t lo_a = smem_addr(lo_s), wt_a = smem_addr(wt_s) + hl * 4;
  const uint32_t go_a = smem_addr(go_s), zrow_a = smem_addr(zrow);
  const uint32_t tcol = smem_addr(at) + hl * 1024 + (j & 7) * 2;
  const int jb = (j >> 3) & 1;

  for (int sg0 = 0; sg0 < nseg; sg0 += NW) {
    // this warp's segment: (plane pz, row ry, segment sgi)
    const int sg = sg0 + warp;
    const int sgi = sg % segs, t = sg / segs;
    const int ry = t % U.vt.ny, pz = t / U.vt.ny;
    const int32_t xw = U.x0 + sgi * 32;
    const bool wactive = sg < nseg && U.y0 + ry < U.Hs && U.vz + pz < D && xw < U.W;
    float d[2][NT][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int jn = 0; jn < NT; ++jn) d[mi][jn][0] = d[mi][jn][1] = d[mi][jn][2] = d[mi][jn][3] = 0.0f;

    for (int32_t q0 = 0; q0 < total; q0 += sp.vcap) {
      const int nr = min(sp.vcap, total - q0);
      if (sg0 == 0 || !one_round) {
        // stage the round: per slot its cell row, record (into registers),
        // corner weights, x offset and grad_out row; at most two slots per thread
        if (q0 > 0 || sg0 > 0) __syncthreads();
        uint4 r0[2], r1[2];
        int crs[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int q = threadIdx.x + i * kThreads;
          crs[i] = -1;
          if (q < nr) {
            const int32_t qq = q0 + q;
            int lo = 0, hi = ncr;  // cell row: off_s[lo] <= qq < off_s[lo + 1]
            while (hi - lo > 1) {
              const int mid = (lo + hi) >> 1;
              if (off_s[mid] <= qq) lo = mid; else hi = mid;
            }
            crs[i] = lo;
            ld_rec(sp.srec + bnd_s[lo * nb] + (qq - off_s[lo]), r0[i], r1[i]);
          }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (crs[i] < 0) continue;
          const int q = threadIdx.x + i * kThreads;
          const int cr = crs[i];
          const int iz = cr / nyr, iy = cr - iz * nyr;
          // the cell's x offset in the tile (cell i0x = x0 + offset - 1)
          lo_s[q] = static_cast<int32_t>(r1[i].y) -
                    (U.kb + ((U.vz + iz) * U.cyn + (U.y0 + iy)) * U.cxn) - U.x0;
          uint32_t wt[NWW];
          vm_stage_weights<T, NDIM>(r0[i], wt);
          uint4* wq = reinterpret_cast<uint4*>(wt_s + static_cast<size_t>(q) * NWW);
#pragma unroll
          for (int k = 0; k < NWW / 4; ++k)
            wq[k] = make_uint4(wt[4 * k], wt[4 * k + 1], wt[4 * k + 2], wt[4 * k + 3]);
          const char* src = reinterpret_cast<const char*>(grad_out) + static_cast<int64_t>(r1[i].x) * ROWB;
#pragma unroll
          for (int c = 0; c < NT; ++c)
            cp_async<16>(go_s + static_cast<size_t>(q) * ROWB + vm_swz<NT>(c, q) * 16, src + c * 16);
        }
        cp_async_wait_all();
        __syncthreads();
      }
      if (!wactive) continue;
      // the segment's cell rows r = (dz, dy) = (r >> 1, r & 1) (lower corner
      // dz, dy below the voxel row) in this round: slots rng[r] ..
      // rng[r] + rng[NR + r] - 1
      int32_t n = 0;
      if (lane < NR) {
        const int r = lane;
        const int cr = (NDIM == 3 ? pz + 1 - (r >> 1) : 0) * nyr + (ry + 1 - (r & 1));
        const int32_t* bp = bnd_s + cr * nb;
        const int32_t slot0 = off_s[cr] - bp[0] - q0;  // position -> round slot
        const int32_t a = max(bp[2 * sgi] + slot0, 0);
        const int32_t e = min(bp[2 * sgi + 1] + slot0, nr);
        rng[r] = a;
        rng[NR + r] = max(e - a, 0);
      }
      __syncwarp();
#pragma unroll
      for (int r = 0; r < NR; ++r) n += rng[NR + r];
      for (int32_t c0 = 0; c0 < n; c0 += kVmList) {
        // the chunk's list: entries slot | r << 12
        const int m = min(kVmList, n - c0);
        for (int e = lane; e < m; e += 32) {
          int32_t rem = c0 + e;
          uint32_t ent = 0;
#pragma unroll
          for (int r = 0; r < NR; ++r) {
            const int32_t nn = rng[NR + r];
            if (rem >= 0 && rem < nn) ent = static_cast<uint32_t>(rng[r] + rem) | (r << 12);
            rem -= nn;
          }
          lst[e] = static_cast<uint16_t>(ent);
        }
        __syncwarp();
        for (int k0 = 0; k0 < m; k0 += 16) {
          const bool ok = k0 + j < m;
          uint32_t q = 0, ta = 0, tb = 0;
          bool wa_lo = false, wa_hi = false;
          if (ok) {
            const uint32_t ent = lds_u16(lst_a + k0 * 2);
            q = ent & 0xfffu;
            // the cell's lower-x voxel in the segment, and this lane's weight half
            const int vlo = static_cast<int>(lds_u32(lo_a + q * 4)) - (1 + sgi * 32);
            const uint32_t w2 = lds_u32(wt_a + q * (NWW * 4) + (ent >> 12) * 8);
            wa_lo = static_cast<unsigned>(vlo) < 32u;
            wa_hi = static_cast<unsigned>(vlo + 1) < 32u;
            ta = tcol + vlo * 32 + (((jb ^ (vlo >> 2)) & 1) << 4);
            tb = tcol + (vlo + 1) * 32 + (((jb ^ ((vlo + 1) >> 2)) & 1) << 4);
            if (wa_lo) sts_u16(ta, w2);
            if (wa_hi) sts_u16(tb, w2 >> 16);
          }
          __syncwarp();
          // B (grad_out rows) for every n-tile pair, then A one m-tile at a time
          uint32_t bq[NT / 2][4];
          const uint32_t rowa = go_a + q * ROWB;
#pragma unroll
          for (int jp = 0; jp < NT / 2; ++jp)
            ldmatrix_x4_trans_m(ok ? rowa + (vm_swz<NT>(2 * jp + jo, static_cast<int>(q)) << 4) : zrow_a,
                                bq[jp][0], bq[jp][1], bq[jp][2], bq[jp][3]);
#pragma unroll
          for (int mi = 0; mi < 2; ++mi) {
            uint32_t ah[4], al[4];
            ldmatrix_x4_m(a_addr + mi * 16 * 32, ah);
            ldmatrix_x4_m(a_addr + 1024 + mi * 16 * 32, al);
#pragma unroll
            for (int jp = 0; jp < NT / 2; ++jp) {
              MmaT<T>::mma4(d[mi][2 * jp], ah, bq[jp][0], bq[jp][1]);
              MmaT<T>::mma4(d[mi][2 * jp], al, bq[jp][0], bq[jp][1]);
              MmaT<T>::mma4(d[mi][2 * jp + 1], ah, bq[jp][2], bq[jp][3]);
              MmaT<T>::mma4(d[mi][2 * jp + 1], al, bq[jp][2], bq[jp][3]);
            }
          }
          __syncwarp();
          if (wa_lo) sts_u16(ta, 0u);
          if (wa_hi) sts_u16(tb, 0u);
        }
        __syncwarp();
      }
    }
    if (!wactive) continue;
    // round once; the 32 rows (chunks swizzled by voxel) into the warp's area
    // with stmatrix: 8x8 matrices (m-tile, half, n-tile), n-tile fastest
    unsigned char* wa = wa_s + warp * WB;
    __syncwarp();
#pragma unroll
    for (int s = 0; s < NT; ++s) {
      uint32_t rr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int mm = 4 * s + k;
        const int jn = mm % NT, hf = (mm / NT) & 1, mi = mm / (2 * NT);
        rr[k] = MmaT<T>::pack(d[mi][jn][2 * hf], d[mi][jn][2 * hf + 1]);
      }
      const int mm = 4 * s + (lane >> 3);
      const int jn = mm % NT, hf = (mm / NT) & 1, mi = mm / (2 * NT);
      const int row = 16 * mi + 8 * hf + (lane & 7);
      stmatrix_x4(smem_addr(wa + row * ROWB + vm_swz<NT>(jn, row) * 16), rr[0], rr[1], rr[2], rr[3]);
    }
    __syncwarp();
    const int32_t y = U.y0 + ry;
    const int64_t key0 =
        static_cast<int64_t>(p.lv.start[U.l]) + (static_cast<int64_t>(U.vz + pz) * U.Hs + y) * U.W;
    const int64_t ks = key_stride(p);
    const int nvox = min(32, U.W - xw);
    T* gvb = grad_value + bh_base(p, U.b, U.h, p.K);
#pragma unroll
    for (int i = lane; i < 32 * NT; i += 32) {
      const int v = i / NT, c = i % NT;
      if (v < nvox)
        *reinterpret_cast<uint4*>(gvb + (key0 + xw + v) * ks + c * 8) =
            *reinterpret_cast<const uint4*>(wa + v * ROWB + vm_swz<NT>(c, v) * 16);
    }
    // the area is the next segment's A tiles again: all zero
    __syncwarp();
    for (int i = lane; i < WB / 16; i += 32)
      reinterpret_cast<uint4*>(wa)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
  }
}

// ------------------------------------------------------------------ voxel levels, tcgen05
// The voxel-level value gradient of 16-bit values (C = 8 * NT, NT 2, 4 or 8)
// on the fifth-generation tensor cores.  A CTA takes four voxel rows of at
// most 128 voxels (3D: 2 planes x 2 rows; 2D: 4 rows); each row is one
// 128 x C fp32 accumulator in tensor memory (TMEM), formed as
//   D[v][ch] = sum over the samples s of the row's 2^(d-1) cell rows of
//              A[v][s] * go[s][ch],
// A[v][s] = a * w of sample s's corner at voxel v (two entries per sample,
// split into 16-bit high and low halves, two products).  Warp R (0-3) owns
// row R: per step of 16 staged slots it writes their weights into its
// zeroed 128 x 16 A tiles (K-major, no swizzle), fences them for the tensor
// core, and one lane issues `tcgen05.mma ... kind::f16` for the high and the
// low halves against 16 consecutive staged grad_out rows and commits to the
// row's mbarrier; the warp waits (bounded) and clears what it wrote.  The
// staged grad_out rows are the B operand in place: their chunk XOR (see
// vm_swz) is the 32/64/128-byte swizzle of the MN-major layout for 32, 64
// and 128-byte rows, so no copy is made.  A step starts at a multiple of 8
// slots and may take slots of other cell rows or past the staged ones: their
// A entries are zero and the rows past the end are zero-filled.  The
// epilogue reads the accumulators with `tcgen05.ld` (warp w: TMEM lanes
// 32 (w mod 4) ..) and stores each voxel row once in the value dtype.
// Every wait is bounded: on a timeout the warp stops issuing, the kernel
// frees its TMEM and returns, and g_msda_tc_timeouts counts it (checked
// build: bit 16 of the check word).

__device__ unsigned int g_msda_tc_timeouts;

// Shared-memory matrix descriptor (tcgen05): start address, leading and
// stride byte offsets (16-byte units), descriptor version 1, layout type
// (0: no swizzle; 6, 4, 2: 32, 64, 128-byte swizzle).
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                             uint32_t layout) {
  return static_cast<uint64_t>((addr >> 4) & 0x3fffu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (uint64_t{1} << 46) |
         (static_cast<uint64_t>(layout & 7u) << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulator, 16-bit A and B of
// type T (bf16 or f16), A K-major, B MN-major, N columns, M = 128.
template <typename T>
__device__ __forceinline__ uint32_t tc_idesc(uint32_t n) {
  const uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | (1u << 16) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mbar)
               : "memory");
}
// mbarrier phase wait with an iteration limit; false when it ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity) {
  for (int it = 0; it < (1 << 20); ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred P1;\n mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n"
        " selp.b32 %0, 1, 0, P1;\n}"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// 16 consecutive fp32 TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Layout of msda_voxel_tc_kernel's dynamic shared memory (byte offsets from
// a 1024-byte aligned base), shared with the host plan.
struct VtcLayout {
  int32_t a, go, wt, lo, cr, bnd, mbar, end;
};
__host__ __device__ constexpr int vtc_rows_extra() { return 24; }  // zero rows after the staged ones
__host__ __device__ inline VtcLayout vtc_layout(int nt, int ndim, int vcap, int ncr) {
  VtcLayout L{};
  const int rowb = 16 * nt;
  const int nww = (ndim == 3 ? 4 : 2) * 2;
  L.a = 0;                                              // 4 rows x (high, low) x 4 KB
  L.go = 4 * 2 * 4096;                                  // (vcap + extra) x rowb, 1024-aligned
  L.wt = L.go + ((vcap + vtc_rows_extra()) * rowb + 1023) / 1024 * 1024;  // vcap x nww words
  L.lo = L.wt + vcap * nww * 4;                         // vcap x 4 (x offset)
  L.cr = L.lo + vcap * 4;                               // vcap bytes (cell row iz << 4 | iy)
  L.bnd = L.cr + (vcap + 15) / 16 * 16;                 // ncr x 2 bounds, then ncr + 1 offsets
  L.mbar = L.bnd + ((ncr * 3 + 1) * 4 + 15) / 16 * 16;  // 4 mbarriers, TMEM slot, flags
  L.end = L.mbar + 64;
  return L;
}

template <typename T, int NDIM, int NT>
__global__ void __launch_bounds__(kThreads, 2)
    msda_voxel_tc_kernel(const Problem p, const SortPlan sp, const T* __restrict__ grad_out,
                         T* __restrict__ grad_value) {
  constexpr int ROWB = 16 * NT;                 // grad_out row bytes
  constexpr int N = 8 * NT;                     // channels: accumulator columns per voxel row
  constexpr int NR = NDIM == 3 ? 4 : 2;         // cell rows per voxel row
  constexpr int NWW = NR * 2;                   // weight words per staged sample
  constexpr int VR = 4;                         // voxel rows per CTA
  constexpr uint32_t TCOLS = VR * N < 32 ? 32 : VR * N;  // TMEM columns (a power of 2)
  constexpr uint32_t BLAYOUT = NT == 2 ? 6u : NT == 4 ? 4u : 2u;  // B swizzle: 32 / 64 / 128 B
  extern __shared__ __align__(16) unsigned char vsm[];
  const int lane = static_cast<int>(threadIdx.x & 31u);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const VoxUnit U = voxel_unit<NDIM>(p, sp);
  const int nzp = NDIM == 3 ? U.vt.nz : 1;      // voxel planes of the tile (ny * nzp = VR)
  const int D = NDIM == 3 ? p.lv.size[U.l][2] : 1;
  const int nyr = U.vt.ny + 1;
  const int ncr = (NDIM == 3 ? nzp + 1 : 1) * nyr;  // cell rows (iz, iy), iz slowest
  const uint32_t pad = ((smem_addr(vsm) + 1023u) & ~1023u) - smem_addr(vsm);
  unsigned char* base = vsm + pad;
  const VtcLayout LY = vtc_layout(NT, NDIM, sp.vcap, ncr);
  {
    // the layout inside the launch's dynamic shared memory, or no access at
    // all (checked build: bit 8 of the check word)
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if (pad + static_cast<uint32_t>(LY.end) > dyn) {
#ifdef MSDA_CHECKED
      if (threadIdx.x == 0) atomicOr(p.check_flag, 8u);
#endif
      return;
    }
  }
  const uint32_t a_a = smem_addr(base + LY.a), go_a = smem_addr(base + LY.go);
  uint32_t* wt_s = reinterpret_cast<uint32_t*>(base + LY.wt);
  int32_t* lo_s = reinterpret_cast<int32_t*>(base + LY.lo);
  uint8_t* cr_s = base + LY.cr;
  int32_t* bnd_s = reinterpret_cast<int32_t*>(base + LY.bnd);  // ncr x 2
  int32_t* off_s = bnd_s + ncr * 2;                              // ncr + 1
  uint64_t* mbar_s = reinterpret_cast<uint64_t*>(base + LY.mbar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + LY.mbar + 8 * VR);
  uint32_t* any_s = tslot + 1;                  // per voxel row: a product was issued
  uint32_t* bad_s = tslot + 2;                  // a wait ran out

  // zero A tiles; mbarriers; TMEM; each cell row's range (start of cell 0,
  // start of cell TX+1 = the row's end)
  for (int i = threadIdx.x; i < 4 * 2 * 4096 / 16; i += kThreads)
    reinterpret_cast<uint4*>(base + LY.a)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x < VR) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(mbar_s + threadIdx.x)));
    any_s[0] = 0u;
  }
  if (threadIdx.x == 0) {
    *bad_s = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tslot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int i = threadIdx.x; i < ncr * 2; i += kThreads) {
    const int cr = i >> 1, iz = cr / nyr, iy = cr - iz * nyr;
    const int32_t yc = U.y0 - 1 + iy, zc = NDIM == 3 ? U.vz - 1 + iz : -1;
    const int c = (i & 1) ? U.cw - 1 : 0;
    if (yc <= U.Hs - 1 && zc <= D - 1)
      cp_async<4>(bnd_s + i, sp.cnt + U.kb + ((zc + 1) * U.cyn + (yc + 1)) * U.cxn +
                                 min(U.x0 + c, U.cxn));
    else
      bnd_s[i] = 0;  // rows outside the level are empty
  }
  cp_async_wait_all();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  if (threadIdx.x == 0) {
    int32_t o = 0;
    for (int cr = 0; cr < ncr; ++cr) {
      off_s[cr] = o;
      o += bnd_s[2 * cr + 1] - bnd_s[2 * cr];
    }
    off_s[ncr] = o;
  }
  __syncthreads();
  const int32_t total = off_s[ncr];

  // this warp's voxel row (warps 0-3): plane pz, row ry
  const int R = warp;
  const int pz = R / U.vt.ny, ry = R - (R / U.vt.ny) * U.vt.ny;
  const bool issuer = warp < VR && U.y0 + ry < U.Hs && U.vz + pz < D;
  const int j = lane & 15, hl = lane >> 4;      // this lane's slot of a step, its weight half
  const uint32_t tile = a_a + static_cast<uint32_t>(R * 2 + hl) * 4096u;  // its A tile
  const uint32_t idesc = tc_idesc<T>(N);
  const uint32_t mbar = smem_addr(mbar_s + (R & 3));
  uint32_t phase = 0;
  bool started = false;

  for (int32_t q0 = 0; q0 < total; q0 += sp.vcap) {
    const int nr = min(sp.vcap, total - q0);
    // stage the round (every product of the previous one has completed):
    // per slot its cell row, record (into registers), corner weights as
    // 16-bit halves, x offset and grad_out row; zero rows past the end
    if (q0 > 0) __syncthreads();
    {
      uint4 r0[2], r1[2];
      int crs[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int q = threadIdx.x + i * kThreads;
        crs[i] = -1;
        if (q < nr) {
          const int32_t qq = q0 + q;
          int lo = 0, hi = ncr;  // cell row: off_s[lo] <= qq < off_s[lo + 1]
          while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (off_s[mid] <= qq) lo = mid; else hi = mid;
          }
          crs[i] = lo;
          ld_rec(sp.srec + bnd_s[2 * lo] + (qq - off_s[lo]), r0[i], r1[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (crs[i] < 0) continue;
        const int q = threadIdx.x + i * kThreads;
        const int cr = crs[i];
        const int iz = cr / nyr, iy = cr - iz * nyr;
        // the cell's x offset in the tile (cell i0x = x0 + offset - 1)
        lo_s[q] = static_cast<int32_t>(r1[i].y) -
                  (U.kb + ((U.vz + iz) * U.cyn + (U.y0 + iy)) * U.cxn) - U.x0;
        cr_s[q] = static_cast<uint8_t>((iz << 4) | iy);
        uint32_t wt[NWW];
        vm_stage_weights<T, NDIM>(r0[i], wt);
        uint4* wq = reinterpret_cast<uint4*>(wt_s + static_cast<size_t>(q) * NWW);
#pragma unroll
        for (int k = 0; k < NWW / 4; ++k)
          wq[k] = make_uint4(wt[4 * k], wt[4 * k + 1], wt[4 * k + 2], wt[4 * k + 3]);
        const char* src = reinterpret_cast<const char*>(grad_out) + static_cast<int64_t>(r1[i].x) * ROWB;
#pragma unroll
        for (int c = 0; c < NT; ++c)
          cp_async<16>(base + LY.go + static_cast<size_t>(q) * ROWB + vm_swz<NT>(c, q) * 16,
                       src + c * 16);
      }
      for (int i = threadIdx.x; i < vtc_rows_extra() * ROWB / 16; i += kThreads)
        reinterpret_cast<uint4*>(base + LY.go + static_cast<size_t>(nr) * ROWB)[i] =
            make_uint4(0u, 0u, 0u, 0u);
    }
    cp_async_wait_all();
    __syncthreads();
    if (!issuer) continue;
    // the row's two blocks of slots (3D: cell planes pz and pz+1, each the
    // cell rows ry and ry+1; 2D: one block), in this round's slots
#pragma unroll
    for (int blk = 0; blk < (NDIM == 3 ? 2 : 1); ++blk) {
      const int cr0 = (NDIM == 3 ? pz + blk : 0) * nyr + ry;
      const int32_t a = max(off_s[cr0] - q0, 0), e = min(off_s[cr0 + 2] - q0, nr);
      for (int32_t s0 = a & ~7; s0 < e; s0 += 16) {
        if (__shfl_sync(0xffffffffu, *bad_s, 0)) break;  // warp-uniform
        const int32_t q = s0 + j;
        uint32_t ta = 0, tb = 0;
        bool wl = false, wh = false;
        if (q >= a && q < e) {
          const uint32_t code = cr_s[q];
          const int dz = NDIM == 3 ? pz + 1 - static_cast<int>(code >> 4) : 0;
          const int dy = ry + 1 - static_cast<int>(code & 15u);
          const uint32_t w2 = wt_s[static_cast<size_t>(q) * NWW + (dz * 2 + dy) * 2 + hl];
          const int v = lo_s[q] - 1;  // the cell's lower-x voxel in the row
          // K-major, no swizzle: (v, k) at (v / 8) * 256 + (k / 8) * 128 + (v % 8) * 16 + (k % 8) * 2
          const uint32_t kb2 = static_cast<uint32_t>((j >> 3) * 128 + (j & 7) * 2);
          wl = static_cast<unsigned>(v) < 128u;
          wh = static_cast<unsigned>(v + 1) < 128u;
          ta = tile + static_cast<uint32_t>((v >> 3) * 256 + (v & 7) * 16) + kb2;
          tb = tile + static_cast<uint32_t>(((v + 1) >> 3) * 256 + ((v + 1) & 7) * 16) + kb2;
          if (wl) sts_u16(ta, w2);
          if (wh) sts_u16(tb, w2 >> 16);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          const uint64_t bd = tc_sdesc(go_a + static_cast<uint32_t>(s0) * ROWB, 16, 8 * ROWB, BLAYOUT);
          const uint32_t ah = a_a + static_cast<uint32_t>(R * 2) * 4096u;
          tc_mma(tmem + static_cast<uint32_t>(R * N), tc_sdesc(ah, 128, 256, 0), bd, idesc,
                 started ? 1u : 0u);
          tc_mma(tmem + static_cast<uint32_t>(R * N), tc_sdesc(ah + 4096u, 128, 256, 0), bd, idesc, 1u);
          tc_commit(mbar);
        }
        started = true;
        const bool ok = mbar_wait(mbar, phase);
        phase ^= 1u;
        if (!ok && lane == 0) {
          atomicAdd(&g_msda_tc_timeouts, 1u);
#ifdef MSDA_CHECKED
          atomicOr(p.check_flag, 0x10000u);
#endif
          *bad_s = 1u;
        }
        __syncwarp();
        if (wl) sts_u16(ta, 0u);
        if (wh) sts_u16(tb, 0u);
      }
    }
    if (lane == 0 && started) atomicOr(any_s, 1u << R);
  }
  // every issued product has completed (each step waited): read each valid
  // row's accumulators (warp w: voxels 32 (w mod 4) .., rows w / 4, + 2),
  // round once and store; rows without samples are zero
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  {
    const uint32_t anyb = *any_s;
    const bool bad = *bad_s != 0u;
    const int qd = warp & 3;
    const int v = 32 * qd + lane;
    const int64_t ks = key_stride(p);
    T* gvb = grad_value + bh_base(p, U.b, U.h, p.K);
    for (int rr = warp >> 2; rr < VR; rr += kThreads / 32 / 4) {
      const int pz2 = rr / U.vt.ny, ry2 = rr - (rr / U.vt.ny) * U.vt.ny;
      if (U.y0 + ry2 >= U.Hs || U.vz + pz2 >= D) continue;  // warp-uniform
      uint32_t r[N];
      if (((anyb >> rr) & 1u) && !bad) {
#pragma unroll
        for (int c16 = 0; c16 < N / 16; ++c16)
          tc_ld16(tmem + (static_cast<uint32_t>(qd * 32) << 16) + static_cast<uint32_t>(rr * N + c16 * 16),
                  r + 16 * c16);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      } else {
#pragma unroll
        for (int c = 0; c < N; ++c) r[c] = 0u;
      }
      const int32_t xv = U.x0 + v;
      if (v < U.vt.tx && xv < U.W) {
        const int64_t key = static_cast<int64_t>(p.lv.start[U.l]) +
                            (static_cast<int64_t>(U.vz + pz2) * U.Hs + (U.y0 + ry2)) * U.W + xv;
        uint4* dst = reinterpret_cast<uint4*>(gvb + key * ks);
#pragma unroll
        for (int c8 = 0; c8 < N / 8; ++c8) {
          const float* f = reinterpret_cast<const float*>(r + 8 * c8);
          dst[c8] = make_uint4(MmaT<T>::pack(f[0], f[1]), MmaT<T>::pack(f[2], f[3]),
                               MmaT<T>::pack(f[4], f[5]), MmaT<T>::pack(f[6], f[7]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
}

}  // namespace msda
