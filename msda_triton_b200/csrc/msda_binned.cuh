// msda_binned.cuh -- spatially binned backward.
//
// The gather/scatter backward (msda_bwd_kernel) moves 8 corner rows per
// sample through L2 twice (value gather + fp32 atomic scatter of the value
// gradient).  For large problems that traffic, not HBM, is the bound.  This
// path sorts the samples of every (batch, head, level) into spatial tiles of
// the level and lets one CTA own one tile:
//
//   * the tile's value rows plus a +1 halo are staged once in shared memory
//     (every corner of a sample whose lower corner lies in the tile is there),
//   * the tile's value gradient is accumulated in shared memory (fp32) and
//     written ONCE, in the output dtype -- no global atomics, no fp32
//     workspace, no zero-fill, no cast pass,
//   * a sample whose corners straddle into neighbouring tiles gets a
//     "secondary" record in each of them, so every corner contribution is
//     accumulated by the tile that owns that voxel; the "primary" tile (the
//     one holding its lower corner) computes the dot products and writes the
//     sample's grad_attn / grad_loc directly (one owner per sample).
//
// Coarse levels concentrate many samples in few tiles; their tiles are split
// into several work items that reduce into a compact fp32 accumulator with
// vector atomics (small: coarse levels hold few keys), rounded at the end.
//
// Binning is a counting sort: per-(b,h) chunks of queries build shared-memory
// histograms, an exclusive scan gives bucket starts, and a fill pass reserves
// ranges per chunk with one atomic per (chunk, bucket).
#pragma once

#include "msda_kernels.cuh"

namespace msda {

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 8;         // elements per thread in the scan

struct BinPlan {
  int32_t tile[3];                    // tile extent (x, y, z); z = 1 for 2D
  int32_t ntile[kMaxLevels][3];       // tiles per axis per level
  int32_t tile_base[kMaxLevels];      // first local bucket of each level
  int32_t ntl;                        // buckets per (b, h)
  int32_t atomic_mask;                // bit l: level l reduces through the fp32 accumulator
  int32_t acc_start[kMaxLevels];      // key offset of level l in the accumulator
  int64_t acc_keys;                   // keys held by the accumulator (per batch entry)
  int32_t s_max;                      // records per work item on atomic levels
  int32_t rows_per_chunk;             // queries per binning CTA
  int32_t nchunk;                     // chunks per (b, h)
  int32_t nlevels;
};

struct BinBuffers {
  int32_t* counts;       // [NB]
  int32_t* starts;       // [NB + 1] exclusive scan of counts
  int32_t* cursor;       // [NB] fill cursors
  int32_t* item_start;   // [NB + 1] exclusive scan of work items per bucket
  int32_t* item_counter; // [1]
  int32_t* scan_tmp;     // block sums
  int32_t* records;      // [max records]
  float* acc;            // fp32 accumulator for atomic levels (or grad_value for fp32)
};

// Tiles touched by one sample's valid corners along one axis.
struct AxisTiles {
  int32_t prim;   // primary tile coordinate (tile of clamp(i0))
  int32_t other;  // second tile (valid corner in the next tile) or -1
  bool any;       // at least one valid corner on this axis
};

__device__ __forceinline__ AxisTiles axis_tiles(int32_t i0, int32_t size, int32_t T) {
  AxisTiles t;
  const bool v0 = i0 >= 0 && i0 < size;
  const bool v1 = i0 + 1 >= 0 && i0 + 1 < size;
  int32_t c = i0 < 0 ? 0 : (i0 >= size ? size - 1 : i0);
  c = c < 0 ? 0 : c;
  t.prim = c / T;
  t.any = v0 || v1;
  t.other = (v0 && v1 && (i0 + 1) / T != i0 / T) ? (i0 + 1) / T : -1;
  return t;
}

// Enumerate the records of a sample: the primary bucket first, then the
// secondary ones.  Returns the count (1..8) and fills local bucket ids.
template <int NDIM>
__device__ __forceinline__ int sample_buckets(const Point<NDIM>& pt, const int32_t* sz, int l,
                                              const BinPlan& bp, int32_t* lb) {
  AxisTiles at[3];
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    if (a < NDIM) {
      at[a] = axis_tiles(pt.i0[a], sz[a], bp.tile[a]);
    } else {
      at[a].prim = 0; at[a].other = -1; at[a].any = true;
    }
  }
  const int32_t nx = bp.ntile[l][0], ny = bp.ntile[l][1];
  const int32_t base = bp.tile_base[l];
  lb[0] = base + (at[2].prim * ny + at[1].prim) * nx + at[0].prim;
  int n = 1;
  if (!(at[0].any && at[1].any && at[2].any)) return n;  // no valid corner: primary only
#pragma unroll
  for (int c = 1; c < 8; ++c) {
    const int32_t tx = (c & 1) ? at[0].other : at[0].prim;
    const int32_t ty = (c & 2) ? at[1].other : at[1].prim;
    const int32_t tz = (c & 4) ? at[2].other : at[2].prim;
    if (tx >= 0 && ty >= 0 && tz >= 0) lb[n++] = base + (tz * ny + ty) * nx + tx;
  }
  return n;
}

// ---------------------------------------------------------------- binning
// Record encoding: (q << 5) | (p << 1) | secondary  (P <= 16, Q < 2^26).
__device__ __forceinline__ int32_t make_record(int32_t q, int pp, bool secondary) {
  return (q << 5) | (pp << 1) | (secondary ? 1 : 0);
}

// One CTA per (b, h, chunk of queries).  Each thread keeps one (level, point)
// index for the whole chunk and strides over the chunk's queries, so there is
// no per-sample division.  FILL = false counts records per bucket; FILL = true
// places them.
template <typename TS, int NDIM, bool FILL>
__global__ void __launch_bounds__(512)
    msda_bin_kernel(const Problem p, const BinPlan bp, BinBuffers bb) {
  extern __shared__ int32_t s_hist[];        // [ntl] counts, then [ntl] bases (fill)
  __shared__ LevelSmem lv;
  load_levels(p, lv, NDIM);
  const int ntl = bp.ntl;
  for (int i = threadIdx.x; i < ntl; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();

  const int64_t chunk = blockIdx.x % bp.nchunk;
  const int64_t bh = blockIdx.x / bp.nchunk;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int32_t q0 = static_cast<int32_t>(chunk * bp.rows_per_chunk);
  const int32_t q1 = min(static_cast<int32_t>(p.Q), q0 + bp.rows_per_chunk);
  const int LP = static_cast<int>(p.L * p.P);
  const int per_row = static_cast<int>(blockDim.x) / LP;   // host guarantees >= 1
  const int lp = static_cast<int>(threadIdx.x) % LP;
  const int roff = static_cast<int>(threadIdx.x) / LP;
  const bool worker = roff < per_row;
  const int l = lp / static_cast<int>(p.P);
  const int pp = lp - l * static_cast<int>(p.P);
  const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
  const TS* loc = static_cast<const TS*>(p.loc);
  const int64_t row0 = (b * p.Q) * p.H + h;   // row of query 0 of this (b, h)

  if (worker) {
    for (int32_t q = q0 + roff; q < q1; q += per_row) {
      const int64_t s = (row0 + static_cast<int64_t>(q) * p.H) * LP + lp;
      const Point<NDIM> pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
      int32_t lb[8];
      const int n = sample_buckets<NDIM>(pt, sz, l, bp, lb);
      for (int k = 0; k < n; ++k) atomicAdd(&s_hist[lb[k]], 1);
    }
  }
  __syncthreads();
  const int64_t gbase = bh * ntl;
  if (!FILL) {
    for (int i = threadIdx.x; i < ntl; i += blockDim.x)
      if (s_hist[i]) atomicAdd(&bb.counts[gbase + i], s_hist[i]);
    return;
  }
  // Fill: reserve one range per non-empty bucket, then place records.
  int32_t* s_base = s_hist + ntl;
  for (int i = threadIdx.x; i < ntl; i += blockDim.x) {
    const int32_t c = s_hist[i];
    s_base[i] = c ? atomicAdd(&bb.cursor[gbase + i], c) : 0;
    s_hist[i] = 0;
  }
  __syncthreads();
  if (worker) {
    for (int32_t q = q0 + roff; q < q1; q += per_row) {
      const int64_t s = (row0 + static_cast<int64_t>(q) * p.H) * LP + lp;
      const Point<NDIM> pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
      int32_t lb[8];
      const int n = sample_buckets<NDIM>(pt, sz, l, bp, lb);
      for (int k = 0; k < n; ++k) {
        const int32_t pos = s_base[lb[k]] + atomicAdd(&s_hist[lb[k]], 1);
        bb.records[pos] = make_record(q, pp, k > 0);
      }
    }
  }
}

// ---------------------------------------------------------------- scan
// Exclusive scan of n int32 (in place allowed: in != out is not required),
// out[n] = total.  Three kernels: block sums, scan of block sums (one CTA),
// block-local scan plus offset.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t* s_warp,
                                                        int32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int32_t w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s_warp[lane] = w;
  }
  __syncthreads();
  total = s_warp[(blockDim.x >> 5) - 1];
  const int32_t before = warp ? s_warp[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_reduce_kernel(const int32_t* __restrict__ in, int64_t n, int32_t* __restrict__ sums) {
  __shared__ int32_t s_warp[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * kScanItems;
  int32_t v = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
    if (i < n) v += in[i];
  }
  int32_t total;
  block_exclusive_scan(v, s_warp, total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_top_kernel(int32_t* __restrict__ sums, int64_t nblocks) {
  __shared__ int32_t s_warp[32];
  int32_t carry = 0;
  for (int64_t base = 0; base < nblocks; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const int32_t v = i < nblocks ? sums[i] : 0;
    int32_t total;
    const int32_t ex = block_exclusive_scan(v, s_warp, total);
    if (i < nblocks) sums[i] = carry + ex;
    carry += total;
  }
}

static __global__ void __launch_bounds__(kScanThreads)
    msda_scan_apply_kernel(const int32_t* __restrict__ in, int64_t n,
                           const int32_t* __restrict__ sums, int32_t* __restrict__ out,
                           int32_t* __restrict__ out2) {
  __shared__ int32_t s_warp[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanThreads * kScanItems;
  int32_t vals[kScanItems];
  int32_t v = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
    vals[k] = i < n ? in[i] : 0;
    v += vals[k];
  }
  int32_t total;
  int32_t run = block_exclusive_scan(v, s_warp, total) + sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
    if (i < n) {
      out[i] = run;
      if (out2) out2[i] = run;
    }
    if (i == n - 1) {
      out[n] = run + vals[k];
    }
    run += vals[k];
  }
}

// Work items per bucket: direct levels get exactly one item per tile (even an
// empty tile must write its zero gradient); atomic levels one item per s_max
// records (none when empty).
static __global__ void msda_items_kernel(const int32_t* __restrict__ counts, int64_t nb,
                                  const BinPlan bp, int32_t* __restrict__ items) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nb) return;
  const int32_t lb = static_cast<int32_t>(i % bp.ntl);
  int l = 0;
  while (l + 1 < bp.nlevels && lb >= bp.tile_base[l + 1]) ++l;
  const bool atomic_level = (bp.atomic_mask >> l) & 1;
  items[i] = atomic_level ? (counts[i] + bp.s_max - 1) / bp.s_max : 1;
}

// ---------------------------------------------------------------- main kernel
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int src_size = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem),
               "r"(src_size)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Rotate an array of N floats left by r (0 <= r < N, N a power of two) with
// a fixed network of selects (no dynamic register indexing).
template <int N>
__device__ __forceinline__ void rotate_left(float* x, int r) {
#pragma unroll
  for (int k = 1; k < N; k <<= 1) {
    if (r & k) {
      float t[N];
#pragma unroll
      for (int i = 0; i < N; ++i) t[i] = x[(i + k) & (N - 1)];
#pragma unroll
      for (int i = 0; i < N; ++i) x[i] = t[i];
    }
  }
}

// Dot product of EPV channels held as raw 16-byte chunks (8 x 16-bit or 4 x
// fp32), fp32 accumulation.  16-bit inputs use sm_100's mixed-precision FMA
// (fp16/bf16 multiplicands, fp32 addend) so no conversion is issued.
template <typename T>
__device__ __forceinline__ float chunk_dot(const uint4& x, const uint4& y, float acc);
template <>
__device__ __forceinline__ float chunk_dot<float>(const uint4& x, const uint4& y, float acc) {
  acc = fmaf(__uint_as_float(x.x), __uint_as_float(y.x), acc);
  acc = fmaf(__uint_as_float(x.y), __uint_as_float(y.y), acc);
  acc = fmaf(__uint_as_float(x.z), __uint_as_float(y.z), acc);
  acc = fmaf(__uint_as_float(x.w), __uint_as_float(y.w), acc);
  return acc;
}
#define MSDA_MIXED_FMA(TYPE)                                                              \
  __device__ __forceinline__ float mixed_fma_##TYPE(uint32_t a, uint32_t b, float acc) {  \
    uint16_t al, ah, bl, bh;                                                              \
    asm("mov.b32 {%0, %1}, %2;" : "=h"(al), "=h"(ah) : "r"(a));                          \
    asm("mov.b32 {%0, %1}, %2;" : "=h"(bl), "=h"(bh) : "r"(b));                          \
    asm("fma.rn.f32." #TYPE " %0, %1, %2, %0;" : "+f"(acc) : "h"(al), "h"(bl));          \
    asm("fma.rn.f32." #TYPE " %0, %1, %2, %0;" : "+f"(acc) : "h"(ah), "h"(bh));          \
    return acc;                                                                           \
  }
MSDA_MIXED_FMA(bf16)
MSDA_MIXED_FMA(f16)
#undef MSDA_MIXED_FMA
template <>
__device__ __forceinline__ float chunk_dot<__nv_bfloat16>(const uint4& x, const uint4& y,
                                                           float acc) {
  acc = mixed_fma_bf16(x.x, y.x, acc);
  acc = mixed_fma_bf16(x.y, y.y, acc);
  acc = mixed_fma_bf16(x.z, y.z, acc);
  acc = mixed_fma_bf16(x.w, y.w, acc);
  return acc;
}
template <>
__device__ __forceinline__ float chunk_dot<__half>(const uint4& x, const uint4& y, float acc) {
  acc = mixed_fma_f16(x.x, y.x, acc);
  acc = mixed_fma_f16(x.y, y.y, acc);
  acc = mixed_fma_f16(x.z, y.z, acc);
  acc = mixed_fma_f16(x.w, y.w, acc);
  return acc;
}

constexpr int kTileThreads = 256;
constexpr int kTileCtasPerSm = 3;
#ifndef MSDA_MIXED_PRECISION_DOT
#define MSDA_MIXED_PRECISION_DOT 0
#endif

// Shared-memory fp32 reduction without a return value.
__device__ __forceinline__ void red_shared_f32(float* addr, float v) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(addr));
  asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// Work item: one tile of one (b, h, level), records [r0, r1).  C * sizeof(T)
// is a multiple of 16 and at most 512 bytes: G lanes per record own one
// 16-byte chunk (EPV channels) each.
//
// Per record: corner weights from the sample's location; for a primary
// record the dot products of grad_out with the staged corner rows give
// grad_attn and grad_loc (written directly, one owner per sample); for every
// corner inside the tile, a*w*grad_out is added to the tile's fp32 gradient
// with shared-memory atomics.  Lanes of different record slots add their
// elements in a rotated order so a warp's 32 atomics hit 32 banks.  At the end
// of the item the tile gradient is written once (direct levels) or reduced
// into the fp32 accumulator (atomic levels).
template <typename T, typename TS, int NDIM>
__global__ void __launch_bounds__(kTileThreads, kTileCtasPerSm)
    msda_bwd_binned_kernel(const Problem p, const BinPlan bp, const BinBuffers bb,
                           const T* __restrict__ grad_out, T* __restrict__ grad_value,
                           TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  using CK = Chunk<T, 16>;
  constexpr int EPV = CK::EPV;      // channels per 16-byte chunk (8 or 4)
  constexpr int NC = 1 << NDIM;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ LevelSmem lv;
  __shared__ int32_t s_item[2];
  load_levels(p, lv, NDIM);

  const int TX = bp.tile[0], TY = bp.tile[1], TZ = bp.tile[2];
  const int HX = TX + 1, HY = TY + 1, HZ = (NDIM == 3) ? TZ + 1 : 1;
  const int nhalo = HX * HY * HZ;
  const int V = TX * TY * TZ;
  const int C = static_cast<int>(p.C);
  const int row_bytes = C * static_cast<int>(sizeof(T));
  unsigned char* s_val = smem;                                               // nhalo + 1 rows
  float* s_grad = reinterpret_cast<float*>(smem + (nhalo + 1) * row_bytes);  // V x C

  const int G = 1 << p.log2g;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int slot = lane / G;
  const int j = lane & (G - 1);
  const int spw = 32 / G;                              // record slots per warp
  const int stride = (kTileThreads / 32) * spw;        // records per CTA pass
  const bool has = j < p.nv;
  const int rot = slot & (EPV - 1);
  const int LP = static_cast<int>(p.L * p.P);
  const int P = static_cast<int>(p.P);
  const int64_t NB = p.B * p.H * bp.ntl;
  const TS* loc = static_cast<const TS*>(p.loc);
  const TS* attn = static_cast<const TS*>(p.attn);
  // Element e of this lane's chunk goes to channel j*EPV + ((e + rot) & (EPV-1)).
  int eoff[EPV];
#pragma unroll
  for (int e = 0; e < EPV; ++e) eoff[e] = j * EPV + ((e + rot) & (EPV - 1));

  // The zero row after the halo: corners outside the level read it.
  for (int i = threadIdx.x; i < row_bytes / 16; i += kTileThreads)
    reinterpret_cast<uint4*>(s_val + nhalo * row_bytes)[i] = make_uint4(0, 0, 0, 0);

  for (;;) {
    if (threadIdx.x == 0) {
      const int32_t item = atomicAdd(bb.item_counter, 1);
      int32_t bucket = -1;
      if (item < bb.item_start[NB]) {
        int64_t lo = 0, hi = NB;  // last bucket with item_start <= item
        while (hi - lo > 1) {
          const int64_t mid = (lo + hi) >> 1;
          if (bb.item_start[mid] <= item) lo = mid; else hi = mid;
        }
        bucket = static_cast<int32_t>(lo);
      }
      s_item[0] = item;
      s_item[1] = bucket;
    }
    __syncthreads();
    const int32_t item = s_item[0];
    const int32_t bucket = s_item[1];
    if (bucket < 0) break;

    const int64_t bh = bucket / bp.ntl;
    const int32_t lb = static_cast<int32_t>(bucket - bh * bp.ntl);
    const int64_t b = bh / p.H, h = bh % p.H;
    int l = 0;
    while (l + 1 < p.L && lb >= bp.tile_base[l + 1]) ++l;
    const int32_t t = lb - bp.tile_base[l];
    const int32_t nx = bp.ntile[l][0], ny = bp.ntile[l][1];
    const int32_t org[3] = {(t % nx) * TX, ((t / nx) % ny) * TY, (t / (nx * ny)) * TZ};
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int32_t start = lv.start[l];
    const bool atomic_level = (bp.atomic_mask >> l) & 1;
    int32_t r0 = bb.starts[bucket];
    int32_t r1 = bb.starts[bucket + 1];
    if (atomic_level) {
      r0 += (item - bb.item_start[bucket]) * bp.s_max;
      r1 = min(r1, r0 + bp.s_max);
    }

    // Stage the value tile + halo (zero outside the level); clear the grads.
    const int cpr = row_bytes / 16;
    const char* vsrc = static_cast<const char*>(p.value) + (b * p.K * p.H + h) * row_bytes;
    for (int i = threadIdx.x; i < nhalo * cpr; i += kTileThreads) {
      const int r = i / cpr, c = i - r * cpr;
      const int hx = r % HX, hy = (r / HX) % HY, hz = r / (HX * HY);
      const int32_t x = org[0] + hx, y = org[1] + hy, z = org[2] + hz;
      const bool in = x < sz[0] && y < sz[1] && z < sz[2];
      const int64_t key = in ? start + (static_cast<int64_t>(z) * sz[1] + y) * sz[0] + x : start;
      cp_async16(s_val + r * row_bytes + c * 16, vsrc + key * p.H * row_bytes + c * 16, in);
    }
    for (int i = threadIdx.x; i < V * C / 4; i += kTileThreads)
      reinterpret_cast<float4*>(s_grad)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    cp_async_wait_all();
    __syncthreads();

    const int64_t row_b = b * p.Q * p.H + h;   // row of query 0
    for (int32_t rb = r0 + warp * spw; rb < r1; rb += stride) {
      const int32_t ri = rb + slot;
      const bool active = ri < r1;
      const int32_t rec = active ? __ldg(bb.records + ri) : 0;
      const bool secondary = rec & 1;
      const int32_t q = rec >> 5;
      const int pp = (rec >> 1) & 15;
      const int64_t row = row_b + static_cast<int64_t>(q) * p.H;
      const int64_t s = row * LP + l * P + pp;

      Point<NDIM> pt;
      float a = 0.0f;
      uint4 gor = make_uint4(0, 0, 0, 0);
      if (active) {
        pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
        a = Elem<TS>::to_f(attn[s]);
        if (has) gor = __ldg(reinterpret_cast<const uint4*>(
                              reinterpret_cast<const char*>(grad_out) + row * row_bytes + j * 16));
      } else {
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) { pt.i0[ax] = -2; pt.f[ax] = 0.0f; pt.pass[ax] = false; }
      }
      // grad_out in fp32 (dots) and a * grad_out rotated into this slot's
      // accumulation order (value-gradient contributions).
      float gof[EPV], ga[EPV];
      {
        Raw<16> rg;
        rg.w[0] = gor.x; rg.w[1] = gor.y; rg.w[2] = gor.z; rg.w[3] = gor.w;
        CK::unpack(rg, gof);
#pragma unroll
        for (int e = 0; e < EPV; ++e) ga[e] = a * gof[e];
        rotate_left<EPV>(ga, rot);
      }
      // Per-axis: validity in the level, ownership by the tile, weights.
      bool vv[3][2], ow[3][2];
      float wt[3][2];
      int32_t lo[3];
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        if (ax < NDIM) {
          const int32_t i0 = pt.i0[ax];
          const int32_t T_ = ax == 0 ? TX : (ax == 1 ? TY : TZ);
          lo[ax] = i0 - org[ax];
          vv[ax][0] = static_cast<uint32_t>(i0) < static_cast<uint32_t>(sz[ax]);
          vv[ax][1] = static_cast<uint32_t>(i0 + 1) < static_cast<uint32_t>(sz[ax]);
          ow[ax][0] = static_cast<uint32_t>(lo[ax]) < static_cast<uint32_t>(T_);
          ow[ax][1] = static_cast<uint32_t>(lo[ax] + 1) < static_cast<uint32_t>(T_);
          wt[ax][0] = __fsub_rn(1.0f, pt.f[ax]);
          wt[ax][1] = pt.f[ax];
        } else {
          lo[ax] = 0;
          vv[ax][0] = true; vv[ax][1] = false;
          ow[ax][0] = true; ow[ax][1] = false;
          wt[ax][0] = 1.0f; wt[ax][1] = 0.0f;
        }
      }
      const int hbase = (lo[2] * HY + lo[1]) * HX + lo[0];
      const int tbase = (lo[2] * TY + lo[1]) * TX + lo[0];
      float dots[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int bx = c & 1, by = (c >> 1) & 1, bz = (c >> 2) & 1;
        const bool valid = vv[0][bx] && vv[1][by] && vv[2][bz];
        float w = __fmul_rn(wt[0][bx], wt[1][by]);
        if (NDIM == 3) w = __fmul_rn(w, wt[2][bz]);
        w = valid ? w : 0.0f;
        dots[c] = 0.0f;
        if (!secondary) {
          // All valid corners of a primary record lie in the tile + halo.
          const int hidx = valid ? hbase + bx + by * HX + bz * HX * HY : nhalo;
          const uint4 xv = *reinterpret_cast<const uint4*>(s_val + hidx * row_bytes + j * 16);
#if MSDA_MIXED_PRECISION_DOT
          dots[c] = chunk_dot<T>(gor, xv, 0.0f);
#else
          Raw<16> rv;
          rv.w[0] = xv.x; rv.w[1] = xv.y; rv.w[2] = xv.z; rv.w[3] = xv.w;
          float xf[EPV];
          CK::unpack(rv, xf);
          float d = 0.0f;
#pragma unroll
          for (int e = 0; e < EPV; ++e) d = fmaf(gof[e], xf[e], d);
          dots[c] = d;
#endif
        }
        if (valid && ow[0][bx] && ow[1][by] && ow[2][bz] && has) {
          float* gr = s_grad + (tbase + bx + by * TX + bz * TX * TY) * C;
#pragma unroll
          for (int e = 0; e < EPV; ++e) red_shared_f32(gr + eoff[e], w * ga[e]);
        }
      }
      // Per-sample scalars (d out / d attn, d out / d source index).
      float g_attn = 0.0f, g_ix[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int bx = c & 1, by = (c >> 1) & 1, bz = (c >> 2) & 1;
        const float wyz = (NDIM == 3) ? wt[1][by] * wt[2][bz] : wt[1][by];
        const float wxz = (NDIM == 3) ? wt[0][bx] * wt[2][bz] : wt[0][bx];
        const float d = dots[c];
        g_attn = fmaf(wt[0][bx] * wyz, d, g_attn);
        g_ix[0] = fmaf(bx ? wyz : -wyz, d, g_ix[0]);
        g_ix[1] = fmaf(by ? wxz : -wxz, d, g_ix[1]);
        if (NDIM == 3) {
          const float wxy = wt[0][bx] * wt[1][by];
          g_ix[2] = fmaf(bz ? wxy : -wxy, d, g_ix[2]);
        }
      }
      for (int o = G >> 1; o > 0; o >>= 1) {
        g_attn += __shfl_xor_sync(0xffffffffu, g_attn, o);
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) g_ix[ax] += __shfl_xor_sync(0xffffffffu, g_ix[ax], o);
      }
      if (active && !secondary && j == 0) {
        grad_attn[s] = Elem<TS>::from_f(g_attn);
        TS* gl = grad_loc + s * NDIM;
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) {
          const float gval = a * g_ix[ax] * static_cast<float>(sz[ax]);
          gl[ax] = Elem<TS>::from_f(pt.pass[ax] ? gval : 0.0f);
        }
      }
    }
    __syncthreads();

    // Flush: one write per gradient element (direct levels) or one vector
    // reduction into the fp32 accumulator (atomic levels).
    for (int i = threadIdx.x; i < V * (C / EPV); i += kTileThreads) {
      const int v = i / (C / EPV);
      const int ck = i - v * (C / EPV);
      const int lx = v % TX, ly = (v / TX) % TY, lz = v / (TX * TY);
      const int32_t x = org[0] + lx, y = org[1] + ly, z = org[2] + lz;
      if (x >= sz[0] || y >= sz[1] || z >= sz[2]) continue;
      const float* src = s_grad + v * C + ck * EPV;
      float f[EPV];
#pragma unroll
      for (int e = 0; e < EPV; e += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(src + e);
        f[e] = t4.x; f[e + 1] = t4.y; f[e + 2] = t4.z; f[e + 3] = t4.w;
      }
      const int64_t kil = (static_cast<int64_t>(z) * sz[1] + y) * sz[0] + x;
      if (atomic_level) {
        float* dst = bb.acc + ((b * bp.acc_keys + bp.acc_start[l] + kil) * p.H + h) * C + ck * EPV;
        red_add_f32<EPV>(dst, f);
      } else {
        char* dst = reinterpret_cast<char*>(grad_value) +
                    ((b * p.K + start + kil) * p.H + h) * static_cast<int64_t>(row_bytes) + ck * 16;
        st_chunk<16>(dst, CK::pack(f));
      }
    }
    __syncthreads();
  }
}

// Round the fp32 accumulator of the atomic levels into grad_value.
template <typename T>
__global__ void __launch_bounds__(256)
    msda_acc_cast_kernel(const Problem p, const BinPlan bp, const float* __restrict__ acc,
                         T* __restrict__ grad_value) {
  __shared__ LevelSmem lv;
  load_levels(p, lv, 3);  // host-resolved table: ndim only matters for device shapes
  const int64_t per_key = p.H * p.C;
  const int64_t n = p.B * bp.acc_keys * per_key;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t rem = i % per_key;
    const int64_t ak = (i / per_key) % bp.acc_keys;
    const int64_t b = i / (per_key * bp.acc_keys);
    int l = 0;
    for (int k = 0; k < p.L; ++k)
      if (((bp.atomic_mask >> k) & 1) && ak >= bp.acc_start[k]) l = k;
    const int64_t key = lv.start[l] + (ak - bp.acc_start[l]);
    grad_value[(b * p.K + key) * per_key + rem] = Elem<T>::from_f(acc[i]);
  }
}

}  // namespace msda
