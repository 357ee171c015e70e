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
// One CTA per (b, h, chunk of queries).  Pass 0 counts, pass 1 fills.
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
  const int64_t q0 = chunk * bp.rows_per_chunk;
  int64_t q1 = q0 + bp.rows_per_chunk;
  if (q1 > p.Q) q1 = p.Q;
  const int LP = static_cast<int>(p.L * p.P);
  const int64_t nsmp = (q1 - q0) * LP;
  const TS* loc = static_cast<const TS*>(p.loc);

  // Pass A: local histogram.
  for (int64_t i = threadIdx.x; i < nsmp; i += blockDim.x) {
    const int64_t q = q0 + i / LP;
    const int lp = static_cast<int>(i % LP);
    const int l = lp / static_cast<int>(p.P);
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int64_t s = ((b * p.Q + q) * p.H + h) * LP + lp;
    const Point<NDIM> pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
    int32_t lb[8];
    const int n = sample_buckets<NDIM>(pt, sz, l, bp, lb);
    for (int k = 0; k < n; ++k) atomicAdd(&s_hist[lb[k]], 1);
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
  for (int64_t i = threadIdx.x; i < nsmp; i += blockDim.x) {
    const int64_t q = q0 + i / LP;
    const int lp = static_cast<int>(i % LP);
    const int l = lp / static_cast<int>(p.P);
    const int pp = lp - l * static_cast<int>(p.P);
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int64_t s = ((b * p.Q + q) * p.H + h) * LP + lp;
    const Point<NDIM> pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
    int32_t lb[8];
    const int n = sample_buckets<NDIM>(pt, sz, l, bp, lb);
    const int32_t rec = static_cast<int32_t>((q * p.P + pp) << 1);
    for (int k = 0; k < n; ++k) {
      const int32_t pos = s_base[lb[k]] + atomicAdd(&s_hist[lb[k]], 1);
      bb.records[pos] = rec | (k > 0 ? 1 : 0);
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

// Work item: one tile of one (b, h, level), records [r0, r1).  VB = 16 only
// (C * sizeof(T) % 16 == 0, C % 8 == 0).
//
// Records are processed in chunks of R = kTileThreads / G (G lanes per record,
// each owning EPV channels):
//   A. per record: corner weights, dot products against the staged value rows
//      (primary records: write grad_attn / grad_loc), stage a*grad_out in
//      shared memory, and emit one (voxel, weight) pair per corner the tile
//      owns, counting pairs per voxel with an integer shared-memory atomic;
//   B. exclusive scan of the per-voxel counts;
//   C. scatter the pairs into voxel order;
//   D. every thread owns fixed (voxel, 8-channel) units and adds
//      w * a*grad_out for the voxel's pairs into registers.
// The value gradient of the tile is never touched by an atomic: it lives in
// the owners' registers until the item ends and is written once.
constexpr int kTileThreads = 256;
constexpr int kMaxUnitsPerThread = 8;

template <typename T, typename TS, int NDIM>
__global__ void __launch_bounds__(kTileThreads, 2)
    msda_bwd_binned_kernel(const Problem p, const BinPlan bp, const BinBuffers bb,
                           const T* __restrict__ grad_out, T* __restrict__ grad_value,
                           TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  using CK = Chunk<T, 16>;
  constexpr int EPV = CK::EPV;      // channels per 16-byte chunk
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
  const int NU = C / 8;                       // 8-channel units per voxel
  const int64_t row_bytes = static_cast<int64_t>(C) * sizeof(T);
  const int G = 1 << p.log2g;
  const int R = kTileThreads / G;             // records per chunk
  // Shared memory carve-up (byte offsets are multiples of 16).
  unsigned char* s_val = smem;                                                // nhalo rows
  float* s_go = reinterpret_cast<float*>(smem + nhalo * row_bytes);           // R x C
  int32_t* s_pvr = reinterpret_cast<int32_t*>(s_go + R * C);                  // R*8: voxel | rank<<10
  float* s_pw = reinterpret_cast<float*>(s_pvr + R * 8);                      // R*8: weight
  int2* s_sorted = reinterpret_cast<int2*>(s_pw + R * 8);                     // R*8: (slot, w)
  int32_t* s_cnt = reinterpret_cast<int32_t*>(s_sorted + R * 8);              // V
  int32_t* s_off = s_cnt + V;                                                 // V + 1
  __shared__ int32_t s_warp[32];

  const int slot = threadIdx.x / G;           // record slot within the chunk
  const int j = threadIdx.x & (G - 1);        // channel chunk of this lane
  const bool has = j < p.nv;
  const int LP = static_cast<int>(p.L * p.P);
  const int64_t NB = p.B * p.H * bp.ntl;
  const TS* loc = static_cast<const TS*>(p.loc);
  const TS* attn = static_cast<const TS*>(p.attn);
  const int nunits = V * NU;
  const int upt = (nunits + kTileThreads - 1) / kTileThreads;

  for (int i = threadIdx.x; i < V; i += kTileThreads) s_cnt[i] = 0;

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
    const int32_t ox = (t % nx) * TX, oy = ((t / nx) % ny) * TY, oz = (t / (nx * ny)) * TZ;
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int32_t start = lv.start[l];
    const bool atomic_level = (bp.atomic_mask >> l) & 1;
    int32_t r0 = bb.starts[bucket];
    int32_t r1 = bb.starts[bucket + 1];
    if (atomic_level) {
      r0 += (item - bb.item_start[bucket]) * bp.s_max;
      r1 = min(r1, r0 + bp.s_max);
    }

    // Stage the value tile + halo (zero outside the level).
    const int cpr = static_cast<int>(row_bytes / 16);
    const char* vsrc = static_cast<const char*>(p.value) + (b * p.K * p.H + h) * row_bytes;
    for (int i = threadIdx.x; i < nhalo * cpr; i += kTileThreads) {
      const int r = i / cpr, c = i - r * cpr;
      const int hx = r % HX, hy = (r / HX) % HY, hz = r / (HX * HY);
      const int32_t x = ox + hx, y = oy + hy, z = oz + hz;
      const bool in = x < sz[0] && y < sz[1] && z < sz[2];
      const int64_t key = in ? start + (static_cast<int64_t>(z) * sz[1] + y) * sz[0] + x : start;
      cp_async16(s_val + r * row_bytes + c * 16, vsrc + key * p.H * row_bytes + c * 16, in);
    }
    float acc[kMaxUnitsPerThread][8];
#pragma unroll
    for (int k = 0; k < kMaxUnitsPerThread; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[k][e] = 0.0f;
    cp_async_wait_all();
    __syncthreads();

    for (int32_t c0 = r0; c0 < r1; c0 += R) {
      // ---- A: records -> dots, staged a*grad_out, owned-corner pairs
      const int32_t ri = c0 + slot;
      const bool active = ri < r1;
      const int32_t rec = active ? bb.records[ri] : 0;
      const bool secondary = rec & 1;
      const int32_t qp = rec >> 1;
      const int32_t q = qp / static_cast<int32_t>(p.P);
      const int pp = qp - q * static_cast<int32_t>(p.P);
      const int64_t row = (b * p.Q + q) * p.H + h;
      const int64_t s = row * LP + l * static_cast<int>(p.P) + pp;
      Point<NDIM> pt;
      float a = 0.0f;
      if (active) {
        pt = load_point<TS, NDIM>(loc + s * NDIM, sz, p);
        a = Elem<TS>::to_f(attn[s]);
      } else {
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) { pt.i0[ax] = -2; pt.f[ax] = 0.0f; pt.pass[ax] = false; }
      }
      float go[EPV];
      {
        const Raw<16> rg = (active && has)
            ? ld_chunk<16>(reinterpret_cast<const char*>(grad_out) + row * row_bytes + j * 16)
            : raw_zero<16>();
        CK::unpack(rg, go);
      }
      if (has) {
        float4* dst = reinterpret_cast<float4*>(s_go + slot * C + j * EPV);
#pragma unroll
        for (int e = 0; e < EPV; e += 4)
          dst[e / 4] = make_float4(a * go[e], a * go[e + 1], a * go[e + 2], a * go[e + 3]);
      }
      // Per-axis corner data.
      int32_t lo[3];
      bool v0[3], v1[3];
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        const int32_t o = ax == 0 ? ox : (ax == 1 ? oy : oz);
        lo[ax] = pt.i0[ax] - o;
        v0[ax] = pt.i0[ax] >= 0 && pt.i0[ax] < sz[ax];
        v1[ax] = pt.i0[ax] + 1 >= 0 && pt.i0[ax] + 1 < sz[ax];
      }
      if (NDIM == 2) { lo[2] = 0; v0[2] = true; v1[2] = false; }
      float g_attn = 0.0f;
      float g_ix[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int bx = c & 1, by = (c >> 1) & 1, bz = (c >> 2) & 1;
        const bool valid = (bx ? v1[0] : v0[0]) && (by ? v1[1] : v0[1]) && (bz ? v1[2] : v0[2]);
        const int32_t lx = lo[0] + bx, ly = lo[1] + by, lz = lo[2] + bz;
        const float wx = bx ? pt.f[0] : 1.0f - pt.f[0];
        const float wy = by ? pt.f[1] : 1.0f - pt.f[1];
        const float wz = (NDIM == 3) ? (bz ? pt.f[2] : 1.0f - pt.f[2]) : 1.0f;
        const float w = wx * wy * wz;
        if (!secondary) {
          float dot = 0.0f;
          if (valid && has && lx >= 0 && lx <= TX && ly >= 0 && ly <= TY && lz >= 0 && lz < HZ) {
            Raw<16> rv;
            const uint4 u = *reinterpret_cast<const uint4*>(
                s_val + ((lz * HY + ly) * HX + lx) * row_bytes + j * 16);
            rv.w[0] = u.x; rv.w[1] = u.y; rv.w[2] = u.z; rv.w[3] = u.w;
            float x[EPV];
            CK::unpack(rv, x);
#pragma unroll
            for (int e = 0; e < EPV; ++e) dot = fmaf(go[e], x[e], dot);
          }
          g_attn = fmaf(w, dot, g_attn);
          const float sx = bx ? 1.0f : -1.0f, sy = by ? 1.0f : -1.0f, sz_ = bz ? 1.0f : -1.0f;
          g_ix[0] = fmaf(sx * wy * wz, dot, g_ix[0]);
          g_ix[1] = fmaf(sy * wx * wz, dot, g_ix[1]);
          if (NDIM == 3) g_ix[2] = fmaf(sz_ * wx * wy, dot, g_ix[2]);
        }
        // Corner c's pair is emitted by lane (c mod G) of the record.
        if ((c & (G - 1)) == j) {
          const bool owned = active && valid && lx >= 0 && lx < TX && ly >= 0 && ly < TY &&
                             lz >= 0 && lz < TZ;
          int32_t pv = -1;
          if (owned) {
            const int vox = (lz * TY + ly) * TX + lx;
            const int rank = atomicAdd(&s_cnt[vox], 1);
            pv = vox | (rank << 10);
          }
          s_pvr[slot * 8 + c] = pv;
          s_pw[slot * 8 + c] = w;
        }
      }
      if (NC == 4 && j == 0) {  // 2D: the unused pair slots
#pragma unroll
        for (int c = 4; c < 8; ++c) s_pvr[slot * 8 + c] = -1;
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
      __syncthreads();
      // ---- B: exclusive scan of the per-voxel pair counts
      for (int base = 0; base < V; base += kTileThreads) {
        const int i = base + threadIdx.x;
        const int32_t cnt = i < V ? s_cnt[i] : 0;
        int32_t total;
        const int32_t ex = block_exclusive_scan(cnt, s_warp, total);
        const int32_t carry = base ? s_off[base] : 0;
        if (i < V) {
          s_off[i] = carry + ex;
          s_cnt[i] = 0;
        }
        __syncthreads();
        if (threadIdx.x == 0) s_off[min(base + kTileThreads, V)] = carry + total;
        __syncthreads();
      }
      // ---- C: pairs into voxel order
      for (int i = threadIdx.x; i < R * 8; i += kTileThreads) {
        const int32_t pv = s_pvr[i];
        if (pv >= 0) s_sorted[s_off[pv & 1023] + (pv >> 10)] = make_int2(i >> 3, __float_as_int(s_pw[i]));
      }
      __syncthreads();
      // ---- D: owners accumulate in registers
#pragma unroll
      for (int k = 0; k < kMaxUnitsPerThread; ++k) {
        if (k < upt) {
          const int u = threadIdx.x + k * kTileThreads;
          if (u < nunits) {
            const int vox = u / NU, g8 = u - vox * NU;
            const int32_t e0 = s_off[vox], e1 = s_off[vox + 1];
            for (int32_t e = e0; e < e1; ++e) {
              const int2 sp = s_sorted[e];
              const float w = __int_as_float(sp.y);
              const float4* src = reinterpret_cast<const float4*>(s_go + sp.x * C + g8 * 8);
              const float4 lo4 = src[0], hi4 = src[1];
              acc[k][0] = fmaf(w, lo4.x, acc[k][0]);
              acc[k][1] = fmaf(w, lo4.y, acc[k][1]);
              acc[k][2] = fmaf(w, lo4.z, acc[k][2]);
              acc[k][3] = fmaf(w, lo4.w, acc[k][3]);
              acc[k][4] = fmaf(w, hi4.x, acc[k][4]);
              acc[k][5] = fmaf(w, hi4.y, acc[k][5]);
              acc[k][6] = fmaf(w, hi4.z, acc[k][6]);
              acc[k][7] = fmaf(w, hi4.w, acc[k][7]);
            }
          }
        }
      }
      __syncthreads();
    }

    // Flush the owned units: one write per gradient element (direct levels)
    // or one vector reduction into the fp32 accumulator (atomic levels).
#pragma unroll
    for (int k = 0; k < kMaxUnitsPerThread; ++k) {
      if (k < upt) {
        const int u = threadIdx.x + k * kTileThreads;
        if (u < nunits) {
          const int vox = u / NU, g8 = u - vox * NU;
          const int lx = vox % TX, ly = (vox / TX) % TY, lz = vox / (TX * TY);
          const int32_t x = ox + lx, y = oy + ly, z = oz + lz;
          if (x < sz[0] && y < sz[1] && z < sz[2]) {
            const int64_t kil = (static_cast<int64_t>(z) * sz[1] + y) * sz[0] + x;
            if (atomic_level) {
              float* dst = bb.acc + ((b * bp.acc_keys + bp.acc_start[l] + kil) * p.H + h) * C + g8 * 8;
              red_add_f32<8>(dst, acc[k]);
            } else {
              char* dst = reinterpret_cast<char*>(grad_value) +
                          ((b * p.K + start + kil) * p.H + h) * row_bytes + g8 * 8 * sizeof(T);
              if constexpr (sizeof(T) == 2) {
                st_chunk<16>(dst, Chunk<T, 16>::pack(acc[k]));
              } else {
                st_chunk<16>(dst, Chunk<T, 16>::pack(acc[k]));
                st_chunk<16>(dst + 16, Chunk<T, 16>::pack(acc[k] + 4));
              }
            }
          }
        }
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
