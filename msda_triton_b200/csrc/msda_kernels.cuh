// msda_kernels.cuh -- forward and backward MSDA kernels for sm_100a.
//
// Work decomposition (both kernels).  One (b, q, h) output row of C channels
// is owned by a group of G = 2^log2g adjacent lanes; lane j of the group owns
// the VB-byte channel chunks j, j+G, ... (VPL of them).  For the common C=32
// case that is 4 lanes x 16 B (bf16/fp16) or 8 lanes x 16 B (fp32), so every
// corner gather is a 128-bit load and a warp touches 8 (or 4) full 64/128-byte
// value rows per load instruction.  Accumulation is in fp32 registers and the
// output row is written once, directly in (B, Q, H*C) layout and the input
// dtype -- there is no fp32 staging tensor and no permute pass.
//
// Reference kernels these replace: _fwd_kernel_2d / _bwd_kernel_2d
// (src/msda_triton/triton/msda_2d.py:85-260, :263-510) and _fwd_kernel /
// _bwd_kernel (src/msda_triton/triton/msda_3d.py:80-288, :291-653).
#pragma once

#include <type_traits>

#include "msda_common.cuh"

namespace msda {

template <int NDIM>
struct Point {
  int32_t i0[3];
  float f[3];
  bool pass[3];
};

// d(weight of corner c)/d(source index) along each axis.
template <int NDIM>
__device__ __forceinline__ void corner_dweights(const Point<NDIM>& pt, int c, float* dw) {
  const float wx = (c & 1) ? pt.f[0] : 1.0f - pt.f[0];
  const float wy = (c & 2) ? pt.f[1] : 1.0f - pt.f[1];
  const float sx = (c & 1) ? 1.0f : -1.0f;
  const float sy = (c & 2) ? 1.0f : -1.0f;
  if (NDIM == 2) {
    dw[0] = sx * wy;
    dw[1] = sy * wx;
  } else {
    const float wz = (c & 4) ? pt.f[2] : 1.0f - pt.f[2];
    const float sz = (c & 4) ? 1.0f : -1.0f;
    dw[0] = sx * wy * wz;
    dw[1] = sy * wx * wz;
    dw[2] = sz * wx * wy;
  }
}

template <typename TS, int NDIM>
__device__ __forceinline__ Point<NDIM> load_point(const TS* lp, const int32_t* sz,
                                                  const Problem& p) {
  Point<NDIM> pt;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    pt.i0[a] = 0;
    pt.f[a] = 0.0f;
    pt.pass[a] = true;
  }
#pragma unroll
  for (int a = 0; a < NDIM; ++a) {
    const float x = Elem<TS>::to_f(lp[a]);
    resolve_axis(x, sz[a], p.clamp, p.lo, p.hi, pt.i0[a], pt.f[a], pt.pass[a]);
  }
  return pt;
}

// x / n rounded to nearest for a level size n, given r = 1/n rounded to
// nearest: the product x*r corrected once by its exact FMA residual
// (Markstein's method), which reproduces the IEEE quotient of the separate
// tensor division without a division per sample.
__device__ __forceinline__ float div_by_size(float x, float n, float r) {
  const float q = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q, n, x);
  return __fmaf_rn(e, r, q);
}

// Per-level sizes and their reciprocals for div_by_size.
template <int NDIM>
struct LevelRcp {
  float n[3];
  float r[3];
};

template <int NDIM>
__device__ __forceinline__ LevelRcp<NDIM> level_rcp(const int32_t* sz, const float* rcp) {
  LevelRcp<NDIM> lr;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    lr.n[a] = static_cast<float>(sz[a]);
    lr.r[a] = rcp[a];
  }
  return lr;
}

// Fused prologue: the location of one sample from its raw offset and the
// level's reference point, ref + offset / size per axis (size = W, H, D for
// x, y, z), with the rounding of the separate `ref + offsets / normalizer`
// expression (pytorch/msda_3d.py:336-339, pytorch/msda_2d.py:335-339).
template <typename TS, int NDIM>
__device__ __forceinline__ Point<NDIM> load_point_fused(const TS* off, const float* ref,
                                                        const int32_t* sz,
                                                        const LevelRcp<NDIM>& lr,
                                                        const Problem& p) {
  Point<NDIM> pt;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    pt.i0[a] = 0;
    pt.f[a] = 0.0f;
    pt.pass[a] = true;
  }
#pragma unroll
  for (int a = 0; a < NDIM; ++a) {
    const float x = __fadd_rn(ref[a], div_by_size(Elem<TS>::to_f(off[a]), lr.n[a], lr.r[a]));
    resolve_axis(x, sz[a], p.clamp, p.lo, p.hi, pt.i0[a], pt.f[a], pt.pass[a]);
  }
  return pt;
}

// Softmax of one row's L*P weight logits, shared by the row's G lanes: lane
// j takes logits j, j+G, ... in one pass (running maximum, the sum rescaled
// whenever it rises), then the G partial (max, sum) pairs are merged with
// butterfly shuffles, which leaves the same pair on every lane.  The weight
// of a sample is exp(x - max) * (1 / sum).  -inf logits weigh 0.  All lanes
// of the warp must call it.
struct RowSoftmax {
  float mx;
  float inv;
};

template <typename TS>
__device__ __forceinline__ RowSoftmax row_softmax(const TS* logits, int n, int j, int G) {
  float mx = -INFINITY;
  float sum = 0.0f;
  for (int i = j; i < n; i += G) {
    const float x = Elem<TS>::to_f(logits[i]);
    if (x > mx) {
      sum = fmaf(sum, expf(mx - x), 1.0f);
      mx = x;
    } else if (x != -INFINITY) {
      sum += expf(x - mx);
    }
  }
  for (int o = 1; o < G; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, mx, o);
    const float so = __shfl_xor_sync(0xffffffffu, sum, o);
    const float m = fmaxf(mx, mo);
    const float ta = sum == 0.0f ? 0.0f : sum * expf(mx - m);
    const float tb = so == 0.0f ? 0.0f : so * expf(mo - m);
    sum = ta + tb;
    mx = m;
  }
  return {mx, __frcp_rn(sum)};
}

__device__ __forceinline__ float softmax_weight(float x, const RowSoftmax& sm) {
  return expf(x - sm.mx) * sm.inv;
}

// A zero value row: invalid corners point here, so every lane loads finite
// zeros instead of selecting per register (the widest row is 2048 bytes).
static __device__ __align__(16) unsigned char g_zero_row[2048];

// Checked build (-DMSDA_CHECKED): every value gather and value-gradient
// scatter address is tested against the buffer it must stay inside.  A
// violation sets a bit in *p.check_flag (1: value gather, 2: 16-bit
// grad_value scatter, 4: fp32 accumulator scatter, 8: a shared-memory layout
// larger than its launch's) and the access is skipped; nothing traps.  The normal build compiles the plain accesses.
#ifdef MSDA_CHECKED
__device__ __forceinline__ bool msda_within(const void* a, int n, const void* base,
                                            int64_t bytes) {
  const char* c = static_cast<const char*>(a);
  const char* b = static_cast<const char*>(base);
  return b != nullptr && c >= b && c + n <= b + bytes;
}
template <typename T>
__device__ __forceinline__ int64_t msda_value_bytes(const Problem& p) {
  return p.B * p.K * p.H * p.C * static_cast<int64_t>(sizeof(T));
}
template <int VB, typename T>
__device__ __forceinline__ Raw<VB> checked_ld_value(const char* a, const Problem& p) {
  if (msda_within(a, VB, p.value, msda_value_bytes<T>(p)) ||
      msda_within(a, VB, g_zero_row, sizeof(g_zero_row)))
    return ld_chunk<VB>(a);
  atomicOr(p.check_flag, 1u);
  return raw_zero<VB>();
}
#define MSDA_LD_VALUE(VB, a) checked_ld_value<VB, T>((a), p)
#define MSDA_SCATTER_OK(a, n, base, bytes, bit) \
  (msda_within((a), (n), (base), (bytes)) || (atomicOr(p.check_flag, (bit)), false))
#else
#define MSDA_LD_VALUE(VB, a) ld_chunk<VB>(a)
#define MSDA_SCATTER_OK(a, n, base, bytes, bit) true
#endif

// Per-level constants of the gather kernels.
struct LevelGeom {
  int32_t sz[3];
  int32_t start;
  int64_t dx, dy, dz;   // byte offsets of the +1 neighbour along x, y, z
};

__device__ __forceinline__ LevelGeom level_geom(const LevelSmem& lv, int l, int64_t key_bytes) {
  LevelGeom g;
  g.sz[0] = lv.size[l][0];
  g.sz[1] = lv.size[l][1];
  g.sz[2] = lv.size[l][2];
  g.start = lv.start[l];
  g.dx = key_bytes;
  g.dy = key_bytes * g.sz[0];
  g.dz = g.dy * g.sz[1];
  return g;
}

// The 2^NDIM corners of one sample: row pointers (already offset to the lane's
// channels; the zero row for corners outside the level), interpolation weights
// (zero outside) and validity.
template <int NDIM>
struct Corners {
  const char* ptr[1 << NDIM];
  float w[1 << NDIM];
  bool valid[1 << NDIM];
};

template <int NDIM>
__device__ __forceinline__ Corners<NDIM> make_corners(const Point<NDIM>& pt, const LevelGeom& g,
                                                      const char* vbase, int64_t key_bytes,
                                                      int lane_off) {
  Corners<NDIM> cs;
  bool v[3][2];
  float wt[3][2];
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    if (a < NDIM) {
      v[a][0] = static_cast<uint32_t>(pt.i0[a]) < static_cast<uint32_t>(g.sz[a]);
      v[a][1] = static_cast<uint32_t>(pt.i0[a] + 1) < static_cast<uint32_t>(g.sz[a]);
      wt[a][0] = __fsub_rn(1.0f, pt.f[a]);
      wt[a][1] = pt.f[a];
    } else {
      v[a][0] = true; v[a][1] = false; wt[a][0] = 1.0f; wt[a][1] = 0.0f;
    }
  }
  const int32_t zi = (NDIM == 3) ? pt.i0[2] : 0;
  const int32_t key0 = g.start + (zi * g.sz[1] + pt.i0[1]) * g.sz[0] + pt.i0[0];
  const char* p0 = vbase + static_cast<int64_t>(key0) * key_bytes + lane_off;
  const char* zero = reinterpret_cast<const char*>(g_zero_row);
#pragma unroll
  for (int c = 0; c < (1 << NDIM); ++c) {
    const int bx = c & 1, by = (c >> 1) & 1, bz = (c >> 2) & 1;
    const bool ok = v[0][bx] && v[1][by] && v[2][bz];
    const char* pc = p0 + (bx ? g.dx : 0) + (by ? g.dy : 0) + (bz ? g.dz : 0);
    cs.ptr[c] = ok ? pc : zero;
    float w = __fmul_rn(wt[0][bx], wt[1][by]);
    if (NDIM == 3) w = __fmul_rn(w, wt[2][bz]);
    cs.w[c] = ok ? w : 0.0f;
    cs.valid[c] = ok;
  }
  return cs;
}

// One sample as a lane group needs it to gather its chunks: resolved once
// by one lane of the group and broadcast to the others (the scalar work of a
// sample -- location loads, axis resolution, corner validity, key of the
// lower corner -- then costs each lane a fraction, not all of it).
struct SampleMeta {
  int32_t key0;   // key of the lower corner (start + linear index; may lie
                  // outside the level where that corner is invalid)
  uint32_t info;  // bits 0-7: corner c valid; 8-10: clamp pass per axis;
                  // 12-15: level; bit 16: sample skipped by this kernel
  float f[3];     // fractional offsets
  float a;        // attention weight
};
constexpr uint32_t kMetaSkip = 1u << 16;

template <int NDIM>
__device__ __forceinline__ SampleMeta make_meta(const Point<NDIM>& pt, const LevelGeom& g,
                                                float a, int l) {
  SampleMeta m;
  bool v[3][2];
#pragma unroll
  for (int ax = 0; ax < 3; ++ax) {
    if (ax < NDIM) {
      v[ax][0] = static_cast<uint32_t>(pt.i0[ax]) < static_cast<uint32_t>(g.sz[ax]);
      v[ax][1] = static_cast<uint32_t>(pt.i0[ax] + 1) < static_cast<uint32_t>(g.sz[ax]);
    } else {
      v[ax][0] = true;
      v[ax][1] = false;
    }
  }
  uint32_t info = static_cast<uint32_t>(l) << 12;
#pragma unroll
  for (int c = 0; c < (1 << NDIM); ++c)
    if (v[0][c & 1] && v[1][(c >> 1) & 1] && v[2][(c >> 2) & 1]) info |= 1u << c;
#pragma unroll
  for (int ax = 0; ax < NDIM; ++ax)
    if (pt.pass[ax]) info |= 1u << (8 + ax);
  const int32_t zi = (NDIM == 3) ? pt.i0[2] : 0;
  m.key0 = g.start + (zi * g.sz[1] + pt.i0[1]) * g.sz[0] + pt.i0[0];
  m.info = info;
  m.f[0] = pt.f[0];
  m.f[1] = pt.f[1];
  m.f[2] = NDIM == 3 ? pt.f[2] : 0.0f;
  m.a = a;
  return m;
}

// Lane `src` of each G-lane segment of the warp -> every lane of the segment
// (all 32 lanes of the warp must take part).
template <int NDIM>
__device__ __forceinline__ SampleMeta shfl_meta(const SampleMeta& m, int src, int G) {
  SampleMeta r;
  r.key0 = __shfl_sync(0xffffffffu, m.key0, src, G);
  r.info = __shfl_sync(0xffffffffu, m.info, src, G);
#pragma unroll
  for (int ax = 0; ax < NDIM; ++ax) r.f[ax] = __shfl_sync(0xffffffffu, m.f[ax], src, G);
  if constexpr (NDIM == 2) r.f[2] = 0.0f;
  r.a = __shfl_sync(0xffffffffu, m.a, src, G);
  return r;
}

// The lane's chunks of the 2^d corner rows of a broadcast sample (corners
// outside the level read as zero).
template <typename T, int NDIM, int VB, int VPL>
__device__ __forceinline__ void gather_meta_corners(const Problem& p, const SampleMeta& m,
                                                    const LevelGeom& g, const char* vbase,
                                                    int64_t key_bytes, int lane_off, int G,
                                                    const bool* has,
                                                    Raw<VB> (&raw)[1 << NDIM][VPL]) {
  (void)p;
  const char* p0 = vbase + static_cast<int64_t>(m.key0) * key_bytes + lane_off;
#pragma unroll
  for (int c = 0; c < (1 << NDIM); ++c) {
    const char* pc = p0 + ((c & 1) ? g.dx : 0) + ((c & 2) ? g.dy : 0) + ((c & 4) ? g.dz : 0);
    const bool ok = (m.info >> c) & 1u;
#pragma unroll
    for (int vv = 0; vv < VPL; ++vv)
      raw[c][vv] = (ok && has[vv]) ? MSDA_LD_VALUE(VB, pc + vv * G * VB) : raw_zero<VB>();
  }
}

// ------------------------------------------------------------------ forward
template <typename T, typename TS, int NDIM, int VB, int VPL, bool FUSED>
__device__ __forceinline__ void msda_fwd_body(const Problem p, T* __restrict__ out) {
  __shared__ LevelSmem lv;
  load_levels(p, lv, NDIM);
  if constexpr (FUSED) load_level_rcps(p, lv);

  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;

  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  uint64_t r = tid >> p.log2g;
  const int G = 1 << p.log2g;
  const int j = static_cast<int>(tid & static_cast<uint64_t>(G - 1));
  bool active = true;
  if constexpr (FUSED) {
    // the fused prologue shuffles within lane groups: rows past the end stay
    // (on row 0, storing nothing) instead of leaving the warp
    active = r < static_cast<uint64_t>(p.B * p.Q * p.H);
    if (!active) r = 0;
  } else {
    if (r >= static_cast<uint64_t>(p.B * p.Q * p.H)) return;
  }

  const RowCoord rc = decode_row(static_cast<uint32_t>(r), p);
  const int64_t row = (rc.b * p.Q + rc.q) * p.H + rc.h;
  const int64_t key_bytes = key_stride(p) * static_cast<int64_t>(sizeof(T));
  const char* vbase = static_cast<const char*>(p.value) +
                      bh_base(p, rc.b, rc.h, p.K) * static_cast<int64_t>(sizeof(T));
  const int LP = static_cast<int>(p.L * p.P);
  const TS* lrow = static_cast<const TS*>(p.loc) + row * LP * NDIM;
  const TS* arow = static_cast<const TS*>(p.attn) + row * LP;

  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) has[v] = active && (j + v * G < p.nv);

  // FUSED: lrow / arow hold the raw offsets / logits of the row.  Lane j
  // computes the weight of every G-th sample; the others get it by shuffle.
  const float* rrow = nullptr;
  RowSoftmax sm{0.0f, 1.0f};
  float wchunk = 0.0f;
  const int gbase = static_cast<int>(threadIdx.x & 31u) & ~(G - 1);
  if constexpr (FUSED) {
    rrow = p.ref + (rc.b * p.Q + rc.q) * p.L * NDIM;
    sm = row_softmax<TS>(arow, LP, j, G);
  }

  float acc[VPL][EPV];
#pragma unroll
  for (int v = 0; v < VPL; ++v)
#pragma unroll
    for (int e = 0; e < EPV; ++e) acc[v][e] = 0.0f;

  const int P = static_cast<int>(p.P);
  for (int l = 0; l < p.L; ++l) {
    const LevelGeom g = level_geom(lv, l, key_bytes);
    LevelRcp<NDIM> lr;
    float rl[3];
    if constexpr (FUSED) {
      lr = level_rcp<NDIM>(g.sz, lv.rcp[l]);
#pragma unroll
      for (int ax = 0; ax < NDIM; ++ax) rl[ax] = rrow[l * NDIM + ax];
    }
    for (int pp = 0; pp < P; ++pp) {
      const int s = l * P + pp;
      Point<NDIM> pt;
      float a;
      if constexpr (FUSED) {
        if ((s & (G - 1)) == 0)
          wchunk = s + j < LP ? softmax_weight(Elem<TS>::to_f(arow[s + j]), sm) : 0.0f;
        a = __shfl_sync(0xffffffffu, wchunk, gbase | (s & (G - 1)));
        pt = load_point_fused<TS, NDIM>(lrow + s * NDIM, rl, g.sz, lr, p);
      } else {
        pt = load_point<TS, NDIM>(lrow + s * NDIM, g.sz, p);
        a = Elem<TS>::to_f(arow[s]);
      }
      const Corners<NDIM> cs = make_corners<NDIM>(pt, g, vbase, key_bytes, j * VB);
      Raw<VB> raw[NC][VPL];
#pragma unroll
      for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          raw[c][v] = has[v] ? MSDA_LD_VALUE(VB, cs.valid[c] ? cs.ptr[c] + v * G * VB : cs.ptr[c])
                             : raw_zero<VB>();
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float cw = a * cs.w[c];
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          float x[EPV];
          CK::unpack(raw[c][v], x);
#pragma unroll
          for (int e = 0; e < EPV; ++e) acc[v][e] = fmaf(cw, x[e], acc[v][e]);
        }
      }
    }
  }

  char* orow = reinterpret_cast<char*>(out) + row * p.C * static_cast<int64_t>(sizeof(T));
#pragma unroll
  for (int v = 0; v < VPL; ++v)
    if (has[v]) st_chunk<VB>(orow + (j + v * G) * VB, CK::pack(acc[v]));
}

template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads)
    msda_fwd_kernel(const Problem p, T* __restrict__ out) {
  msda_fwd_body<T, TS, NDIM, VB, VPL, false>(p, out);
}

// The fused one-chunk-per-lane variants (the common row shapes) are held to
// the occupancy of the plain kernels; wider rows would spill.
template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads, VPL == 1 ? 4 : 1)
    msda_fwd_fused_kernel(const Problem p, T* __restrict__ out) {
  msda_fwd_body<T, TS, NDIM, VB, VPL, true>(p, out);
}

// ------------------------------------------------------------------ backward
// Vector fp32 reductions into global memory (red.global.add.v{2,4}.f32 is
// sm_90+; the address is aligned to the vector width by construction).
template <int N>
__device__ __forceinline__ void red_add_f32(float* dst, const float* v) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + i),
                   "f"(v[i]), "f"(v[i + 1]), "f"(v[i + 2]), "f"(v[i + 3])
                   : "memory");
  } else if constexpr (N == 2) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(dst), "f"(v[0]), "f"(v[1])
                 : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) atomicAdd(dst + i, v[i]);
  }
}

// Vector reductions of N 16-bit channels straight into a bf16/fp16 tensor
// (red.global.add.noftz.v{2,4}.{bf16x2,f16x2} is sm_90+).  Each pair of fp32
// contributions is rounded to the element type once, then added by the L2.
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T, int N>
__device__ __forceinline__ void red_add_16(T* dst, const float* v) {
  constexpr bool kBf = std::is_same<T, __nv_bfloat16>::value;
  if constexpr (N % 8 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 8) {
      const uint32_t a = pack_pair<T>(v[i], v[i + 1]), b = pack_pair<T>(v[i + 2], v[i + 3]);
      const uint32_t c = pack_pair<T>(v[i + 4], v[i + 5]), d = pack_pair<T>(v[i + 6], v[i + 7]);
      if constexpr (kBf)
        asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst + i),
                     "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
      else
        asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst + i),
                     "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
    }
  } else if constexpr (N == 4) {
    const uint32_t a = pack_pair<T>(v[0], v[1]), b = pack_pair<T>(v[2], v[3]);
    if constexpr (kBf)
      asm volatile("red.global.add.noftz.v2.bf16x2 [%0], {%1, %2};" ::"l"(dst), "r"(a), "r"(b)
                   : "memory");
    else
      asm volatile("red.global.add.noftz.v2.f16x2 [%0], {%1, %2};" ::"l"(dst), "r"(a), "r"(b)
                   : "memory");
  } else if constexpr (N == 2) {
    const uint32_t a = pack_pair<T>(v[0], v[1]);
    if constexpr (kBf)
      asm volatile("red.global.add.noftz.bf16x2 [%0], %1;" ::"l"(dst), "r"(a) : "memory");
    else
      asm volatile("red.global.add.noftz.f16x2 [%0], %1;" ::"l"(dst), "r"(a) : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) atomicAdd(dst + i, Elem<T>::from_f(v[i]));
  }
}

// One pass produces all three gradients.  grad_out is read once per row
// (the reference re-reads it for every (level, point), msda_3d.py:451-455).
// grad_loc and grad_attn are reduced inside the lane group with shuffles and
// written with plain stores by the group's first lane (one owner per sample:
// no atomics and no zero-fill).  grad_value is scattered with vector fp32
// reductions into `gacc` (grad_value itself for fp32, else an fp32 workspace
// that msda_cast_kernel rounds to the input dtype).  For 16-bit inputs the
// host picks 8-byte chunks (VB = 8): lane j then owns channel groups j, j+G,
// ... of 4 channels, so one red.v4.f32 per group and the G lanes of a row
// cover whole 32-byte sectors of the accumulator.  Levels flagged in
// p.direct16 (few contributions per element) instead reduce with 16-bit
// vector reductions straight into grad_value, as the reference's own
// atomic_add into a grad_value of the input dtype does
// (src/msda_triton/triton/msda_3d.py:477, :942); the other levels keep fp32
// accumulation, possibly in a compacted accumulator (p.acc_start).
//
// FUSED (prologue inside the kernel): grad_loc receives the offset gradient
// (location gradient / size), p.ref_partial the per-level sums over points of
// the location gradient (the reference-point gradient before the sum over
// heads), and grad_attn the logit gradient: during the sample loop it holds
// dL/dweight, and the row's last step turns it into the softmax backward
// w * (dL/dw - sum(w * dL/dw)).
template <typename T, typename TS, int NDIM, int VB, int VPL, bool FUSED>
__device__ __forceinline__ void msda_bwd_body(const Problem p, const T* __restrict__ grad_out,
                                              float* __restrict__ gacc, TS* __restrict__ grad_loc,
                                              TS* __restrict__ grad_attn) {
  __shared__ LevelSmem lv;
  load_levels(p, lv, NDIM);
  if constexpr (FUSED) load_level_rcps(p, lv);

  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;

  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const uint64_t r = tid >> p.log2g;
  const int G = 1 << p.log2g;
  const int j = static_cast<int>(tid & static_cast<uint64_t>(G - 1));
  // Rows past the end still run the loop (masked) so the group shuffles
  // below always see every lane of the warp.
  const bool active = r < static_cast<uint64_t>(p.B * p.Q * p.H);

  RowCoord rc{0, 0, 0};
  if (active) rc = decode_row(static_cast<uint32_t>(r), p);
  const int64_t row = (rc.b * p.Q + rc.q) * p.H + rc.h;
  const int64_t key_bytes = key_stride(p) * static_cast<int64_t>(sizeof(T));
  const char* vbase = static_cast<const char*>(p.value) +
                      bh_base(p, rc.b, rc.h, p.K) * static_cast<int64_t>(sizeof(T));
  const int LP = static_cast<int>(p.L * p.P);
  const TS* lrow = static_cast<const TS*>(p.loc) + row * LP * NDIM;
  const TS* arow = static_cast<const TS*>(p.attn) + row * LP;

  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) has[v] = active && (j + v * G < p.nv);

  // FUSED: lrow / arow hold the raw offsets / logits of the row (row 0's for
  // the masked lanes past the end, which never store).
  const float* rrow = nullptr;
  RowSoftmax sm{0.0f, 1.0f};
  float wdot = 0.0f;  // sum over the row's samples of weight * dL/dweight
  float wchunk = 0.0f;
  const int gbase = static_cast<int>(threadIdx.x & 31u) & ~(G - 1);
  if constexpr (FUSED) {
    rrow = p.ref + (rc.b * p.Q + rc.q) * p.L * NDIM;
    sm = row_softmax<TS>(arow, LP, j, G);
  }

  float go[VPL][EPV];
  const char* gorow = reinterpret_cast<const char*>(grad_out) +
                      row * p.C * static_cast<int64_t>(sizeof(T));
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const Raw<VB> rg = has[v] ? ld_chunk<VB>(gorow + (j + v * G) * VB) : raw_zero<VB>();
    CK::unpack(rg, go[v]);
  }

  const int P = static_cast<int>(p.P);
  const char* vlane = vbase + j * VB;
  // A corner's value row sits at byte offset vo from vlane (key * key_bytes).
  // The same key's fp32 accumulator row is at vo * 4 / sizeof(T) from the
  // level's accumulator base (keys shifted to the compacted layout), and its
  // grad_value row (direct levels) at the same byte offset vo.
  const int64_t vrow = bh_base(p, rc.b, rc.h, p.K);
  char* g16lane = static_cast<char*>(p.grad_value16) + vrow * static_cast<int64_t>(sizeof(T)) +
                  j * VB;
  for (int l = 0; l < p.L; ++l) {
    const LevelGeom g = level_geom(lv, l, key_bytes);
    const bool d16 = (sizeof(T) == 2) && ((p.direct16 >> l) & 1);
    float ref_sum[3] = {0.0f, 0.0f, 0.0f};  // FUSED: this level's location-gradient sum
    LevelRcp<NDIM> lr;
    float rl[3];
    if constexpr (FUSED) {
      lr = level_rcp<NDIM>(g.sz, lv.rcp[l]);
#pragma unroll
      for (int ax = 0; ax < NDIM; ++ax) rl[ax] = rrow[l * NDIM + ax];
    }
    const int64_t kshift = p.acc_compact ? p.acc_start[l] - g.start : 0;
    char* acc_lane = reinterpret_cast<char*>(
        gacc + bh_base(p, rc.b, rc.h, p.acc_keys) + kshift * key_stride(p) + j * EPV);
    for (int pp = 0; pp < P; ++pp) {
      const int s = l * P + pp;
      Point<NDIM> pt;
      float a = 0.0f;
      if constexpr (FUSED) {
        // every G-th weight per lane, shared by shuffle (all lanes take part)
        if ((s & (G - 1)) == 0)
          wchunk = s + j < LP ? softmax_weight(Elem<TS>::to_f(arow[s + j]), sm) : 0.0f;
        a = __shfl_sync(0xffffffffu, wchunk, gbase | (s & (G - 1)));
        if (!active) a = 0.0f;
      }
      if (active) {
        if constexpr (FUSED) {
          pt = load_point_fused<TS, NDIM>(lrow + s * NDIM, rl, g.sz, lr, p);
        } else {
          pt = load_point<TS, NDIM>(lrow + s * NDIM, g.sz, p);
          a = Elem<TS>::to_f(arow[s]);
        }
      } else {
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) {
          pt.i0[ax] = -2;
          pt.f[ax] = 0.0f;
          pt.pass[ax] = false;
        }
      }
      const Corners<NDIM> cs = make_corners<NDIM>(pt, g, vbase, key_bytes, j * VB);
      Raw<VB> raw[NC][VPL];
#pragma unroll
      for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          raw[c][v] = has[v] ? MSDA_LD_VALUE(VB, cs.valid[c] ? cs.ptr[c] + v * G * VB : cs.ptr[c])
                             : raw_zero<VB>();

      float dots[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        float dot = 0.0f;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          float x[EPV];
          CK::unpack(raw[c][v], x);
#pragma unroll
          for (int e = 0; e < EPV; ++e) dot = fmaf(go[v][e], x[e], dot);
        }
        dots[c] = dot;
        if (cs.valid[c]) {
          const float aw = a * cs.w[c];
          const int64_t vo = cs.ptr[c] - vlane;
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            if (has[v]) {
              float t[EPV];
#pragma unroll
              for (int e = 0; e < EPV; ++e) t[e] = aw * go[v][e];
              if constexpr (sizeof(T) == 2) {
                if (d16) {
                  T* dst16 = reinterpret_cast<T*>(g16lane + vo + v * G * VB);
                  if (MSDA_SCATTER_OK(dst16, EPV * static_cast<int>(sizeof(T)), p.grad_value16,
                                      p.B * p.K * p.H * p.C * static_cast<int64_t>(sizeof(T)), 2u))
                    red_add_16<T, EPV>(dst16, t);
                  continue;
                }
              }
              float* dst32 = reinterpret_cast<float*>(acc_lane + vo * (4 / sizeof(T))) +
                             v * G * EPV;
              if (MSDA_SCATTER_OK(dst32, EPV * 4, gacc,
                                  p.B * p.acc_keys * p.H * p.C * int64_t{4}, 4u))
                red_add_f32<EPV>(dst32, t);
            }
          }
        }
      }
      // Per-sample scalars: d out / d attn and d out / d (source index).
      float g_attn = 0.0f;
#pragma unroll
      for (int c = 0; c < NC; ++c) g_attn = fmaf(cs.w[c], dots[c], g_attn);
      float g_ix[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < NC; ++c) {  // invalid corners read the zero row: dots[c] == 0
        float dw[3];
        corner_dweights<NDIM>(pt, c, dw);
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) g_ix[ax] = fmaf(dw[ax], dots[c], g_ix[ax]);
      }
      for (int o = G >> 1; o > 0; o >>= 1) {
        g_attn += __shfl_xor_sync(0xffffffffu, g_attn, o);
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) g_ix[ax] += __shfl_xor_sync(0xffffffffu, g_ix[ax], o);
      }
      if constexpr (FUSED) wdot = fmaf(a, g_attn, wdot);
      if (active && j == 0) {
        grad_attn[row * LP + s] = Elem<TS>::from_f(g_attn);
        TS* gl = grad_loc + (row * LP + s) * NDIM;
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) {
          const float size = static_cast<float>(g.sz[ax]);
          const float gval = pt.pass[ax] ? a * g_ix[ax] * size : 0.0f;
          if constexpr (FUSED) {
            gl[ax] = Elem<TS>::from_f(div_by_size(gval, lr.n[ax], lr.r[ax]));
            ref_sum[ax] += gval;
          } else {
            gl[ax] = Elem<TS>::from_f(gval);
          }
        }
      }
    }
    if constexpr (FUSED) {
      if (active && j == 0) {
        float* rp = p.ref_partial + (row * p.L + l) * NDIM;
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) rp[ax] = ref_sum[ax];
      }
    }
  }
  if constexpr (FUSED) {
    // softmax backward over the row's L*P logits, spread over the row's
    // lanes (lane 0 stored dL/dw above; every lane holds wdot)
    __syncwarp();
    if (active) {
      TS* ga = grad_attn + row * LP;
      for (int s = j; s < LP; s += G) {
        const float w = softmax_weight(Elem<TS>::to_f(arow[s]), sm);
        ga[s] = Elem<TS>::from_f(w * (Elem<TS>::to_f(ga[s]) - wdot));
      }
    }
  }
}

template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads)
    msda_bwd_kernel(const Problem p, const T* __restrict__ grad_out, float* __restrict__ gacc,
                    TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  msda_bwd_body<T, TS, NDIM, VB, VPL, false>(p, grad_out, gacc, grad_loc, grad_attn);
}

// One-chunk rows are held to the plain kernel's occupancy (3 CTAs/SM for
// 16-bit values, 2 for fp32); wider rows would spill.
template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads, VPL == 1 ? (sizeof(T) == 2 ? 3 : 2) : 1)
    msda_bwd_fused_kernel(const Problem p, const T* __restrict__ grad_out,
                          float* __restrict__ gacc, TS* __restrict__ grad_loc,
                          TS* __restrict__ grad_attn) {
  msda_bwd_body<T, TS, NDIM, VB, VPL, true>(p, grad_out, gacc, grad_loc, grad_attn);
}

// fp32 accumulation buffer -> grad_value in the input dtype.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    msda_cast_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads * 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * 4; i < n;
       i += stride) {
    if (i + 4 <= n) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      dst[i] = Elem<T>::from_f(v.x);
      dst[i + 1] = Elem<T>::from_f(v.y);
      dst[i + 2] = Elem<T>::from_f(v.z);
      dst[i + 3] = Elem<T>::from_f(v.w);
    } else {
      for (int64_t k = i; k < n; ++k) dst[k] = Elem<T>::from_f(src[k]);
    }
  }
}

// Compacted fp32 accumulator (the keys of the levels not in p.direct16,
// p.acc_keys per batch entry) -> their grad_value rows in the input dtype.
// One lane group per row (a key's H*C elements, or a (head, key)'s C
// elements head-major): the row's batch entry, level and destination key are
// resolved once per row, then the lanes stream its elements.
// V = 4: float4 in, one 8-byte store out (16-bit T, H*C % 4 == 0, grad_value
// 8-byte aligned); V = 1 otherwise.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads)
    msda_compact_cast_kernel(const Problem p, const float* __restrict__ acc, T* __restrict__ gv) {
  // A row: one key's H*C elements (channel-last) or one (head, key)'s C
  // elements (head-major); rows run batch entry, [head,] key.
  // Lane groups of lpr lanes (the power of two covering a row's vectors, at
  // most 32) take one row each.
  const int64_t row = key_stride(p);
  const int64_t rv = row / V;
  const int64_t rows_b = p.head_major ? p.H * p.acc_keys : p.acc_keys;  // rows per batch entry
  const int64_t nrows = p.B * rows_b;
  int lpr = 1;
  while (lpr < 32 && lpr < rv) lpr <<= 1;
  const int lane = static_cast<int>(threadIdx.x) & (lpr - 1);
  const int64_t ngroups = static_cast<int64_t>(gridDim.x) * (kThreads / lpr);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / lpr; r < nrows;
       r += ngroups) {
    const int64_t b = r / rows_b;
    const int64_t rr = r - b * rows_b;
    const int64_t h = p.head_major ? rr / p.acc_keys : 0;
    const int64_t ak = rr - h * p.acc_keys;
    int64_t shift = 0;  // key - accumulator key of the level holding ak
#pragma unroll
    for (int k = 0; k < kMaxLevels; ++k)
      if (k < p.L && !((p.direct16 >> k) & 1) && ak >= p.acc_start[k])
        shift = static_cast<int64_t>(p.lv.start[k]) - p.acc_start[k];
    const float* src = acc + r * row;
    T* dst = gv + bh_base(p, b, h, p.K) + (ak + shift) * row;
    for (int64_t e = lane; e < rv; e += lpr) {
      if constexpr (V == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + e * 4);
        struct alignas(8) Quad { T h[4]; } o;
        o.h[0] = Elem<T>::from_f(v.x);
        o.h[1] = Elem<T>::from_f(v.y);
        o.h[2] = Elem<T>::from_f(v.z);
        o.h[3] = Elem<T>::from_f(v.w);
        *reinterpret_cast<Quad*>(dst + e * 4) = o;
      } else {
        dst[e] = Elem<T>::from_f(src[e]);
      }
    }
  }
}

// The same rounding as msda_compact_cast_kernel, one (batch entry[, head],
// level) span per blockIdx.y: the accumulator rows of a level and its
// grad_value rows are each one contiguous range (rows of H*C elements, or C
// head-major), so a span is a plain streaming cast of float4 -> 4 elements.
// Needs rows of a multiple of 4 elements and grad_value 8-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    msda_span_cast_kernel(const Problem p, const float* __restrict__ acc, T* __restrict__ gv) {
  const int l = static_cast<int>(blockIdx.y % static_cast<uint32_t>(p.L));
  const int64_t bh = blockIdx.y / static_cast<uint32_t>(p.L);
  if ((p.direct16 >> l) & 1) return;  // a level the accumulator does not hold
  const int64_t b = p.head_major ? bh / p.H : bh;
  const int64_t h = p.head_major ? bh - b * p.H : 0;
  const int64_t row = key_stride(p);
  const int64_t nvox = int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2];
  const float4* src = reinterpret_cast<const float4*>(
      acc + bh_base(p, b, h, p.acc_keys) + int64_t{p.acc_start[l]} * row);
  T* dst = gv + bh_base(p, b, h, p.K) + int64_t{p.lv.start[l]} * row;
  const int64_t n4 = nvox * row / 4;
  struct alignas(8) Quad { T e[4]; };
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const float4 v = src[i];
    Quad o;
    o.e[0] = Elem<T>::from_f(v.x);
    o.e[1] = Elem<T>::from_f(v.y);
    o.e[2] = Elem<T>::from_f(v.z);
    o.e[3] = Elem<T>::from_f(v.w);
    reinterpret_cast<Quad*>(dst)[i] = o;
  }
}

}  // namespace msda
