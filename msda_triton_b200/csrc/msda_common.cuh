// msda_common.cuh -- shared device code for the multi-scale deformable
// attention (MSDA) kernels: problem description, level table, vector
// load/convert helpers and the sampling-coordinate resolution.
//
// Semantics follow the reference's pure-PyTorch path
// (src/msda_triton/pytorch/msda_2d.py:58-114, msda_3d.py:58-118), i.e.
// grid_sample(align_corners=False, padding_mode="zeros") on a grid-space
// clamp:
//   g  = 2*loc - 1, clamped to [lo, hi] = [-1+eps, 1-eps] when clamp_grid
//   ix = ((g + 1) * size - 1) / 2
//   corners floor(ix) and floor(ix)+1 per axis, zero outside [0, size).
// Every coordinate step is an explicitly rounded float op (__f*_rn), so nvcc
// cannot contract it into an FMA and the cell a point falls in is the same
// one the CPU restatement picks.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace msda {

constexpr int kMaxLevels = 16;
constexpr int kThreads = 256;

// Per-level metadata.  Axis order is (x, y, z) = (W, H, D); z size is 1 in 2D.
struct LevelTable {
  int32_t size[kMaxLevels][3];
  int32_t start[kMaxLevels];
};

// Everything a launch needs, passed by value as one kernel parameter.
struct Problem {
  const void* value;          // (B, K, H, C) of T, or (B, H, K, C) with head_major
  const void* loc;            // (B, Q, H, L, P, d) of TS
  const void* attn;           // (B, Q, H, L, P) of TS
  const int32_t* shapes_dev;  // (L, d) int32 on device, or nullptr
  int64_t B, K, H, C, Q, L, P;
  int32_t nv;         // vectors per (b,q,h) row: C * sizeof(T) / VB
  int32_t log2g;      // lanes per row = 1 << log2g
  int32_t hg;         // heads per scheduling group (divides H)
  int32_t clamp;      // clamp_grid
  int32_t head_major; // value / grad_value / fp32 accumulators laid out (B, H, K, C)
  float lo, hi;       // clamp window in grid space
  LevelTable lv;      // host-resolved table (used when shapes_dev == nullptr)
  // Backward value-gradient targets of the gather/scatter kernel (16-bit
  // values).  Level l reduces straight into grad_value16 (same layout as
  // value) when bit l of direct16 is set, else into the fp32 accumulator,
  // whose rows are keys [0, acc_keys) per batch: with acc_compact the keys of
  // level l start at acc_start[l] (only non-direct levels are stored), else
  // the accumulator has value's own key layout (acc_keys == K).
  int32_t direct16;
  int32_t acc_compact;
  int64_t acc_keys;
  int32_t acc_start[kMaxLevels];
  void* grad_value16;
  // Fused prologue (kernels instantiated with FUSED): `loc` holds the raw
  // sampling offsets and `attn` the raw weight logits (same shapes); the
  // location is ref + offset / size per axis and the weight is the softmax
  // of the row's L*P logits.  ref: fp32 reference points (B, Q, L, d).
  // ref_partial (backward output): fp32 (B, Q, H, L, d), the sum over the
  // row's points of each level's location gradient.
  const float* ref;
  float* ref_partial;
  // Checked build (MSDA_CHECKED): device word whose bits record the gather
  // and scatter addresses that fell outside their buffers (never set
  // otherwise; nullptr in the normal build).
  unsigned int* check_flag;
};

// ---------------------------------------------------------------- layout
// Element offsets into value, grad_value and the fp32 value-gradient
// accumulators.  Channel-last, the reference's tensor contract: (B, K, H, C),
// the H heads of a key side by side.  Head-major: (B, H, K, C), each head's
// keys contiguous (what a value projection can write directly,
// pytorch/msda_3d.py:302-305 reshapes its output to (B, K, H, C)).  An
// accumulator has the layout of value with `keys` keys per batch entry.
__host__ __device__ __forceinline__ int64_t key_stride(const Problem& p) {
  return p.head_major ? p.C : p.H * p.C;
}
__host__ __device__ __forceinline__ int64_t bh_base(const Problem& p, int64_t b, int64_t h,
                                                    int64_t keys) {
  return p.head_major ? (b * p.H + h) * keys * p.C : (b * keys * p.H + h) * p.C;
}

// ---------------------------------------------------------------- types
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// A VB-byte chunk of a channel row, held as 32-bit words (VB >= 4) or one
// 16-bit word (VB == 2).
template <int VB> struct Raw { uint32_t w[VB / 4]; };
template <> struct Raw<2> { uint16_t h; };

template <int VB> __device__ __forceinline__ Raw<VB> raw_zero() {
  Raw<VB> r;
#pragma unroll
  for (int i = 0; i < VB / 4; ++i) r.w[i] = 0u;
  return r;
}
template <> __device__ __forceinline__ Raw<2> raw_zero<2>() { Raw<2> r; r.h = 0; return r; }

// Read-only (non-coherent path) loads of one chunk.
template <int VB> __device__ __forceinline__ Raw<VB> ld_chunk(const void* p);
template <> __device__ __forceinline__ Raw<16> ld_chunk<16>(const void* p) {
  uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  Raw<16> r; r.w[0] = v.x; r.w[1] = v.y; r.w[2] = v.z; r.w[3] = v.w; return r;
}
template <> __device__ __forceinline__ Raw<8> ld_chunk<8>(const void* p) {
  uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
  Raw<8> r; r.w[0] = v.x; r.w[1] = v.y; return r;
}
template <> __device__ __forceinline__ Raw<4> ld_chunk<4>(const void* p) {
  Raw<4> r; r.w[0] = __ldg(reinterpret_cast<const unsigned int*>(p)); return r;
}
template <> __device__ __forceinline__ Raw<2> ld_chunk<2>(const void* p) {
  Raw<2> r; r.h = __ldg(reinterpret_cast<const unsigned short*>(p)); return r;
}

template <int VB> __device__ __forceinline__ void st_chunk(void* p, const Raw<VB>& r);
template <> __device__ __forceinline__ void st_chunk<16>(void* p, const Raw<16>& r) {
  *reinterpret_cast<uint4*>(p) = make_uint4(r.w[0], r.w[1], r.w[2], r.w[3]);
}
template <> __device__ __forceinline__ void st_chunk<8>(void* p, const Raw<8>& r) {
  *reinterpret_cast<uint2*>(p) = make_uint2(r.w[0], r.w[1]);
}
template <> __device__ __forceinline__ void st_chunk<4>(void* p, const Raw<4>& r) {
  *reinterpret_cast<unsigned int*>(p) = r.w[0];
}
template <> __device__ __forceinline__ void st_chunk<2>(void* p, const Raw<2>& r) {
  *reinterpret_cast<unsigned short*>(p) = r.h;
}

// Unpack a chunk into EPV = VB / sizeof(T) floats, and pack floats back.
template <typename T, int VB> struct Chunk;
template <int VB> struct Chunk<float, VB> {
  static constexpr int EPV = VB / 4;
  static __device__ __forceinline__ void unpack(const Raw<VB>& r, float* f) {
#pragma unroll
    for (int i = 0; i < EPV; ++i) f[i] = __uint_as_float(r.w[i]);
  }
  static __device__ __forceinline__ Raw<VB> pack(const float* f) {
    Raw<VB> r;
#pragma unroll
    for (int i = 0; i < EPV; ++i) r.w[i] = __float_as_uint(f[i]);
    return r;
  }
};
template <int VB> struct Chunk<__nv_bfloat16, VB> {
  static constexpr int EPV = VB / 2;
  static __device__ __forceinline__ void unpack(const Raw<VB>& r, float* f) {
#pragma unroll
    for (int i = 0; i < VB / 4; ++i) {
      f[2 * i] = __uint_as_float(r.w[i] << 16);
      f[2 * i + 1] = __uint_as_float(r.w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ Raw<VB> pack(const float* f) {
    Raw<VB> r;
#pragma unroll
    for (int i = 0; i < VB / 4; ++i) {
      __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      r.w[i] = *reinterpret_cast<uint32_t*>(&v);
    }
    return r;
  }
};
template <> struct Chunk<__nv_bfloat16, 2> {
  static constexpr int EPV = 1;
  static __device__ __forceinline__ void unpack(const Raw<2>& r, float* f) {
    f[0] = __uint_as_float(static_cast<uint32_t>(r.h) << 16);
  }
  static __device__ __forceinline__ Raw<2> pack(const float* f) {
    __nv_bfloat16 v = __float2bfloat16_rn(f[0]);
    Raw<2> r; r.h = *reinterpret_cast<uint16_t*>(&v); return r;
  }
};
template <int VB> struct Chunk<__half, VB> {
  static constexpr int EPV = VB / 2;
  static __device__ __forceinline__ void unpack(const Raw<VB>& r, float* f) {
#pragma unroll
    for (int i = 0; i < VB / 4; ++i) {
      uint32_t w = r.w[i];
      float2 v = __half22float2(*reinterpret_cast<__half2*>(&w));
      f[2 * i] = v.x; f[2 * i + 1] = v.y;
    }
  }
  static __device__ __forceinline__ Raw<VB> pack(const float* f) {
    Raw<VB> r;
#pragma unroll
    for (int i = 0; i < VB / 4; ++i) {
      __half2 v = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      r.w[i] = *reinterpret_cast<uint32_t*>(&v);
    }
    return r;
  }
};
template <> struct Chunk<__half, 2> {
  static constexpr int EPV = 1;
  static __device__ __forceinline__ void unpack(const Raw<2>& r, float* f) {
    uint16_t h = r.h;
    f[0] = __half2float(*reinterpret_cast<__half*>(&h));
  }
  static __device__ __forceinline__ Raw<2> pack(const float* f) {
    __half v = __float2half_rn(f[0]);
    Raw<2> r; r.h = *reinterpret_cast<uint16_t*>(&v); return r;
  }
};

// acc + <g, x> over one chunk's elements in element order, each product
// exact and each step rounded once (an fp32 FMA on the widened operands).
// 16-bit chunks use the mixed-precision FMA (fma.rn.f32.{bf16,f16}, sm_100),
// which takes the 16-bit operands as they are: no unpacking.
template <typename T, int VB> struct DotChunk {
  static __device__ __forceinline__ float fma(const Raw<VB>& g, const Raw<VB>& x, float acc) {
    float gf[Chunk<T, VB>::EPV], xf[Chunk<T, VB>::EPV];
    Chunk<T, VB>::unpack(g, gf);
    Chunk<T, VB>::unpack(x, xf);
#pragma unroll
    for (int e = 0; e < Chunk<T, VB>::EPV; ++e) acc = fmaf(gf[e], xf[e], acc);
    return acc;
  }
};
#define MSDA_MIXED_DOT(TY, SUF)                                                             \
  template <int VB> struct DotChunk<TY, VB> {                                                \
    static __device__ __forceinline__ float fma(const Raw<VB>& g, const Raw<VB>& x,          \
                                                float acc) {                                \
      _Pragma("unroll") for (int i = 0; i < VB / 4; ++i)                                    \
        asm("{\n .reg .b16 gl, gh, xl, xh;\n mov.b32 {gl, gh}, %1;\n mov.b32 {xl, xh}, %2;\n" \
            " fma.rn.f32." SUF " %0, gl, xl, %0;\n fma.rn.f32." SUF " %0, gh, xh, %0;\n}"  \
            : "+f"(acc) : "r"(g.w[i]), "r"(x.w[i]));                                        \
      return acc;                                                                            \
    }                                                                                        \
  };                                                                                         \
  template <> struct DotChunk<TY, 2> {                                                       \
    static __device__ __forceinline__ float fma(const Raw<2>& g, const Raw<2>& x,            \
                                                float acc) {                                \
      asm("fma.rn.f32." SUF " %0, %1, %2, %0;" : "+f"(acc) : "h"(g.h), "h"(x.h));            \
      return acc;                                                                            \
    }                                                                                        \
  };
MSDA_MIXED_DOT(__nv_bfloat16, "bf16")
MSDA_MIXED_DOT(__half, "f16")
#undef MSDA_MIXED_DOT

// ---------------------------------------------------------------- levels
struct LevelSmem {
  int32_t size[kMaxLevels][3];
  int32_t start[kMaxLevels];
  float rcp[kMaxLevels][3];  // 1 / size rounded to nearest (fused prologue only)
};

// Fill the CTA's level table.  Host-resolved tables are copied.  Device
// shapes are read here (no host sync, like the reference's GPU-shape path,
// triton/msda_2d.py:76-82); a level that would reach past K -- and every
// level after it -- is disabled, with the size product checked before it can
// overflow, so a malformed device table can never cause an out-of-range read.
__device__ __forceinline__ void load_levels(const Problem& p, LevelSmem& s, int ndim) {
  if (threadIdx.x == 0) {
    if (p.shapes_dev == nullptr) {
      for (int l = 0; l < p.L; ++l) {
        s.size[l][0] = p.lv.size[l][0];
        s.size[l][1] = p.lv.size[l][1];
        s.size[l][2] = p.lv.size[l][2];
        s.start[l] = p.lv.start[l];
      }
    } else {
      int64_t start = 0;
      for (int l = 0; l < p.L; ++l) {
        int32_t sz[3] = {1, 1, 1};
        int64_t n = 1;
        bool fits = true;
        for (int a = 0; a < ndim; ++a) {
          int32_t v = p.shapes_dev[l * ndim + (ndim - 1 - a)];
          v = v < 0 ? 0 : v;
          sz[a] = v;
          // stop before the product can overflow: a level larger than K
          // cannot fit anyway
          if (v > p.K || (v > 0 && n > p.K / v)) fits = false;
          else n *= v;
        }
        fits = fits && start + n <= p.K;
        if (!fits) n = p.K + 1;  // the levels after a misfit start past K as well
        s.size[l][0] = fits ? sz[0] : 0;
        s.size[l][1] = fits ? sz[1] : 0;
        s.size[l][2] = fits ? sz[2] : 0;
        s.start[l] = fits ? static_cast<int32_t>(start) : 0;
        start += n;
      }
    }
  }
  __syncthreads();
}

// The reciprocals of the level sizes for the fused prologue's divisions,
// once per CTA (after load_levels).
__device__ __forceinline__ void load_level_rcps(const Problem& p, LevelSmem& s) {
  const int t = static_cast<int>(threadIdx.x);
  if (t < p.L * 3) s.rcp[t / 3][t % 3] = __frcp_rn(static_cast<float>(s.size[t / 3][t % 3]));
  __syncthreads();
}

// ---------------------------------------------------------------- coordinates
// Resolve one normalised coordinate on an axis of `size` cells to the lower
// corner index i0, the fractional offset f, and the clamp-backward mask.
__device__ __forceinline__ void resolve_axis(float x, int32_t size, int clamp, float lo,
                                             float hi, int32_t& i0, float& f, bool& pass) {
  float g = __fsub_rn(__fmul_rn(2.0f, x), 1.0f);
  pass = true;
  if (clamp) {
    pass = (g >= lo) && (g <= hi);
    g = (g < lo) ? lo : g;
    g = (g > hi) ? hi : g;
  }
  const float t = __fsub_rn(__fmul_rn(__fadd_rn(g, 1.0f), static_cast<float>(size)), 1.0f);
  const float ix = __fmul_rn(t, 0.5f);
  const float fl = floorf(ix);
  // NaN coordinates resolve to cells -2/-1: both corners read zero padding.
  i0 = (ix == ix) ? __float2int_rd(fl) : -2;
  f = __fsub_rn(ix, fl);
}

// Row scheduling order.  Rows (b, q, h) are enumerated as (b, head-group,
// q, head-in-group) so CTAs that run at the same time share a small set of
// heads and therefore a smaller slice of `value` in L2.
struct RowCoord {
  int64_t b, q, h;
};
__device__ __forceinline__ RowCoord decode_row(uint32_t r, const Problem& p) {
  const uint32_t hg = static_cast<uint32_t>(p.hg);
  const uint32_t Q = static_cast<uint32_t>(p.Q);
  const uint32_t ngroups = static_cast<uint32_t>(p.H) / hg;
  const uint32_t hi = r % hg;
  uint32_t t = r / hg;
  const uint32_t q = t % Q;
  t /= Q;
  const uint32_t grp = t % ngroups;
  const uint32_t b = t / ngroups;
  RowCoord rc;
  rc.b = b;
  rc.q = q;
  rc.h = static_cast<int64_t>(grp) * hg + hi;
  return rc;
}

}  // namespace msda
