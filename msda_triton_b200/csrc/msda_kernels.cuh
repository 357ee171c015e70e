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

#include "msda_common.cuh"

namespace msda {

template <int NDIM>
struct Point {
  int32_t i0[3];
  float f[3];
  bool pass[3];
};

template <int NDIM>
__device__ __forceinline__ void corner_coords(const Point<NDIM>& pt, int c, const int32_t* sz,
                                              int32_t start, bool& valid, int32_t& key,
                                              float& w) {
  const int32_t xi = pt.i0[0] + (c & 1);
  const int32_t yi = pt.i0[1] + ((c >> 1) & 1);
  const int32_t zi = (NDIM == 3) ? pt.i0[2] + ((c >> 2) & 1) : 0;
  valid = static_cast<uint32_t>(xi) < static_cast<uint32_t>(sz[0]) &&
          static_cast<uint32_t>(yi) < static_cast<uint32_t>(sz[1]);
  if (NDIM == 3) valid = valid && static_cast<uint32_t>(zi) < static_cast<uint32_t>(sz[2]);
  key = start + (zi * sz[1] + yi) * sz[0] + xi;
  const float wx = (c & 1) ? pt.f[0] : __fsub_rn(1.0f, pt.f[0]);
  const float wy = (c & 2) ? pt.f[1] : __fsub_rn(1.0f, pt.f[1]);
  w = __fmul_rn(wx, wy);
  if (NDIM == 3) {
    const float wz = (c & 4) ? pt.f[2] : __fsub_rn(1.0f, pt.f[2]);
    w = __fmul_rn(w, wz);
  }
}

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

// ------------------------------------------------------------------ forward
template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads)
    msda_fwd_kernel(const Problem p, T* __restrict__ out) {
  __shared__ LevelSmem lv;
  load_levels(p, lv, NDIM);

  using CK = Chunk<T, VB>;
  constexpr int EPV = CK::EPV;
  constexpr int NC = 1 << NDIM;

  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const uint64_t r = tid >> p.log2g;
  const int G = 1 << p.log2g;
  const int j = static_cast<int>(tid & static_cast<uint64_t>(G - 1));
  if (r >= static_cast<uint64_t>(p.B * p.Q * p.H)) return;

  const RowCoord rc = decode_row(static_cast<uint32_t>(r), p);
  const int64_t row = (rc.b * p.Q + rc.q) * p.H + rc.h;
  const int64_t key_bytes = p.H * p.C * static_cast<int64_t>(sizeof(T));
  const char* vbase = static_cast<const char*>(p.value) +
                      (rc.b * p.K * p.H + rc.h) * p.C * static_cast<int64_t>(sizeof(T));
  const int LP = static_cast<int>(p.L * p.P);
  const TS* lrow = static_cast<const TS*>(p.loc) + row * LP * NDIM;
  const TS* arow = static_cast<const TS*>(p.attn) + row * LP;

  int off[VPL];
  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int chunk = j + v * G;
    has[v] = chunk < p.nv;
    off[v] = chunk * VB;
  }

  float acc[VPL][EPV];
#pragma unroll
  for (int v = 0; v < VPL; ++v)
#pragma unroll
    for (int e = 0; e < EPV; ++e) acc[v][e] = 0.0f;

  for (int l = 0; l < p.L; ++l) {
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int32_t start = lv.start[l];
    for (int pp = 0; pp < p.P; ++pp) {
      const int s = l * static_cast<int>(p.P) + pp;
      const Point<NDIM> pt = load_point<TS, NDIM>(lrow + s * NDIM, sz, p);
      const float a = Elem<TS>::to_f(arow[s]);

      Raw<VB> raw[NC][VPL];
      float cw[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        bool valid;
        int32_t key;
        float w;
        corner_coords<NDIM>(pt, c, sz, start, valid, key, w);
        cw[c] = valid ? a * w : 0.0f;
        const char* kp = vbase + static_cast<int64_t>(key) * key_bytes;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          raw[c][v] = (valid && has[v]) ? ld_chunk<VB>(kp + off[v]) : raw_zero<VB>();
      }
#pragma unroll
      for (int c = 0; c < NC; ++c) {
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          float x[EPV];
          CK::unpack(raw[c][v], x);
#pragma unroll
          for (int e = 0; e < EPV; ++e) acc[v][e] = fmaf(cw[c], x[e], acc[v][e]);
        }
      }
    }
  }

  char* orow = reinterpret_cast<char*>(out) + row * p.C * static_cast<int64_t>(sizeof(T));
#pragma unroll
  for (int v = 0; v < VPL; ++v)
    if (has[v]) st_chunk<VB>(orow + off[v], CK::pack(acc[v]));
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

// One pass produces all three gradients.  grad_out is read once per row
// (the reference re-reads it for every (level, point), msda_3d.py:451-455).
// grad_loc and grad_attn are reduced inside the lane group with shuffles and
// written with plain stores by the group's first lane (one owner per sample:
// no atomics and no zero-fill).  grad_value is scattered with vector fp32
// reductions into `gacc` (grad_value itself for fp32, else an fp32 workspace
// that msda_cast_kernel rounds to the input dtype).
template <typename T, typename TS, int NDIM, int VB, int VPL>
__global__ void __launch_bounds__(kThreads)
    msda_bwd_kernel(const Problem p, const T* __restrict__ grad_out, float* __restrict__ gacc,
                    TS* __restrict__ grad_loc, TS* __restrict__ grad_attn) {
  __shared__ LevelSmem lv;
  load_levels(p, lv, NDIM);

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
  const int64_t HC = p.H * p.C;
  const int64_t key_bytes = HC * static_cast<int64_t>(sizeof(T));
  const char* vbase = static_cast<const char*>(p.value) +
                      (rc.b * p.K * p.H + rc.h) * p.C * static_cast<int64_t>(sizeof(T));
  float* gbase = gacc + (rc.b * p.K * p.H + rc.h) * p.C;
  const int LP = static_cast<int>(p.L * p.P);
  const TS* lrow = static_cast<const TS*>(p.loc) + row * LP * NDIM;
  const TS* arow = static_cast<const TS*>(p.attn) + row * LP;

  int chunk[VPL];
  bool has[VPL];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    chunk[v] = j + v * G;
    has[v] = active && chunk[v] < p.nv;
  }

  float go[VPL][EPV];
  const char* gorow = reinterpret_cast<const char*>(grad_out) +
                      row * p.C * static_cast<int64_t>(sizeof(T));
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const Raw<VB> rg = has[v] ? ld_chunk<VB>(gorow + chunk[v] * VB) : raw_zero<VB>();
    CK::unpack(rg, go[v]);
  }

  for (int l = 0; l < p.L; ++l) {
    const int32_t sz[3] = {lv.size[l][0], lv.size[l][1], lv.size[l][2]};
    const int32_t start = lv.start[l];
    for (int pp = 0; pp < p.P; ++pp) {
      const int s = l * static_cast<int>(p.P) + pp;
      Point<NDIM> pt;
      float a = 0.0f;
      if (active) {
        pt = load_point<TS, NDIM>(lrow + s * NDIM, sz, p);
        a = Elem<TS>::to_f(arow[s]);
      } else {
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) {
          pt.i0[ax] = -2;
          pt.f[ax] = 0.0f;
          pt.pass[ax] = false;
        }
      }

      Raw<VB> raw[NC][VPL];
      bool cvalid[NC];
      int32_t ckey[NC];
      float cw[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        corner_coords<NDIM>(pt, c, sz, start, cvalid[c], ckey[c], cw[c]);
        const char* kp = vbase + static_cast<int64_t>(ckey[c]) * key_bytes;
#pragma unroll
        for (int v = 0; v < VPL; ++v)
          raw[c][v] = (cvalid[c] && has[v]) ? ld_chunk<VB>(kp + chunk[v] * VB)
                                            : raw_zero<VB>();
      }

      float g_attn = 0.0f;
      float g_ix[3] = {0.0f, 0.0f, 0.0f};
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
        float dw[3];
        corner_dweights<NDIM>(pt, c, dw);
        g_attn = fmaf(cw[c], dot, g_attn);
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) g_ix[ax] = fmaf(dw[ax], dot, g_ix[ax]);

        if (cvalid[c]) {
          const float aw = a * cw[c];
          float* gk = gbase + static_cast<int64_t>(ckey[c]) * HC;
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            if (has[v]) {
              float t[EPV];
#pragma unroll
              for (int e = 0; e < EPV; ++e) t[e] = aw * go[v][e];
              red_add_f32<EPV>(gk + chunk[v] * EPV, t);
            }
          }
        }
      }

      // Reduce the per-sample scalars over the G lanes of the group.
      for (int o = G >> 1; o > 0; o >>= 1) {
        g_attn += __shfl_xor_sync(0xffffffffu, g_attn, o);
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) g_ix[ax] += __shfl_xor_sync(0xffffffffu, g_ix[ax], o);
      }
      if (active && j == 0) {
        grad_attn[row * LP + s] = Elem<TS>::from_f(g_attn);
        TS* gl = grad_loc + (row * LP + s) * NDIM;
#pragma unroll
        for (int ax = 0; ax < NDIM; ++ax) {
          const float gval = a * g_ix[ax] * static_cast<float>(sz[ax]);
          gl[ax] = Elem<TS>::from_f(pt.pass[ax] ? gval : 0.0f);
        }
      }
    }
  }
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

}  // namespace msda
