// msda_prologue.cu -- the modules' sampling prologue as its own pass (see
// msda_prologue.cuh): a CTA per block of (b, q, h) rows.  Offsets and
// location gradients move as 16-byte vectors; logits, weights and their
// gradients are staged in shared memory for the per-row softmax.
//
// Locations follow the rounding of the reference's separate expression
// `reference_points + sampling_offsets / normalizer` in the sampling dtype:
// the integer size is converted to that dtype, the quotient (correctly
// rounded division) is rounded to it, then the sum.  The weights use the
// fused kernels' row softmax (row_softmax), so the large and the small
// module path agree.
#include "msda_prologue.cuh"

#include "msda_b200.h"
#include <algorithm>

#include "msda_kernels.cuh"

namespace msda {

template <typename TS>
__device__ __forceinline__ float round_to(float x) {
  return Elem<TS>::to_f(Elem<TS>::from_f(x));
}

// n / d for 0 <= n < 2^31 as a multiply and shift (m = ceil(2^(31+l) / d),
// l = ceil(log2 d): the rounding error stays below 1/d).
struct PDiv {
  uint32_t m, s;
};
static PDiv pdiv(uint32_t d) {
  if (d == 0) d = 1;
  uint32_t l = 0;
  while ((uint64_t{1} << l) < d) ++l;
  return PDiv{static_cast<uint32_t>(((uint64_t{1} << (31 + l)) + d - 1) / d), 31 + l};
}
__device__ __forceinline__ uint32_t pd(uint32_t n, const PDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(n) * f.m) >> f.s);
}

// Per launch: rows per CTA, row lengths and their dividers.
struct PrologueShape {
  int32_t R;            // rows (b, q, h) per CTA: a multiple of 8 when the copies are vectors
  int32_t RL, LP, Pd;   // elements per row (L*P*d), samples per row, elements per level (P*d)
  int32_t LPs;          // shared-memory row stride of the weights, in elements: an odd number of words
  PDiv dRL, dPd, dd, dH, dLP;
};

// Each level's size per axis in the sampling dtype (the tensor expression
// converts the integer normalizer to it) and its reciprocal.
template <typename TS, int NDIM>
__device__ __forceinline__ void stage_sizes(const PrologueArgs& a, float* s_n, float* s_r) {
  for (int i = threadIdx.x; i < a.L * NDIM; i += kThreads) {
    const int l = i / NDIM, ax = i - l * NDIM;
    const float n = round_to<TS>(static_cast<float>(a.size[l][ax]));
    s_n[i] = n;
    s_r[i] = __frcp_rn(n);
  }
}

// x / n rounded to the nearest float.  Normal operands take the reciprocal
// and one FMA correction (div_by_size, exact for them); zeros, subnormals,
// infinities, NaNs and a zero size take the IEEE division itself.
__device__ __forceinline__ float size_div(float x, float n, float r) {
  const float ax = fabsf(x);
  return (ax >= 0x1p-100f && ax <= 0x1.fffffep127f && n >= 1.0f && n < 0x1p24f)
             ? div_by_size(x, n, r) : __fdiv_rn(x, n);
}

// n contiguous elements of R rows of LP from global memory into a shared
// tile with row stride LPs (and back): 16-byte vectors on the global side
// when VEC, the shared side element by element.
template <typename TS, bool VEC>
__device__ __forceinline__ void rows_in(TS* s, const TS* g, int n, int LP, int LPs, const PDiv& dLP) {
  constexpr int V = VEC ? 16 / static_cast<int>(sizeof(TS)) : 1;
  for (int e = threadIdx.x * V; e < n; e += kThreads * V) {
    alignas(16) TS x[V];
    if (VEC && e + V <= n) *reinterpret_cast<uint4*>(x) = *reinterpret_cast<const uint4*>(g + e);
    else for (int j = 0; j < V; ++j) if (e + j < n) x[j] = g[e + j];
    int r = static_cast<int>(pd(static_cast<uint32_t>(e), dLP));
    int c = e - r * LP;
    for (int j = 0; j < V && e + j < n; ++j) {
      s[r * LPs + c] = x[j];
      if (++c == LP) c = 0, ++r;
    }
  }
}
template <typename TS, bool VEC>
__device__ __forceinline__ void rows_out(TS* g, const TS* s, int n, int LP, int LPs, const PDiv& dLP) {
  constexpr int V = VEC ? 16 / static_cast<int>(sizeof(TS)) : 1;
  for (int e = threadIdx.x * V; e < n; e += kThreads * V) {
    alignas(16) TS x[V];
    int r = static_cast<int>(pd(static_cast<uint32_t>(e), dLP));
    int c = e - r * LP;
    for (int j = 0; j < V && e + j < n; ++j) {
      x[j] = s[r * LPs + c];
      if (++c == LP) c = 0, ++r;
    }
    if (VEC && e + V <= n) *reinterpret_cast<uint4*>(g + e) = *reinterpret_cast<const uint4*>(x);
    else for (int j = 0; j < V; ++j) if (e + j < n) g[e + j] = x[j];
  }
}

// Where element e of a CTA's row tile lies: row, level, element within the
// level, axis.  Advanced element by element with step().
struct ElemPos {
  int row, l, k, ax;
};
template <int NDIM>
__device__ __forceinline__ ElemPos elem_pos(int e, const PrologueShape& sh) {
  ElemPos p;
  p.row = static_cast<int>(pd(static_cast<uint32_t>(e), sh.dRL));
  const int w = e - p.row * sh.RL;
  p.l = static_cast<int>(pd(static_cast<uint32_t>(w), sh.dPd));
  p.k = w - p.l * sh.Pd;
  p.ax = p.k - static_cast<int>(pd(static_cast<uint32_t>(p.k), sh.dd)) * NDIM;
  return p;
}
// Returns true when the step enters the next row.
template <int NDIM>
__device__ __forceinline__ bool step(ElemPos& p, int L, const PrologueShape& sh) {
  if (++p.ax == NDIM) p.ax = 0;
  if (++p.k == sh.Pd) {
    p.k = 0;
    if (++p.l == L) {
      p.l = 0;
      ++p.row;
      return true;
    }
  }
  return false;
}

// One CTA per R consecutive rows.  Locations: V consecutive offsets per
// thread straight from global memory (16-byte vectors when VEC), the level
// and axis tracked element by element.  Weights: the rows' logits
// staged in shared memory (odd word stride, so one thread per row reads
// without bank conflicts), the fused kernels' row softmax in place, copied
// back out.
template <typename TS, int NDIM, bool VEC>
__global__ void __launch_bounds__(kThreads)
    msda_prologue_fwd_kernel(const PrologueArgs a, const PrologueShape sh) {
  extern __shared__ __align__(16) unsigned char psm[];
  __shared__ float s_n[kMaxLevels * 3], s_r[kMaxLevels * 3];
  constexpr int V = VEC ? 16 / static_cast<int>(sizeof(TS)) : 1;
  const int64_t rows = a.B * a.Q * a.H;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * sh.R;
  const int nr = static_cast<int>(min(static_cast<int64_t>(sh.R), rows - row0));
  const int L = static_cast<int>(a.L);
  TS* s_lg = reinterpret_cast<TS*>(psm);  // R * LPs
  stage_sizes<TS, NDIM>(a, s_n, s_r);
  rows_in<TS, VEC>(s_lg, static_cast<const TS*>(a.logits) + row0 * sh.LP, nr * sh.LP, sh.LP,
                   sh.LPs, sh.dLP);
  __syncthreads();
  // locations
  const TS* ref = static_cast<const TS*>(a.ref);
  const TS* off = static_cast<const TS*>(a.off) + row0 * sh.RL;
  TS* loc = static_cast<TS*>(a.loc) + row0 * sh.RL;
  const int ne = nr * sh.RL;
  for (int e = threadIdx.x * V; e < ne; e += kThreads * V) {
    alignas(16) TS x[V];
    const bool full = e + V <= ne;
    if (VEC && full) *reinterpret_cast<uint4*>(x) = *reinterpret_cast<const uint4*>(off + e);
    else for (int j = 0; j < V; ++j) if (e + j < ne) x[j] = off[e + j];
    ElemPos p = elem_pos<NDIM>(e, sh);
    const TS* rrow = ref + static_cast<int64_t>(pd(static_cast<uint32_t>(row0 + p.row), sh.dH)) * L * NDIM;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (e + j < ne) {
        const int li = p.l * NDIM + p.ax;
        const float q = round_to<TS>(size_div(Elem<TS>::to_f(x[j]), s_n[li], s_r[li]));
        x[j] = Elem<TS>::from_f(__fadd_rn(Elem<TS>::to_f(rrow[li]), q));
        if (step<NDIM>(p, L, sh))
          rrow = ref + static_cast<int64_t>(pd(static_cast<uint32_t>(row0 + p.row), sh.dH)) * L * NDIM;
      }
    }
    if (VEC && full) *reinterpret_cast<uint4*>(loc + e) = *reinterpret_cast<const uint4*>(x);
    else for (int j = 0; j < V; ++j) if (e + j < ne) loc[e + j] = x[j];
  }
  // weights: one thread per row, in place
  if (threadIdx.x < nr) {
    TS* r = s_lg + threadIdx.x * sh.LPs;
    const RowSoftmax sm = row_softmax<TS>(r, sh.LP, 0, 1);
    for (int i = 0; i < sh.LP; ++i) r[i] = Elem<TS>::from_f(softmax_weight(Elem<TS>::to_f(r[i]), sm));
  }
  __syncthreads();
  rows_out<TS, VEC>(static_cast<TS*>(a.wout) + row0 * sh.LP, s_lg, nr * sh.LP, sh.LP, sh.LPs, sh.dLP);
}

// One CTA per R consecutive rows.  The location gradients are copied into
// shared memory as they lie (16-byte vectors when VEC); the weights and
// their gradients into rows of odd word stride.  Offset gradients (g / size)
// go out V elements per thread; the reference-point gradient is summed over
// each row's points per (level, axis); the softmax backward runs one thread
// per row in place.
template <typename TS, int NDIM, bool VEC>
__global__ void __launch_bounds__(kThreads)
    msda_prologue_bwd_kernel(const PrologueArgs a, const PrologueShape sh) {
  extern __shared__ __align__(16) unsigned char psm[];
  __shared__ float s_n[kMaxLevels * 3], s_r[kMaxLevels * 3];
  constexpr int V = VEC ? 16 / static_cast<int>(sizeof(TS)) : 1;
  const int64_t rows = a.B * a.Q * a.H;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * sh.R;
  const int nr = static_cast<int>(min(static_cast<int64_t>(sh.R), rows - row0));
  const int L = static_cast<int>(a.L);
  TS* s_gl = reinterpret_cast<TS*>(psm);  // R * RL
  TS* s_w = s_gl + sh.R * sh.RL;           // R * LPs
  TS* s_ga = s_w + sh.R * sh.LPs;          // R * LPs
  stage_sizes<TS, NDIM>(a, s_n, s_r);
  const int ne = nr * sh.RL;
  const TS* gl = static_cast<const TS*>(a.gloc) + row0 * sh.RL;
  for (int e = threadIdx.x * V; e < ne; e += kThreads * V) {
    if (VEC && e + V <= ne) *reinterpret_cast<uint4*>(s_gl + e) = *reinterpret_cast<const uint4*>(gl + e);
    else for (int j = 0; j < V; ++j) if (e + j < ne) s_gl[e + j] = gl[e + j];
  }
  rows_in<TS, VEC>(s_w, static_cast<const TS*>(a.weights) + row0 * sh.LP, nr * sh.LP, sh.LP, sh.LPs,
                   sh.dLP);
  rows_in<TS, VEC>(s_ga, static_cast<const TS*>(a.gattn) + row0 * sh.LP, nr * sh.LP, sh.LP, sh.LPs,
                   sh.dLP);
  __syncthreads();
  // offsets: grad / size
  TS* go = static_cast<TS*>(a.goff) + row0 * sh.RL;
  for (int e = threadIdx.x * V; e < ne; e += kThreads * V) {
    alignas(16) TS x[V];
    const bool full = e + V <= ne;
    if (VEC && full) *reinterpret_cast<uint4*>(x) = *reinterpret_cast<const uint4*>(s_gl + e);
    else for (int j = 0; j < V; ++j) if (e + j < ne) x[j] = s_gl[e + j];
    ElemPos p = elem_pos<NDIM>(e, sh);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (e + j < ne) {
        const int li = p.l * NDIM + p.ax;
        x[j] = Elem<TS>::from_f(size_div(Elem<TS>::to_f(x[j]), s_n[li], s_r[li]));
        step<NDIM>(p, L, sh);
      }
    }
    if (VEC && full) *reinterpret_cast<uint4*>(go + e) = *reinterpret_cast<const uint4*>(x);
    else for (int j = 0; j < V; ++j) if (e + j < ne) go[e + j] = x[j];
  }
  // reference points: the sum over the row's points, (row, l, axis) outputs
  const int LD = L * NDIM;
  float* gr = a.gref_partial + row0 * LD;
  const int P = static_cast<int>(a.P);
  for (int i = threadIdx.x; i < nr * LD; i += kThreads) {
    const int lr = i / LD, k = i - lr * LD, l = k / NDIM, ax = k - l * NDIM;
    const TS* src = s_gl + lr * sh.RL + l * sh.Pd + ax;
    float acc = 0.0f;
    for (int pt = 0; pt < P; ++pt) acc += Elem<TS>::to_f(src[pt * NDIM]);
    gr[i] = acc;
  }
  // logits: softmax backward g = w * (dL/dw - sum_j w_j dL/dw_j), one thread per row, in place
  if (threadIdx.x < nr) {
    const TS* wr = s_w + threadIdx.x * sh.LPs;
    TS* gr2 = s_ga + threadIdx.x * sh.LPs;
    float dot = 0.0f;
    for (int i = 0; i < sh.LP; ++i) dot = fmaf(Elem<TS>::to_f(wr[i]), Elem<TS>::to_f(gr2[i]), dot);
    for (int i = 0; i < sh.LP; ++i)
      gr2[i] = Elem<TS>::from_f(Elem<TS>::to_f(wr[i]) * (Elem<TS>::to_f(gr2[i]) - dot));
  }
  __syncthreads();
  rows_out<TS, VEC>(static_cast<TS*>(a.glogits) + row0 * sh.LP, s_ga, nr * sh.LP, sh.LP, sh.LPs,
                    sh.dLP);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename TS, int NDIM, bool VEC>
static void launch_kernel(const PrologueArgs& a, const PrologueShape& sh, bool bwd, dim3 grid,
                          size_t smem, cudaStream_t st) {
  if (bwd) msda_prologue_bwd_kernel<TS, NDIM, VEC><<<grid, kThreads, smem, st>>>(a, sh);
  else msda_prologue_fwd_kernel<TS, NDIM, VEC><<<grid, kThreads, smem, st>>>(a, sh);
}

template <typename TS>
static cudaError_t launch_one(const PrologueArgs& a, bool bwd, cudaStream_t st) {
  const int64_t rows = a.B * a.Q * a.H;
  if (rows == 0) return cudaSuccess;
  PrologueShape sh;
  sh.LP = static_cast<int32_t>(a.L * a.P);
  sh.Pd = static_cast<int32_t>(a.P * a.ndim);
  sh.RL = sh.LP * a.ndim;
  // weight rows padded to an odd number of 32-bit words
  int32_t words = static_cast<int32_t>((int64_t{sh.LP} * sizeof(TS) + 3) / 4);
  if (words % 2 == 0) ++words;
  sh.LPs = static_cast<int32_t>(words * 4 / sizeof(TS));
  // rows per CTA: up to kThreads (one thread per row in the softmax), within
  // 47 KB of dynamic shared memory (the static size tables take the rest of
  // 48 KB), a multiple of 8 (16-byte aligned row tiles).  The entry points
  // cap L*P at 2048, so one row always fits.
  const int64_t row_bytes =
      (bwd ? int64_t{sh.RL} + 2 * int64_t{sh.LPs} : int64_t{sh.LPs}) * int64_t{sizeof(TS)};
  int64_t R = std::max<int64_t>(1, std::min<int64_t>(kThreads, 47 * 1024 / row_bytes));
  if (R >= 8) R -= R % 8;
  sh.R = static_cast<int32_t>(R);
  sh.dRL = pdiv(static_cast<uint32_t>(sh.RL));
  sh.dPd = pdiv(static_cast<uint32_t>(sh.Pd));
  sh.dd = pdiv(static_cast<uint32_t>(a.ndim));
  sh.dH = pdiv(static_cast<uint32_t>(a.H));
  sh.dLP = pdiv(static_cast<uint32_t>(sh.LP));
  const bool vec = R % 8 == 0 &&
                   (bwd ? aligned16(a.gloc) && aligned16(a.goff) && aligned16(a.weights) &&
                              aligned16(a.gattn) && aligned16(a.glogits)
                        : aligned16(a.off) && aligned16(a.loc) && aligned16(a.logits) &&
                              aligned16(a.wout));
  const size_t smem = static_cast<size_t>(R * row_bytes);
  const dim3 grid(static_cast<unsigned>((rows + R - 1) / R));
  if (a.ndim == 3) {
    if (vec) launch_kernel<TS, 3, true>(a, sh, bwd, grid, smem, st);
    else launch_kernel<TS, 3, false>(a, sh, bwd, grid, smem, st);
  } else {
    if (vec) launch_kernel<TS, 2, true>(a, sh, bwd, grid, smem, st);
    else launch_kernel<TS, 2, false>(a, sh, bwd, grid, smem, st);
  }
  return cudaGetLastError();
}

static cudaError_t launch(const PrologueArgs& a, int dtype, bool bwd, cudaStream_t st) {
  switch (dtype) {
    case MSDA_FLOAT32: return launch_one<float>(a, bwd, st);
    case MSDA_FLOAT16: return launch_one<__half>(a, bwd, st);
    case MSDA_BFLOAT16: return launch_one<__nv_bfloat16>(a, bwd, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prologue_fwd(const PrologueArgs& a, int dtype, cudaStream_t st) {
  return launch(a, dtype, false, st);
}
cudaError_t prologue_bwd(const PrologueArgs& a, int dtype, cudaStream_t st) {
  return launch(a, dtype, true, st);
}

}  // namespace msda
