// msda_prologue.cu -- the modules' sampling prologue as its own pass (see
// msda_prologue.cuh): a CTA per block of (b, q, h) rows, staged through
// shared memory.
//
// Locations follow the rounding of the reference's separate expression
// `reference_points + sampling_offsets / normalizer` in the sampling dtype:
// the integer size is converted to that dtype, the quotient (IEEE division)
// is rounded to it, then the sum.  The weights use the fused kernels' row
// softmax (row_softmax), so the large and the small module path agree.
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
  int32_t R;            // rows (b, q, h) per CTA
  int32_t RL, LP, Pd;   // elements per row (L*P*d), samples per row, elements per level (P*d)
  PDiv dRL, dPd, dd, dH;
};

// One CTA per R consecutive rows: the rows' offsets (or location gradients)
// and logits (or weights and their gradients) are contiguous blocks, copied
// in and out of shared memory with consecutive threads on consecutive
// elements; the per-element work reads shared memory, the row softmax (one
// thread per row) too.
template <typename TS, int NDIM>
__global__ void __launch_bounds__(kThreads)
    msda_prologue_fwd_kernel(const PrologueArgs a, const PrologueShape sh) {
  extern __shared__ __align__(16) unsigned char psm[];
  const int64_t rows = a.B * a.Q * a.H;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * sh.R;
  const int nr = static_cast<int>(min(static_cast<int64_t>(sh.R), rows - row0));
  TS* s_off = reinterpret_cast<TS*>(psm);          // R * RL
  TS* s_lg = s_off + sh.R * sh.RL;                 // R * LP
  const TS* off = static_cast<const TS*>(a.off) + row0 * sh.RL;
  const TS* lg = static_cast<const TS*>(a.logits) + row0 * sh.LP;
  for (int i = threadIdx.x; i < nr * sh.RL; i += kThreads) s_off[i] = off[i];
  for (int i = threadIdx.x; i < nr * sh.LP; i += kThreads) s_lg[i] = lg[i];
  __syncthreads();
  // locations, element-parallel
  const TS* ref = static_cast<const TS*>(a.ref);
  TS* loc = static_cast<TS*>(a.loc) + row0 * sh.RL;
  for (int i = threadIdx.x; i < nr * sh.RL; i += kThreads) {
    const uint32_t lr = pd(static_cast<uint32_t>(i), sh.dRL);
    const uint32_t w = static_cast<uint32_t>(i) - lr * static_cast<uint32_t>(sh.RL);
    const uint32_t l = pd(w, sh.dPd);
    const uint32_t ax = w - pd(w, sh.dd) * NDIM;
    const int64_t row = row0 + lr;
    const int64_t bq = pd(static_cast<uint32_t>(row), sh.dH);
    const float rf = Elem<TS>::to_f(ref[(bq * a.L + l) * NDIM + ax]);
    const float sz = round_to<TS>(static_cast<float>(a.size[l][ax]));
    const float t = round_to<TS>(__fdiv_rn(Elem<TS>::to_f(s_off[i]), sz));
    loc[i] = Elem<TS>::from_f(__fadd_rn(rf, t));
  }
  // weights: one thread per row, in place
  if (threadIdx.x < nr) {
    TS* r = s_lg + threadIdx.x * sh.LP;
    const RowSoftmax sm = row_softmax<TS>(r, sh.LP, 0, 1);
    for (int i = 0; i < sh.LP; ++i) r[i] = Elem<TS>::from_f(softmax_weight(Elem<TS>::to_f(r[i]), sm));
  }
  __syncthreads();
  TS* w = static_cast<TS*>(a.wout) + row0 * sh.LP;
  for (int i = threadIdx.x; i < nr * sh.LP; i += kThreads) w[i] = s_lg[i];
}

template <typename TS, int NDIM>
__global__ void __launch_bounds__(kThreads)
    msda_prologue_bwd_kernel(const PrologueArgs a, const PrologueShape sh) {
  extern __shared__ __align__(16) unsigned char psm[];
  const int64_t rows = a.B * a.Q * a.H;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * sh.R;
  const int nr = static_cast<int>(min(static_cast<int64_t>(sh.R), rows - row0));
  TS* s_gl = reinterpret_cast<TS*>(psm);           // R * RL
  TS* s_w = s_gl + sh.R * sh.RL;                   // R * LP
  TS* s_ga = s_w + sh.R * sh.LP;                   // R * LP
  const TS* gl = static_cast<const TS*>(a.gloc) + row0 * sh.RL;
  const TS* w = static_cast<const TS*>(a.weights) + row0 * sh.LP;
  const TS* ga = static_cast<const TS*>(a.gattn) + row0 * sh.LP;
  for (int i = threadIdx.x; i < nr * sh.RL; i += kThreads) s_gl[i] = gl[i];
  for (int i = threadIdx.x; i < nr * sh.LP; i += kThreads) {
    s_w[i] = w[i];
    s_ga[i] = ga[i];
  }
  __syncthreads();
  // offsets: grad / size, element-parallel
  TS* go = static_cast<TS*>(a.goff) + row0 * sh.RL;
  for (int i = threadIdx.x; i < nr * sh.RL; i += kThreads) {
    const uint32_t lr = pd(static_cast<uint32_t>(i), sh.dRL);
    const uint32_t wi = static_cast<uint32_t>(i) - lr * static_cast<uint32_t>(sh.RL);
    const uint32_t l = pd(wi, sh.dPd);
    const uint32_t ax = wi - pd(wi, sh.dd) * NDIM;
    const float sz = round_to<TS>(static_cast<float>(a.size[l][ax]));
    go[i] = Elem<TS>::from_f(__fdiv_rn(Elem<TS>::to_f(s_gl[i]), sz));
  }
  // reference points: the sum over the row's points, (row, l, axis) outputs
  const int LD = static_cast<int>(a.L) * NDIM;
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
    const TS* wr = s_w + threadIdx.x * sh.LP;
    TS* gr2 = s_ga + threadIdx.x * sh.LP;
    float dot = 0.0f;
    for (int i = 0; i < sh.LP; ++i) dot = fmaf(Elem<TS>::to_f(wr[i]), Elem<TS>::to_f(gr2[i]), dot);
    for (int i = 0; i < sh.LP; ++i)
      gr2[i] = Elem<TS>::from_f(Elem<TS>::to_f(wr[i]) * (Elem<TS>::to_f(gr2[i]) - dot));
  }
  __syncthreads();
  TS* glg = static_cast<TS*>(a.glogits) + row0 * sh.LP;
  for (int i = threadIdx.x; i < nr * sh.LP; i += kThreads) glg[i] = s_ga[i];
}

template <typename TS>
static cudaError_t launch_one(const PrologueArgs& a, bool bwd, cudaStream_t st) {
  const int64_t rows = a.B * a.Q * a.H;
  if (rows == 0) return cudaSuccess;
  PrologueShape sh;
  sh.LP = static_cast<int32_t>(a.L * a.P);
  sh.Pd = static_cast<int32_t>(a.P * a.ndim);
  sh.RL = sh.LP * a.ndim;
  // rows per CTA: up to kThreads, within 48 KB of shared memory
  const int64_t row_bytes = (int64_t{sh.RL} + (bwd ? 2 : 1) * sh.LP) * int64_t{sizeof(TS)};
  sh.R = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(kThreads, 48 * 1024 / row_bytes)));
  sh.dRL = pdiv(static_cast<uint32_t>(sh.RL));
  sh.dPd = pdiv(static_cast<uint32_t>(sh.Pd));
  sh.dd = pdiv(static_cast<uint32_t>(a.ndim));
  sh.dH = pdiv(static_cast<uint32_t>(a.H));
  const size_t smem = static_cast<size_t>(sh.R * row_bytes);
  const dim3 grid(static_cast<unsigned>((rows + sh.R - 1) / sh.R));
  if (bwd) {
    if (a.ndim == 3) msda_prologue_bwd_kernel<TS, 3><<<grid, kThreads, smem, st>>>(a, sh);
    else msda_prologue_bwd_kernel<TS, 2><<<grid, kThreads, smem, st>>>(a, sh);
  } else {
    if (a.ndim == 3) msda_prologue_fwd_kernel<TS, 3><<<grid, kThreads, smem, st>>>(a, sh);
    else msda_prologue_fwd_kernel<TS, 2><<<grid, kThreads, smem, st>>>(a, sh);
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
