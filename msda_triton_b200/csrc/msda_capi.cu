// msda_capi.cu -- the C ABI declared in include/msda_b200.h: argument
// validation, level-table resolution, launch-shape selection and dispatch.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>

#include "../../include/msda_b200.h"
#ifdef MSDA_CHECKED
#include "../../include/msda_b200_checked.h"
#endif
#include "msda_launch.cuh"
#include "msda_prologue.cuh"
#include "msda_sorted_launch.cuh"

namespace msda {

MSDA_DECLARE_PAIR(float, float)
MSDA_DECLARE_PAIR(__half, __half)
MSDA_DECLARE_PAIR(__half, float)
MSDA_DECLARE_PAIR(__nv_bfloat16, __nv_bfloat16)
MSDA_DECLARE_PAIR(__nv_bfloat16, float)
MSDA_DECLARE_SORTED(float, float)
MSDA_DECLARE_SORTED(__half, __half)
MSDA_DECLARE_SORTED(__half, float)
MSDA_DECLARE_SORTED(__nv_bfloat16, __nv_bfloat16)
MSDA_DECLARE_SORTED(__nv_bfloat16, float)

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return MSDA_SUCCESS;
}

int64_t dtype_bytes(int dt) {
  switch (dt) {
    case MSDA_FLOAT32: return 4;
    case MSDA_FLOAT16: return 2;
    case MSDA_BFLOAT16: return 2;
    default: return 0;
  }
}

const char* dtype_name(int dt) {
  switch (dt) {
    case MSDA_FLOAT32: return "float32";
    case MSDA_FLOAT16: return "float16";
    case MSDA_BFLOAT16: return "bfloat16";
    default: return "unknown";
  }
}

bool aligned(const void* p, int64_t a) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(a)) == 0;
}

#ifdef MSDA_CHECKED
// Checked build: the device word the kernels' bounds checks report into
// (Problem::check_flag), one per device, looked up once.
__device__ unsigned int g_check_word;
unsigned int* check_word() {
  static unsigned int* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (addr[dev] == nullptr) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_check_word) == cudaSuccess) addr[dev] = static_cast<unsigned int*>(a);
  }
  return addr[dev];
}
#endif

struct Args {
  int ndim;
  const void* value;
  int vdt;
  int64_t B, K, H, C;
  const int32_t* shapes;
  int shapes_dev;
  int64_t L;
  const void* loc;
  const void* attn;
  int sdt;
  int64_t Q, P;
  int clamp;
  double eps;
  // fused prologue: loc / attn are the raw offsets / logits, ref the fp32
  // reference points (B, Q, L, d)
  const float* ref = nullptr;
  int fused = 0;
  // keep the backward on the gather/scatter plan (the static-scratch entry:
  // its workspace bound was set for that plan)
  bool scatter_only = false;
  // value / grad_value laid out (B, H, K, C): MSDA_VALUE_HEAD_MAJOR was set in
  // the value dtype argument (with_layout strips it from vdt)
  bool hm = false;
};

Args with_layout(Args a) {
  a.hm = (a.vdt & MSDA_VALUE_HEAD_MAJOR) != 0;
  a.vdt &= ~MSDA_VALUE_HEAD_MAJOR;
  return a;
}

// Validate arguments, fill the Problem (except the launch shape) and pick
// the launch shape.  `bufs` are the row-strided buffers whose alignment bounds
// the chunk width (value, output / grad_out / grad_value).
int prepare(const Args& a, const void* const* bufs, int nbufs, Problem& p, LaunchShape& ls) {
  if (a.ndim != 2 && a.ndim != 3) return fail(MSDA_ERROR_INVALID_ARGUMENT, "ndim must be 2 or 3");
  const int64_t e = dtype_bytes(a.vdt);
  if (e == 0 || dtype_bytes(a.sdt) == 0)
    return fail(MSDA_ERROR_UNSUPPORTED_DTYPE,
                "MSDA only supports fp32, fp16, and bf16 (got value dtype code %d, sampling "
                "dtype code %d)", a.vdt, a.sdt);
  if (a.sdt != a.vdt && a.sdt != MSDA_FLOAT32)
    return fail(MSDA_ERROR_UNSUPPORTED_DTYPE,
                "sampling_locations/attention_weights dtype (%s) must equal the value dtype "
                "(%s) or be float32", dtype_name(a.sdt), dtype_name(a.vdt));
  if (a.B < 0 || a.K < 0 || a.H < 0 || a.C < 0 || a.L < 0 || a.Q < 0 || a.P < 0)
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "negative tensor dimension");
  if (a.L > kMaxLevels)
    return fail(MSDA_ERROR_TOO_MANY_LEVELS, "num_levels=%lld exceeds the supported maximum %d",
                static_cast<long long>(a.L), kMaxLevels);
  if (a.clamp && !(a.eps >= 0.0 && a.eps < 1.0))
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "clamp_eps must be in [0, 1), got %g", a.eps);
  if (a.K > INT32_MAX)
    return fail(MSDA_ERROR_INT32_OVERFLOW,
                "Total number of keys (%lld) exceeds int32 range. Reduce spatial dimensions or "
                "number of levels.", static_cast<long long>(a.K));
  const int64_t rows = a.B * a.Q * a.H;
  if (a.B != 0 && a.Q != 0 && a.H != 0 && rows / a.B / a.Q != a.H)
    return fail(MSDA_ERROR_INT32_OVERFLOW, "B*Q*H overflows");
  if (rows > INT32_MAX)
    return fail(MSDA_ERROR_INT32_OVERFLOW, "B*Q*H = %lld exceeds int32 range",
                static_cast<long long>(rows));
  if (a.L > 0 && a.shapes == nullptr)
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "spatial_shapes is NULL");

  std::memset(&p, 0, sizeof(p));
  p.value = a.value;
  p.loc = a.loc;
  p.attn = a.attn;
  p.B = a.B; p.K = a.K; p.H = a.H; p.C = a.C; p.Q = a.Q; p.L = a.L; p.P = a.P;
  p.acc_keys = a.K;  // accumulator in value's key layout unless a plan compacts it
  p.clamp = a.clamp ? 1 : 0;
  p.head_major = a.hm ? 1 : 0;
  p.lo = static_cast<float>(-1.0 + a.eps);
  p.hi = static_cast<float>(1.0 - a.eps);
  p.shapes_dev = nullptr;
#ifdef MSDA_CHECKED
  p.check_flag = check_word();
  if (p.check_flag == nullptr)
    return fail(MSDA_ERROR_CUDA, "checked build: bounds-check word not available");
#endif
  if (a.shapes_dev) {
    p.shapes_dev = a.shapes;
  } else {
    int64_t start = 0;
    for (int64_t l = 0; l < a.L; ++l) {
      int64_t n = 1;
      for (int ax = 0; ax < a.ndim; ++ax) {
        const int64_t v = a.shapes[l * a.ndim + (a.ndim - 1 - ax)];
        if (v < 0) return fail(MSDA_ERROR_INVALID_ARGUMENT, "negative spatial shape at level %lld",
                               static_cast<long long>(l));
        p.lv.size[l][ax] = static_cast<int32_t>(v);
        n *= v;
        if (n > INT32_MAX)
          return fail(MSDA_ERROR_INT32_OVERFLOW, "level %lld has more than 2^31-1 keys",
                      static_cast<long long>(l));
      }
      if (a.ndim == 2) p.lv.size[l][2] = 1;
      p.lv.start[l] = static_cast<int32_t>(start);
      start += n;
      if (start > INT32_MAX)
        return fail(MSDA_ERROR_INT32_OVERFLOW,
                    "Total number of keys (%lld) exceeds int32 range. Reduce spatial dimensions "
                    "or number of levels.", static_cast<long long>(start));
    }
    if (start != a.K)
      return fail(MSDA_ERROR_SHAPE_MISMATCH,
                  "value dim 1 (%lld) does not match sum of spatial shapes (%lld).",
                  static_cast<long long>(a.K), static_cast<long long>(start));
  }

  // Pointer checks: element alignment everywhere.
  const int64_t se = dtype_bytes(a.sdt);
  if (!aligned(a.value, e) || !aligned(a.loc, se) || !aligned(a.attn, se))
    return fail(MSDA_ERROR_MISALIGNED, "input buffers must be aligned to their element size");
  for (int i = 0; i < nbufs; ++i)
    if (!aligned(bufs[i], e))
      return fail(MSDA_ERROR_MISALIGNED, "output buffers must be aligned to their element size");

  // Chunk width: the widest of 16/4/2 bytes that divides the row and every
  // row-strided buffer's alignment.
  const int64_t row_bytes = a.C * e;
  int vb = 0;
  const int cands[3] = {16, 4, 2};
  for (int ci = 0; ci < 3 && vb == 0; ++ci) {
    const int c = cands[ci];
    if (c < e || row_bytes % c != 0) continue;
    bool al = aligned(a.value, c);
    for (int i = 0; i < nbufs; ++i) al = al && aligned(bufs[i], c);
    if (al) vb = c;
  }
  if (vb == 0) vb = static_cast<int>(e);  // e divides everything already checked
  const int64_t nv = row_bytes / vb;
  int vpl;
  if (vb == 16) {
    vpl = nv <= 32 ? 1 : nv <= 64 ? 2 : nv <= 128 ? 4 : 0;
  } else {
    vpl = nv <= 32 ? 1 : nv <= 256 ? 8 : 0;
  }
  if (vpl == 0)
    return fail(MSDA_ERROR_UNSUPPORTED_CHANNELS,
                "channels per head C=%lld (%lld bytes) exceeds the supported row size",
                static_cast<long long>(a.C), static_cast<long long>(row_bytes));
  int64_t lanes = (nv + vpl - 1) / vpl;
  int log2g = 0;
  while ((int64_t{1} << log2g) < lanes) ++log2g;
  p.nv = static_cast<int32_t>(nv);
  p.log2g = log2g;

  // Heads per scheduling group: the largest divisor of H whose value slice
  // (K * hg * C * e bytes) stays within a budget that leaves L2 room for the
  // streamed inputs.  MSDA_HEAD_GROUP overrides (tuning).
  int64_t hg = a.H > 0 ? a.H : 1;
  const char* env = std::getenv("MSDA_HEAD_GROUP");
  int64_t forced = env ? std::atoll(env) : 0;
  if (forced > 0 && a.H % forced == 0) {
    hg = forced;
  } else if (a.H > 0) {
    const int64_t budget = int64_t{48} << 20;
    for (hg = a.H; hg > 1; --hg)
      if (a.H % hg == 0 && a.K * hg * row_bytes <= budget) break;
    // At least the heads that share a 128-byte line (channel-last rows of
    // fewer than 128 bytes): a line fetched for one head then serves its
    // neighbours in the same pass, and the set of lines in use is the same.
    // Measured on 3D xl bf16 (64-byte rows, B=8): groups of 2 take the
    // forward from 5.94 to 5.78 ms and the dot-product kernel from 5.19 to
    // 4.88 ms; groups of 4 or 8 are slower (6.60 / 7.58 ms forward).
    if (!a.hm && row_bytes < 128) {
      int64_t lf = 128 / row_bytes;
      while (lf > 1 && a.H % lf != 0) --lf;
      if (lf > hg) hg = lf;
    }
  }
  p.hg = static_cast<int32_t>(hg);

  ls.ndim = a.ndim;
  ls.vb = vb;
  ls.vpl = vpl;
  const int64_t threads = rows << log2g;
  ls.grid = (threads + kThreads - 1) / kThreads;
  return MSDA_SUCCESS;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(MSDA_ERROR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

// Zero keys [start, start + nkeys) of every (batch entry[, head]) of a buffer
// in value's layout (elem_bytes per element, K keys per batch entry).
cudaError_t zero_key_range(const Args& a, void* base, int64_t start, int64_t nkeys, int64_t nb,
                           int64_t elem_bytes, cudaStream_t st) {
  if (nkeys <= 0 || nb <= 0) return cudaSuccess;
  const int64_t run = (a.hm ? a.C : a.H * a.C) * elem_bytes;  // bytes per key of one span
  const int64_t spans = a.hm ? nb * a.H : nb;
  return cudaMemset2DAsync(static_cast<char*>(base) + start * run,
                           static_cast<size_t>(a.K * run), 0, static_cast<size_t>(nkeys * run),
                           static_cast<size_t>(spans), st);
}

template <bool F>
cudaError_t dispatch_fwd_mode(int vdt, int sdt, const LaunchShape& ls, const Problem& p,
                              void* out, cudaStream_t st) {
  switch (vdt) {
    case MSDA_FLOAT32: return launch_fwd<float, float, F>(ls, p, out, st);
    case MSDA_FLOAT16:
      return sdt == MSDA_FLOAT32 ? launch_fwd<__half, float, F>(ls, p, out, st)
                                 : launch_fwd<__half, __half, F>(ls, p, out, st);
    default:
      return sdt == MSDA_FLOAT32 ? launch_fwd<__nv_bfloat16, float, F>(ls, p, out, st)
                                 : launch_fwd<__nv_bfloat16, __nv_bfloat16, F>(ls, p, out, st);
  }
}

cudaError_t dispatch_fwd(const Args& a, const LaunchShape& ls, const Problem& p, void* out,
                         cudaStream_t st) {
  return a.fused ? dispatch_fwd_mode<true>(a.vdt, a.sdt, ls, p, out, st)
                 : dispatch_fwd_mode<false>(a.vdt, a.sdt, ls, p, out, st);
}

template <bool F>
cudaError_t dispatch_bwd_mode(int vdt, int sdt, const LaunchShape& ls, const Problem& p,
                              const void* go, float* gacc, void* gl, void* ga, cudaStream_t st) {
  switch (vdt) {
    case MSDA_FLOAT32: return launch_bwd<float, float, F>(ls, p, go, gacc, gl, ga, st);
    case MSDA_FLOAT16:
      return sdt == MSDA_FLOAT32 ? launch_bwd<__half, float, F>(ls, p, go, gacc, gl, ga, st)
                                 : launch_bwd<__half, __half, F>(ls, p, go, gacc, gl, ga, st);
    default:
      return sdt == MSDA_FLOAT32
                 ? launch_bwd<__nv_bfloat16, float, F>(ls, p, go, gacc, gl, ga, st)
                 : launch_bwd<__nv_bfloat16, __nv_bfloat16, F>(ls, p, go, gacc, gl, ga, st);
  }
}

cudaError_t dispatch_bwd(const Args& a, const LaunchShape& ls, const Problem& p, const void* go,
                         float* gacc, void* gl, void* ga, cudaStream_t st) {
  return a.fused ? dispatch_bwd_mode<true>(a.vdt, a.sdt, ls, p, go, gacc, gl, ga, st)
                 : dispatch_bwd_mode<false>(a.vdt, a.sdt, ls, p, go, gacc, gl, ga, st);
}

// Fused prologue: the reference points are read by every row.
int check_fused(const Args& a) {
  if (!a.fused) return MSDA_SUCCESS;
  if (a.B * a.Q * a.H * a.L * a.P > 0 && a.ref == nullptr)
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "reference_points pointer is NULL");
  if (!aligned(a.ref, 4))
    return fail(MSDA_ERROR_MISALIGNED, "reference_points must be 4-byte aligned (fp32)");
  return MSDA_SUCCESS;
}

int run_fwd(const Args& a, void* out, void* stream) {
  if ((a.value == nullptr && a.B * a.K * a.H * a.C > 0) || (out == nullptr && a.B * a.Q * a.H * a.C > 0))
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "value/output pointer is NULL");
  const void* bufs[1] = {out};
  Problem p;
  LaunchShape ls;
  int rc = prepare(a, bufs, 1, p, ls);
  if (rc == MSDA_SUCCESS) rc = check_fused(a);
  if (rc != MSDA_SUCCESS) return rc;
  if (a.B * a.Q * a.H * a.C == 0) return ok();
  p.ref = a.ref;
  const cudaError_t err = dispatch_fwd(a, ls, p, out, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "forward launch");
  return ok();
}

// Validate the backward arguments; on success `p`/`ls` are ready to launch.
int prepare_bwd(const Args& a, const void* go, const void* gv_like, void* gl, void* ga,
                Problem& p, LaunchShape& ls) {
  const int64_t nval = a.B * a.K * a.H * a.C;
  const int64_t nsmp = a.B * a.Q * a.H * a.L * a.P;
  if (nval > 0 && (a.value == nullptr || gv_like == nullptr))
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "value/grad_value pointer is NULL");
  if (nsmp > 0 && (gl == nullptr || ga == nullptr || a.loc == nullptr || a.attn == nullptr))
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "sampling/attention (grad) pointer is NULL");
  if (a.B * a.Q * a.H * a.C > 0 && go == nullptr)
    return fail(MSDA_ERROR_INVALID_ARGUMENT, "grad_output pointer is NULL");
  const void* bufs[2] = {go, gv_like};
  int rc = prepare(a, bufs, 2, p, ls);
  if (rc != MSDA_SUCCESS) return rc;
  const int64_t se = dtype_bytes(a.sdt);
  if (!aligned(gl, se) || !aligned(ga, se))
    return fail(MSDA_ERROR_MISALIGNED, "gradient buffers must be aligned to their element size");
  return MSDA_SUCCESS;
}

// The gather/scatter backward of 16-bit values reads 8-byte chunks (4
// channels, one 16-byte fp32 vector reduction each): same lanes per row,
// twice the chunks per lane.
void bwd_gather_shape(const Args& a, Problem& p, LaunchShape& ls) {
  // MSDA_BWD_CHUNK16 (tuning): keep the forward's 16-byte chunks.
  if (dtype_bytes(a.vdt) == 2 && ls.vb == 16 && std::getenv("MSDA_BWD_CHUNK16") == nullptr) {
    ls.vb = 8;
    // Twice the lanes per row (up to a warp) rather than twice the chunks per
    // lane: each warp-wide reduction then covers whole 128-byte lines of the
    // accumulator, one line touch per row instead of two.
    const int64_t nv = a.C * 2 / 8;
    if (p.log2g < 5 && (int64_t{1} << (p.log2g + 1)) <= nv && ls.vpl == 1 &&
        std::getenv("MSDA_BWD_WIDE_ROWS") == nullptr) {
      p.log2g += 1;
      ls.grid *= 2;
    } else {
      ls.vpl *= 2;
    }
  }
}

// Launch the scatter kernel (or zero-fill the per-sample gradients when
// C == 0).  `gacc` receives += contributions; it is not cleared here.
int launch_accumulate(const Args& a, const Problem& p, const LaunchShape& ls, const void* go,
                      float* gacc, void* gl, void* ga, cudaStream_t st) {
  const int64_t nsmp = a.B * a.Q * a.H * a.L * a.P;
  if (nsmp == 0) return MSDA_SUCCESS;
  cudaError_t err;
  if (a.C == 0) {
    const int64_t se = dtype_bytes(a.sdt);
    err = cudaMemsetAsync(gl, 0, static_cast<size_t>(nsmp * a.ndim * se), st);
    if (err == cudaSuccess) err = cudaMemsetAsync(ga, 0, static_cast<size_t>(nsmp * se), st);
    if (err == cudaSuccess && a.fused)
      err = cudaMemsetAsync(p.ref_partial, 0,
                            static_cast<size_t>(a.B * a.Q * a.H * a.L * a.ndim) * sizeof(float), st);
    return err == cudaSuccess ? MSDA_SUCCESS : cuda_fail(err, "zeroing gradients");
  }
  err = dispatch_bwd(a, ls, p, go, gacc, gl, ga, st);
  return err == cudaSuccess ? MSDA_SUCCESS : cuda_fail(err, "backward launch");
}

cudaError_t cast_from_f32(const float* src, void* dst, int dt, int64_t n, cudaStream_t st) {
  switch (dt) {
    case MSDA_FLOAT16: return launch_cast<__half>(src, dst, n, st);
    case MSDA_BFLOAT16: return launch_cast<__nv_bfloat16>(src, dst, n, st);
    default: return launch_cast<float>(src, dst, n, st);
  }
}

// ------------------------------------------------------------ backward plan
// The backward has two implementations: the cell-sorted pipeline
// (msda_sorted.cuh; host-resident shapes, large problems) and the
// gather/scatter kernel (any shape; vector reductions into grad_value or an
// fp32 workspace).  The plan picks one and lays out the workspace.

// Gather path, 16-bit values, opt-in (MSDA_BWD_DIRECT16=1): a level whose
// expected contributions per grad_value element (2^d corners x Q x P samples
// / voxels) stay at or below this bound reduces straight into grad_value in
// its own dtype, as the reference does for every level, instead of through
// the fp32 accumulator.  The bound assumes uniformly spread locations:
// clustered samples (a module's points around their reference points) can put
// hundreds of 16-bit roundings on one element, so the default accumulates
// every level in fp32 and rounds once.
constexpr double kDirect16Contrib = 8.0;

struct BwdPlan {
  size_t ws_bytes = 0;
  // gather path
  int32_t direct16 = 0;   // levels reduced straight into grad_value
  bool compact = false;   // fp32 accumulator holds only the other levels
  int64_t acc_keys = 0;   // keys per batch entry in the fp32 accumulator
  int32_t acc_start[kMaxLevels] = {};
  // cell-sorted path (msda_sorted.cuh)
  bool sorted = false;
  SortPlan sp{};          // per-chunk sizes; pointers are set per call
  int64_t chunk_b = 0;    // batch entries per chunk
  int64_t smp_per_b = 0;  // samples per batch entry
  int64_t keys_per_b = 0; // bucket keys per batch entry
  size_t soff[6] = {};    // bucket counts, bsum, ranks, srec, acc, sorted-dots stage
};

size_t align256(size_t x) { return (x + 255) & ~size_t{255}; }

// ------------------------------------------------------------ sorted plan
// The cell-sorted backward runs when the level shapes are on the host and the
// problem is large enough to amortise its launches.  Per level it picks how
// the value gradient is formed: gathered per value row (levels with at most
// kVoxelMaxDensity samples per cell and (b, h)) or aggregated per cell in
// registers and flushed with fp32 reductions (denser levels).  Measured on
// the 3D xl workload (B=8, bf16): level 0 (0.38 samples per cell) 4.07 ms
// gathered on the tensor cores; level 1 (2.9 per cell) 4.2 ms gathered there
// against 2.0 ms aggregated (on the CUDA cores: 7.5 against ~2 ms).
constexpr int64_t kSortedMinSamples = int64_t{1} << 20;
constexpr double kVoxelMaxDensity = 2.0;
constexpr bool kSortedByDefault = true;
// Sorted positions per dense-kernel CTA and at most this many samples staged
// per voxel-kernel round.
constexpr int64_t kDenseChunk = 512;
constexpr int64_t kVoxelCap = 512;
static_assert(kVoxelCap <= 2 * kThreads, "msda_voxel_mma_kernel stages two slots per thread");
// Levels whose value slice of one batch entry is at least this large take
// their dot products in sorted order (msda_sdots_kernel): in query order
// their rows are fetched from DRAM on almost every touch.
constexpr double kSortedDotsMinBytes = 96.0 * 1048576.0;
// Dense levels with at least this many samples per cell and (b, h) aggregate
// on the tensor cores (16-bit values).  Measured on 3D xl (B=8, bf16): level 1
// (2.9 per cell) 1.96 ms on the CUDA cores against 2.43 ms on the tensor
// cores; levels 2-3 (22 and 154 per cell) 2.35 against 1.52 ms.
constexpr double kDenseMmaMinDensity = 8.0;

FastDiv make_fdiv(uint32_t d) {
  if (d == 0) d = 1;
  uint32_t l = 0;
  while ((uint64_t{1} << l) < d) ++l;
  const uint64_t m = ((uint64_t{1} << (31 + l)) + d - 1) / d;
  return FastDiv{static_cast<uint32_t>(m), 31 + l};
}

bool plan_sorted(const Args& a, const Problem& p, const LaunchShape& ls, BwdPlan& pl) {
  if (a.scatter_only || a.fused || p.shapes_dev != nullptr) return false;
  // rows wider than two chunks per lane keep the scatter plan (the sorted
  // walk holds 2^d corner rows and their gradients in registers)
  Problem pw = p;
  LaunchShape lw = ls;
  bwd_gather_shape(a, pw, lw);
  if (lw.vpl > 2) return false;
  const char* env = std::getenv("MSDA_BWD_PATH");
  const bool forced = env && std::strcmp(env, "sorted") == 0;
  if (env && !forced) return false;
  const int64_t samples = a.B * a.Q * a.H * a.L * a.P;
  if (samples == 0 || a.C == 0 || a.L == 0) return false;
  if (!forced && (!kSortedByDefault || samples < kSortedMinSamples)) return false;
  const char* dens_env = std::getenv("MSDA_VOXEL_DENSITY");
  double max_dens = dens_env ? std::atof(dens_env) : kVoxelMaxDensity;
  // 16-bit values with C = 16, 32 or 64 form the voxel levels on the tensor
  // cores (msda_voxel_mma_kernel; MSDA_VOXEL_MMA=0: msda_voxel_kernel;
  // MSDA_VOXEL_MMA=tc: msda_voxel_tc_kernel, tcgen05 with TMEM accumulators).
  const char* vm_env = std::getenv("MSDA_VOXEL_MMA");
  const bool mma16 = dtype_bytes(a.vdt) == 2 && (a.C == 16 || a.C == 32 || a.C == 64);
  const bool vtc = mma16 && vm_env && std::strcmp(vm_env, "tc") == 0;
  const bool vmma = mma16 && !vtc && !(vm_env && std::strcmp(vm_env, "0") == 0);
  // msda_voxel_kernel takes the forward's lane shape (16-byte chunks where
  // the row allows); shapes it is not instantiated for keep every level dense.
  if (!vmma && !vtc && !((ls.vb == 16 && ls.vpl <= 4) || ((ls.vb == 4 || ls.vb == 2) && ls.vpl == 1)))
    max_dens = -1.0;
  const int tile_max = (kThreads / 32) * 32;         // voxels per voxel-kernel CTA (a warp per 32)
  const int64_t row_bytes = a.C * dtype_bytes(a.vdt);
  // samples the voxel kernel stages per round: as many as fit next to the
  // warps' areas (fp32 accumulators, 32 KB; or the tensor-core kernel's
  // 16-bit weight tiles, the zero row and the warps' slot lists and ranges)
  // and the range bounds in 72 KB, at most 512 (two per thread)
  const int64_t nw = kThreads / 32;
  const int64_t bounds_max = int64_t{4} * (tile_max + 2) * 4 + 4 * 64;
  const int64_t acc_bytes =
      vmma ? 32 + nw * vm_warp_bytes(static_cast<int>(a.C / 8)) + nw * kVmList * 2 + nw * 8 * 4
           : nw * 32 * 32 * 4;
  // MSDA_VOXEL_SMEM_KB (tuning): the voxel kernel's shared-memory budget
  const char* vs_env = std::getenv("MSDA_VOXEL_SMEM_KB");
  const int64_t vbudget = (vs_env && std::atoll(vs_env) > 0 ? std::atoll(vs_env) : 72) * 1024;
  // per staged sample: its record (32 B; the tensor-core kernel keeps its
  // 2^d corner weights as 16-bit halves instead), cell row / x offset (4 B)
  // and grad_out row
  const int64_t per_smp = (vmma ? (a.ndim == 3 ? 32 : 16) : 32) + 4 + row_bytes;
  int64_t cap = (vbudget - acc_bytes - bounds_max) / per_smp;
  cap = std::min<int64_t>(cap, kVoxelCap) & ~int64_t{1};
  if (vtc) cap = kVoxelCap;  // its layout (vtc_layout) stays inside two CTAs per SM at C = 32
  if (cap < 16) max_dens = -1.0;
  SortPlan sp{};
  // 16-bit values with C = 16, 32 or 64: dense levels with at least
  // kDenseMmaMinDensity samples per cell and (b, h) go to the tensor-core
  // kernel (MSDA_DENSE_MMA=0: none; MSDA_DENSE_MMA_DENSITY: the threshold)
  const char* mma_env = std::getenv("MSDA_DENSE_MMA");
  const bool mma_ok = dtype_bytes(a.vdt) == 2 && (a.C == 16 || a.C == 32 || a.C == 64) &&
                      !(mma_env && std::strcmp(mma_env, "0") == 0);
  const char* mma_dens_env = std::getenv("MSDA_DENSE_MMA_DENSITY");
  const double mma_dens = mma_dens_env ? std::atof(mma_dens_env) : kDenseMmaMinDensity;
  int64_t seg = 0, vox = 0, acc_keys = 0, units = 0, max_bounds = 0, vtc_ncr = 0;
  int nvl = 0;
  const bool f32 = a.vdt == MSDA_FLOAT32;
  for (int64_t l = 0; l < a.L; ++l) {
    int64_t ncell = 1, nvox = 1;
    for (int ax = 0; ax < 3; ++ax) {
      const int64_t sz = ax < a.ndim ? p.lv.size[l][ax] : 1;
      sp.cells[l][ax] = static_cast<int32_t>(ax < a.ndim ? sz + 1 : 1);
      ncell *= sp.cells[l][ax];
      nvox *= sz;
    }
    sp.lvl_base[l] = static_cast<int32_t>(seg);
    seg += ncell + 1;
    if (seg >= INT32_MAX) return false;
    const double dens = static_cast<double>(a.Q * a.P) / static_cast<double>(ncell);
    if (dens <= max_dens && nvox > 0) {
      // tile: NZ planes x NY rows x TX voxels, TX up to tile_max; fewer rows
      // when the expected samples of its cell rows pass the staging rounds
      // aimed at (two; one for the tensor-core kernel)
      const int64_t W = p.lv.size[l][0], Hl = p.lv.size[l][1];
      const int64_t Dl = a.ndim == 3 ? p.lv.size[l][2] : 1;
      // msda_voxel_kernel: up to 8 segments of 32 voxels (a warp each) in one
      // plane; msda_voxel_mma_kernel: up to 16 (two per warp) in two planes
      // msda_voxel_tc_kernel: four voxel rows of at most 128 voxels (one
      // tensor-memory accumulator each), 2 planes x 2 rows in 3D, 4 rows in 2D
      const int64_t tx = std::min<int64_t>(W, vtc ? 128 : tile_max);
      const int64_t segs = (tx + 31) / 32;
      const int64_t nz = a.ndim == 3 && (vtc || (vmma && Dl >= 2)) ? 2 : 1;
      const int64_t wseg = vmma ? 2 * nw : nw;
      int64_t ny = vtc ? (a.ndim == 3 ? 2 : 4)
                       : std::max<int64_t>(1, std::min<int64_t>(wseg / (segs * nz), Hl));
      const int64_t zr = a.ndim == 3 ? nz + 1 : 1;
      const double rounds = vmma ? 1.0 : 2.0;
      while (!vtc && ny > 1 && static_cast<double>(zr * (ny + 1) * (tx + 1)) * dens > rounds * cap)
        --ny;
      VoxTile vt;
      vt.tx = static_cast<int32_t>(tx);
      vt.ny = static_cast<int32_t>(ny);
      vt.nz = static_cast<int32_t>(nz);
      vt.ntx = static_cast<int32_t>((W + tx - 1) / tx);
      vt.nty = static_cast<int32_t>((Hl + ny - 1) / ny);
      // range bounds: every cell of the tile's cell rows, or (tensor cores)
      // two per segment and cell row; then the cell rows' offsets
      const int64_t nbr = vmma ? vm_bounds_per_row(static_cast<int>(segs)) : tx + 2;
      max_bounds = std::max<int64_t>(max_bounds, zr * (ny + 1) * nbr + zr * (ny + 1) + 1);
      vtc_ncr = std::max<int64_t>(vtc_ncr, zr * (ny + 1));
      sp.voxel_mask |= 1 << l;
      sp.vl_level[nvl] = static_cast<int32_t>(l);
      sp.vl_tile[nvl] = vt;
      sp.vl_ubase[nvl] = static_cast<int32_t>(units);
      units += int64_t{vt.ntx} * vt.nty * ((Dl + nz - 1) / nz);
      vox += nvox;
      ++nvl;
      if (vox >= INT32_MAX || units >= INT32_MAX) return false;
    } else {
      pl.acc_start[l] = static_cast<int32_t>(f32 ? p.lv.start[l] : acc_keys);
      acc_keys += nvox;
      if (mma_ok && dens >= mma_dens)
        sp.ml_level[sp.nml++] = static_cast<int32_t>(l);
      else
        sp.dl_level[sp.ndl++] = static_cast<int32_t>(l);
    }
  }
  sp.vl_ubase[nvl] = static_cast<int32_t>(units);
  // dense kernel: up to 512 positions per CTA, records + grad_out rows in
  // at most 64 KB of shared memory
  {
    // per position: its record (later its corner weights), grad_out row,
    // segment start and segment cell
    const int64_t per = static_cast<int64_t>(sizeof(SRec)) + row_bytes + 8;
    int64_t dchunk = std::min<int64_t>(kDenseChunk, (64 * 1024 - 4) / per);
    dchunk = std::max<int64_t>(dchunk, 2 * kSegMax) & ~int64_t{1};
    sp.dchunk = static_cast<int32_t>(dchunk);
    sp.dchunks = static_cast<int32_t>((a.Q * a.P + dchunk - 1) / dchunk);
    sp.dsmem = static_cast<int32_t>(dchunk * per + 4);
    // the tensor-core kernel: the records' area also holds the corner-weight
    // table, and 16 zero bytes follow
    const int64_t area0 =
        (std::max<int64_t>(dchunk * int64_t{sizeof(SRec)}, kWBytes) + 15) & ~int64_t{15};
    sp.dsmem_mma = static_cast<int32_t>(area0 + dchunk * (row_bytes + 8) + 4 + 32);
  }
  sp.dlog2g = pw.log2g;
  sp.dnv = static_cast<int32_t>(a.C * dtype_bytes(a.vdt) / lw.vb);
  sp.div_dnv = make_fdiv(static_cast<uint32_t>(std::max<int32_t>(sp.dnv, 1)));
  const int64_t per_b_smp = a.Q * a.H * a.L * a.P;
  const int64_t per_b_keys = a.H * seg;
  const int64_t per_b_vox = a.H * vox;
  const int64_t lim = INT32_MAX - 1;
  int64_t nb = a.B;
  nb = std::min(nb, lim / per_b_smp);
  nb = std::min(nb, lim / per_b_keys);
  if (per_b_vox > 0) nb = std::min(nb, lim / per_b_vox);
  if (units > 0) nb = std::min(nb, lim / (a.H * units));
  // MSDA_SORTED_CHUNK_B (tests, tuning): at most this many batch entries per chunk
  const char* cb_env = std::getenv("MSDA_SORTED_CHUNK_B");
  if (cb_env && std::atoll(cb_env) > 0) nb = std::min<int64_t>(nb, std::atoll(cb_env));
  if (nb < 1) return false;
  sp.n = static_cast<int32_t>(nb * per_b_smp);
  sp.nkeys = static_cast<int32_t>(nb * per_b_keys);
  sp.seg_keys = static_cast<int32_t>(seg);
  sp.nvl = nvl;
  sp.units_per_bh = static_cast<int32_t>(units);
  sp.vcap = static_cast<int32_t>(cap);
  sp.vnv = p.nv;
  sp.div_nv = make_fdiv(static_cast<uint32_t>(std::max<int32_t>(p.nv, 1)));
  sp.vsmem = static_cast<int32_t>(acc_bytes + cap * per_smp + max_bounds * 4);
  sp.vmma = vtc ? 2 : vmma ? 1 : 0;
  if (vtc)  // its layout from a 1024-byte aligned base
    sp.vsmem = 1024 + vtc_layout(static_cast<int>(a.C / 8), static_cast<int>(a.ndim),
                                 static_cast<int>(cap), static_cast<int>(vtc_ncr)).end;
  if (nvl > 0 && sp.vsmem > (vtc ? 200 : 100) * 1024) return false;
  sp.div_lp = make_fdiv(static_cast<uint32_t>(a.L * a.P));
  sp.div_p = make_fdiv(static_cast<uint32_t>(a.P));
  sp.div_h = make_fdiv(static_cast<uint32_t>(a.H));
  sp.div_l = make_fdiv(static_cast<uint32_t>(a.L));
  sp.div_q = make_fdiv(static_cast<uint32_t>(a.Q));
  // levels whose dot products run in sorted order: those whose value slice
  // of one batch entry passes kSortedDotsMinBytes (MSDA_SORTED_DOTS_MB, MiB)
  {
    const char* sd_env = std::getenv("MSDA_SORTED_DOTS_MB");
    const double min_bytes = sd_env ? std::atof(sd_env) * 1048576.0 : kSortedDotsMinBytes;
    for (int64_t l = 0; l < a.L; ++l) {
      int64_t nvox = 1;
      for (int ax = 0; ax < a.ndim; ++ax) nvox *= p.lv.size[l][ax];
      sp.div_cx[l] = make_fdiv(static_cast<uint32_t>(sp.cells[l][0]));
      sp.div_cy[l] = make_fdiv(static_cast<uint32_t>(sp.cells[l][1]));
      if (nvox > 0 && static_cast<double>(nvox * a.H * row_bytes) >= min_bytes) {
        sp.sdots_mask |= 1 << l;
        sp.sl_level[sp.nsl++] = static_cast<int32_t>(l);
      }
    }
    // MSDA_SDOTS_PER (tuning): sorted positions per msda_sdots_kernel CTA
    const char* per_env = std::getenv("MSDA_SDOTS_PER");
    const int64_t per = per_env && std::atoll(per_env) > 0 ? std::atoll(per_env) : kSdotsPer;
    sp.sd_per = static_cast<int32_t>(std::min<int64_t>(per, 1 << 20));
    sp.sd_chunks = static_cast<int32_t>((a.Q * a.P + sp.sd_per - 1) / sp.sd_per);
    if (nb * a.H * sp.nsl * sp.sd_chunks >= INT32_MAX) return false;
  }
  pl.sp = sp;
  pl.sorted = true;
  pl.chunk_b = nb;
  pl.smp_per_b = per_b_smp;
  pl.keys_per_b = per_b_keys;
  pl.compact = !f32;
  pl.acc_keys = f32 ? a.K : acc_keys;
  pl.direct16 = 0;
  const int64_t nblk = (int64_t{sp.nkeys} + kScanTile - 1) / kScanTile;
  const int64_t n = sp.n;
  const size_t sizes[6] = {
      static_cast<size_t>(sp.nkeys + 1) * 4, static_cast<size_t>(nblk + 1) * 4,
      static_cast<size_t>(n) * 4, static_cast<size_t>(n) * sizeof(SRec),
      f32 ? 0 : static_cast<size_t>(nb * acc_keys * a.H * a.C) * sizeof(float),
      static_cast<size_t>(nb * a.Q * a.H * sp.nsl * a.P) * 16};
  size_t off = 0;
  for (int i = 0; i < 6; ++i) {
    pl.soff[i] = off;
    off += align256(sizes[i]);
  }
  pl.ws_bytes = off;
  return true;
}

// Gather-path value-gradient targets (see kDirect16Contrib).
void plan_gather_targets(const Args& a, const Problem& p, BwdPlan& pl) {
  pl.acc_keys = a.K;
  if (dtype_bytes(a.vdt) != 2 || p.shapes_dev != nullptr || a.K == 0) return;
  const char* env = std::getenv("MSDA_BWD_DIRECT16");
  if (env == nullptr || std::strcmp(env, "1") != 0) return;
  // MSDA_BWD_DIRECT16_MAX (tuning): the contribution bound.
  const char* mx = std::getenv("MSDA_BWD_DIRECT16_MAX");
  const double bound = mx ? std::atof(mx) : kDirect16Contrib;
  int64_t keys = 0;
  for (int64_t l = 0; l < a.L; ++l) {
    const int64_t nvox = int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2];
    const double contrib = static_cast<double>(int64_t{1} << a.ndim) * a.Q * a.P /
                           static_cast<double>(std::max<int64_t>(nvox, 1));
    if (contrib <= bound) {
      pl.direct16 |= 1 << l;
    } else {
      pl.acc_start[l] = static_cast<int32_t>(keys);
      keys += nvox;
    }
  }
  if (pl.direct16 == 0) return;
  pl.compact = true;
  pl.acc_keys = keys;
}

void plan_bwd(const Args& a, const Problem& p, const LaunchShape& ls, BwdPlan& pl) {
  pl = BwdPlan{};
  if (plan_sorted(a, p, ls, pl)) return;
  plan_gather_targets(a, p, pl);
  pl.ws_bytes = (a.vdt == MSDA_FLOAT32)
                    ? 0 : static_cast<size_t>(a.B * pl.acc_keys * a.H * a.C) * sizeof(float);
}

cudaError_t dispatch_sorted(int vdt, int sdt, const LaunchShape& ls, const LaunchShape& lsd,
                            const Problem& p, const SortPlan& sp, const void* go, float* gacc,
                            void* gv, void* gl, void* ga, cudaStream_t st) {
  switch (vdt) {
    case MSDA_FLOAT32:
      return launch_sorted_bwd<float, float>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st);
    case MSDA_FLOAT16:
      return sdt == MSDA_FLOAT32
                 ? launch_sorted_bwd<__half, float>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st)
                 : launch_sorted_bwd<__half, __half>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st);
    default:
      return sdt == MSDA_FLOAT32
                 ? launch_sorted_bwd<__nv_bfloat16, float>(ls, lsd, p, sp, go, gacc, gv, gl, ga, st)
                 : launch_sorted_bwd<__nv_bfloat16, __nv_bfloat16>(ls, lsd, p, sp, go, gacc, gv,
                                                                   gl, ga, st);
  }
}

// The cell-sorted backward, chunk by chunk of batch entries (pointers
// offset to the chunk; the workspace is reused by every chunk).
int run_bwd_sorted(const Args& a, Problem p, LaunchShape ls, const BwdPlan& pl, const void* go,
                   void* gv, void* gl, void* ga, void* ws, cudaStream_t st) {
  LaunchShape lsd = ls;  // the dense kernel's lane shape
  {
    Problem pd = p;
    bwd_gather_shape(a, pd, lsd);
  }
  const int64_t e = dtype_bytes(a.vdt), se = dtype_bytes(a.sdt);
  const int64_t row_bytes = a.H * a.C * e;  // one key of value / grad_value
  const bool f32 = a.vdt == MSDA_FLOAT32;
  char* w = static_cast<char*>(ws);
  SortPlan sp = pl.sp;
  sp.cnt = reinterpret_cast<int32_t*>(w + pl.soff[0]);
  sp.bsum = reinterpret_cast<int32_t*>(w + pl.soff[1]);
  sp.pos = reinterpret_cast<int32_t*>(w + pl.soff[2]);
  sp.srec = reinterpret_cast<SRec*>(w + pl.soff[3]);
  sp.sd_stage = reinterpret_cast<float4*>(w + pl.soff[5]);
  float* acc = f32 ? nullptr : reinterpret_cast<float*>(w + pl.soff[4]);
  p.acc_compact = pl.compact ? 1 : 0;
  p.acc_keys = pl.acc_keys;
  for (int l = 0; l < kMaxLevels; ++l) p.acc_start[l] = pl.acc_start[l];
  p.direct16 = 0;
  p.grad_value16 = nullptr;
  const int64_t smp_bytes = pl.smp_per_b;  // samples per batch entry
  cudaError_t err = cudaSuccess;
  for (int64_t b0 = 0; b0 < a.B; b0 += pl.chunk_b) {
    const int64_t nb = std::min(pl.chunk_b, a.B - b0);
    Problem pc = p;
    pc.B = nb;
    pc.value = static_cast<const char*>(a.value) + b0 * a.K * row_bytes;
    pc.loc = static_cast<const char*>(a.loc) + b0 * smp_bytes * a.ndim * se;
    pc.attn = static_cast<const char*>(a.attn) + b0 * smp_bytes * se;
    SortPlan sc = sp;
    sc.n = static_cast<int32_t>(nb * pl.smp_per_b);
    sc.nkeys = static_cast<int32_t>(nb * pl.keys_per_b);
    LaunchShape lc = ls;  // dots kernel: one lane group per (b, q, h) row of the chunk
    lc.grid = ((nb * a.Q * a.H << p.log2g) + kThreads - 1) / kThreads;
    const void* go_c = static_cast<const char*>(go) + b0 * a.Q * a.H * a.C * e;
    char* gv_c = static_cast<char*>(gv) + b0 * a.K * row_bytes;
    void* gl_c = static_cast<char*>(gl) + b0 * smp_bytes * a.ndim * se;
    void* ga_c = static_cast<char*>(ga) + b0 * smp_bytes * se;
    // dense levels: zero their reduction targets
    int64_t dense_keys = 0;
    for (int64_t l = 0; l < a.L; ++l) {
      if ((sp.voxel_mask >> l) & 1) continue;
      const int64_t nvox = int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2];
      dense_keys += nvox;
      if (f32 && nvox > 0) {
        err = zero_key_range(a, gv_c, p.lv.start[l], nvox, nb, e, st);
        if (err != cudaSuccess) return cuda_fail(err, "zeroing grad_value rows");
      }
    }
    if (!f32 && dense_keys > 0) {
      err = cudaMemsetAsync(acc, 0, static_cast<size_t>(nb * dense_keys * a.H * a.C) * sizeof(float),
                            st);
      if (err != cudaSuccess) return cuda_fail(err, "zeroing the grad_value accumulator");
    }
    float* gacc = f32 ? reinterpret_cast<float*>(gv_c) : acc;
    err = dispatch_sorted(a.vdt, a.sdt, lc, lsd, pc, sc, go_c, gacc, gv_c, gl_c, ga_c, st);
    if (err != cudaSuccess) return cuda_fail(err, "sorted backward launch");
    if (!f32 && dense_keys > 0) {
      Problem pcast = pc;
      pcast.direct16 = sp.voxel_mask;  // the levels the accumulator does not hold
      err = a.vdt == MSDA_FLOAT16 ? launch_compact_cast<__half>(pcast, acc, gv_c, st)
                                  : launch_compact_cast<__nv_bfloat16>(pcast, acc, gv_c, st);
      if (err != cudaSuccess) return cuda_fail(err, "grad_value cast launch");
    }
  }
  return ok();
}

int run_bwd(const Args& a, const void* go, void* gv, void* gl, void* ga, void* ws,
            size_t ws_bytes, void* stream, float* ref_partial = nullptr) {
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  Problem p;
  LaunchShape ls;
  int rc = prepare_bwd(a, go, gv, gl, ga, p, ls);
  if (rc == MSDA_SUCCESS) rc = check_fused(a);
  if (rc != MSDA_SUCCESS) return rc;
  if (a.fused) {
    if (a.B * a.Q * a.H * a.L * a.P > 0 && ref_partial == nullptr)
      return fail(MSDA_ERROR_INVALID_ARGUMENT, "grad_reference_partial pointer is NULL");
    if (!aligned(ref_partial, 4))
      return fail(MSDA_ERROR_MISALIGNED, "grad_reference_partial must be 4-byte aligned");
    p.ref = a.ref;
    p.ref_partial = ref_partial;
  }
  BwdPlan pl;
  plan_bwd(a, p, ls, pl);
  const int64_t nval = a.B * a.K * a.H * a.C;
  if (pl.ws_bytes > 0) {
    if (ws == nullptr || ws_bytes < pl.ws_bytes)
      return fail(MSDA_ERROR_WORKSPACE, "backward needs %zu workspace bytes, got %zu",
                  pl.ws_bytes, ws == nullptr ? size_t{0} : ws_bytes);
    if (!aligned(ws, 256)) return fail(MSDA_ERROR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  if (pl.sorted)
    return run_bwd_sorted(a, p, ls, pl, go, gv, gl, ga, ws, static_cast<cudaStream_t>(stream));
  cudaError_t err;
  float* gacc = nullptr;
  if (a.vdt == MSDA_FLOAT32) {
    gacc = static_cast<float*>(gv);
  } else if (nval > 0) {
    gacc = static_cast<float*>(ws);
  }
  p.direct16 = pl.direct16;
  p.acc_compact = pl.compact ? 1 : 0;
  p.acc_keys = pl.acc_keys;
  for (int l = 0; l < kMaxLevels; ++l) p.acc_start[l] = pl.acc_start[l];
  p.grad_value16 = pl.direct16 ? gv : nullptr;
  const int64_t row_bytes = a.H * a.C * dtype_bytes(a.vdt);
  const int64_t nacc = a.B * pl.acc_keys * a.H * a.C;
  if (nacc > 0) {
    err = cudaMemsetAsync(gacc, 0, static_cast<size_t>(nacc) * sizeof(float), st);
    if (err != cudaSuccess) return cuda_fail(err, "zeroing the grad_value accumulator");
  }
  // Direct levels: their grad_value rows (one span per batch entry) start at 0.
  for (int64_t l = 0; l < a.L && nval > 0; ++l) {
    if (!((pl.direct16 >> l) & 1)) continue;
    const int64_t nvox = int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2];
    if (nvox == 0) continue;
    err = zero_key_range(a, gv, p.lv.start[l], nvox, a.B, dtype_bytes(a.vdt), st);
    if (err != cudaSuccess) return cuda_fail(err, "zeroing grad_value rows");
  }
  bwd_gather_shape(a, p, ls);
  p.nv = static_cast<int32_t>(a.C * dtype_bytes(a.vdt) / ls.vb);
  rc = launch_accumulate(a, p, ls, go, gacc, gl, ga, st);
  if (rc != MSDA_SUCCESS) return rc;
  if (a.vdt != MSDA_FLOAT32 && nval > 0) {
    if (pl.compact)
      err = a.vdt == MSDA_FLOAT16 ? launch_compact_cast<__half>(p, gacc, gv, st)
                                  : launch_compact_cast<__nv_bfloat16>(p, gacc, gv, st);
    else
      err = cast_from_f32(gacc, gv, a.vdt, nval, st);
    if (err != cudaSuccess) return cuda_fail(err, "grad_value cast launch");
  }
  return ok();
}

int run_bwd_accumulate(const Args& a, const void* go, float* gacc, void* gl, void* ga,
                       void* stream) {
  Problem p;
  LaunchShape ls;
  int rc = prepare_bwd(a, go, gacc, gl, ga, p, ls);
  if (rc != MSDA_SUCCESS) return rc;
  if (a.B * a.K * a.H * a.C > 0 && !aligned(gacc, 16))
    return fail(MSDA_ERROR_MISALIGNED, "grad_value_accum must be 16-byte aligned");
  bwd_gather_shape(a, p, ls);
  p.nv = static_cast<int32_t>(a.C * dtype_bytes(a.vdt) / ls.vb);
  rc = launch_accumulate(a, p, ls, go, gacc, gl, ga, static_cast<cudaStream_t>(stream));
  return rc == MSDA_SUCCESS ? ok() : rc;
}

}  // namespace

// Record an error for msda_last_error() from another translation unit.
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

}  // namespace msda

using msda::Args;

#define MSDA_ARGS(ND)                                                                      \
  Args a = msda::with_layout(Args{                                                         \
      ND, value, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,        \
      spatial_shapes_on_device, num_levels, sampling_locations, attention_weights,         \
      sampling_dtype, num_queries, num_points, clamp_grid, clamp_eps})

extern "C" {

int msda2d_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, void* output, void* stream) {
  MSDA_ARGS(2);
  return msda::run_fwd(a, output, stream);
}

int msda3d_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, void* output, void* stream) {
  MSDA_ARGS(3);
  return msda::run_fwd(a, output, stream);
}

int msda2d_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, void* grad_value,
               void* grad_sampling_locations, void* grad_attention_weights, void* workspace,
               size_t workspace_bytes, void* stream) {
  MSDA_ARGS(2);
  return msda::run_bwd(a, grad_output, grad_value, grad_sampling_locations,
                       grad_attention_weights, workspace, workspace_bytes, stream);
}

int msda3d_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, void* grad_value,
               void* grad_sampling_locations, void* grad_attention_weights, void* workspace,
               size_t workspace_bytes, void* stream) {
  MSDA_ARGS(3);
  return msda::run_bwd(a, grad_output, grad_value, grad_sampling_locations,
                       grad_attention_weights, workspace, workspace_bytes, stream);
}

int msda2d_bwd_accumulate(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                          int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                          int spatial_shapes_on_device, int64_t num_levels,
                          const void* sampling_locations, const void* attention_weights,
                          int sampling_dtype, int64_t num_queries, int64_t num_points,
                          int clamp_grid, double clamp_eps, const void* grad_output,
                          float* grad_value_accum, void* grad_sampling_locations,
                          void* grad_attention_weights, void* stream) {
  MSDA_ARGS(2);
  return msda::run_bwd_accumulate(a, grad_output, grad_value_accum, grad_sampling_locations,
                                  grad_attention_weights, stream);
}

int msda3d_bwd_accumulate(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                          int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                          int spatial_shapes_on_device, int64_t num_levels,
                          const void* sampling_locations, const void* attention_weights,
                          int sampling_dtype, int64_t num_queries, int64_t num_points,
                          int clamp_grid, double clamp_eps, const void* grad_output,
                          float* grad_value_accum, void* grad_sampling_locations,
                          void* grad_attention_weights, void* stream) {
  MSDA_ARGS(3);
  return msda::run_bwd_accumulate(a, grad_output, grad_value_accum, grad_sampling_locations,
                                  grad_attention_weights, stream);
}

#define MSDA_FUSED_ARGS(ND)                                                                \
  Args a = msda::with_layout(Args{                                                         \
      ND, value, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,        \
      spatial_shapes_on_device, num_levels, sampling_offsets, attention_logits,            \
      sampling_dtype, num_queries, num_points, clamp_grid, clamp_eps, reference_points, 1})

int msda2d_fused_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                     int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                     int spatial_shapes_on_device, int64_t num_levels,
                     const float* reference_points, const void* sampling_offsets,
                     const void* attention_logits, int sampling_dtype, int64_t num_queries,
                     int64_t num_points, int clamp_grid, double clamp_eps, void* output,
                     void* stream) {
  MSDA_FUSED_ARGS(2);
  return msda::run_fwd(a, output, stream);
}

int msda3d_fused_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                     int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                     int spatial_shapes_on_device, int64_t num_levels,
                     const float* reference_points, const void* sampling_offsets,
                     const void* attention_logits, int sampling_dtype, int64_t num_queries,
                     int64_t num_points, int clamp_grid, double clamp_eps, void* output,
                     void* stream) {
  MSDA_FUSED_ARGS(3);
  return msda::run_fwd(a, output, stream);
}

int msda2d_fused_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                     int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                     int spatial_shapes_on_device, int64_t num_levels,
                     const float* reference_points, const void* sampling_offsets,
                     const void* attention_logits, int sampling_dtype, int64_t num_queries,
                     int64_t num_points, int clamp_grid, double clamp_eps,
                     const void* grad_output, void* grad_value, float* grad_reference_partial,
                     void* grad_sampling_offsets, void* grad_attention_logits, void* workspace,
                     size_t workspace_bytes, void* stream) {
  MSDA_FUSED_ARGS(2);
  return msda::run_bwd(a, grad_output, grad_value, grad_sampling_offsets, grad_attention_logits,
                       workspace, workspace_bytes, stream, grad_reference_partial);
}

int msda3d_fused_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                     int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                     int spatial_shapes_on_device, int64_t num_levels,
                     const float* reference_points, const void* sampling_offsets,
                     const void* attention_logits, int sampling_dtype, int64_t num_queries,
                     int64_t num_points, int clamp_grid, double clamp_eps,
                     const void* grad_output, void* grad_value, float* grad_reference_partial,
                     void* grad_sampling_offsets, void* grad_attention_logits, void* workspace,
                     size_t workspace_bytes, void* stream) {
  MSDA_FUSED_ARGS(3);
  return msda::run_bwd(a, grad_output, grad_value, grad_sampling_offsets, grad_attention_logits,
                       workspace, workspace_bytes, stream, grad_reference_partial);
}

int msda_cast_from_f32(const float* src, void* dst, int dst_dtype, int64_t count, void* stream) {
  if (count < 0 || msda::dtype_bytes(dst_dtype) == 0)
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "bad count or dtype");
  if (count == 0) return msda::ok();
  if (src == nullptr || dst == nullptr)
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "NULL buffer");
  if (!msda::aligned(src, 16) || !msda::aligned(dst, msda::dtype_bytes(dst_dtype)))
    return msda::fail(MSDA_ERROR_MISALIGNED, "src must be 16-byte aligned, dst element-aligned");
  const cudaError_t err =
      msda::cast_from_f32(src, dst, dst_dtype, count, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? msda::ok() : msda::cuda_fail(err, "cast launch");
}

// The modules' sampling prologue (msda_prologue.cuh): shapes, sizes and
// levels checked, then one launch.
static int prologue_args(int ndim, int64_t batch, int64_t num_queries, int64_t num_heads,
                         int64_t num_levels, int64_t num_points, const int32_t* spatial_shapes,
                         int sampling_dtype, msda::PrologueArgs& pa) {
  if (ndim != 2 && ndim != 3) return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "ndim must be 2 or 3");
  if (batch < 0 || num_queries < 0 || num_heads < 0 || num_levels < 0 || num_points < 0)
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "negative size");
  if (num_levels > msda::kMaxLevels)
    return msda::fail(MSDA_ERROR_TOO_MANY_LEVELS, "num_levels %lld > %d",
                      static_cast<long long>(num_levels), msda::kMaxLevels);
  if (num_levels * num_points > 2048)
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "num_levels * num_points above 2048");
  if (batch * num_queries * num_heads >= (int64_t{1} << 31))
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "batch * num_queries * num_heads above 2^31");
  if (msda::dtype_bytes(sampling_dtype) == 0)
    return msda::fail(MSDA_ERROR_UNSUPPORTED_DTYPE, "sampling_dtype %d", sampling_dtype);
  if (num_levels > 0 && spatial_shapes == nullptr)
    return msda::fail(MSDA_ERROR_INVALID_ARGUMENT, "NULL spatial_shapes");
  pa = msda::PrologueArgs{};
  pa.ndim = ndim;
  pa.B = batch;
  pa.Q = num_queries;
  pa.H = num_heads;
  pa.L = num_levels;
  pa.P = num_points;
  // rows of spatial_shapes in the reference's order ((H, W) or (D, H, W));
  // axis 0 of a location is x
  for (int64_t l = 0; l < num_levels; ++l)
    for (int ax = 0; ax < ndim; ++ax) pa.size[l][ax] = spatial_shapes[l * ndim + (ndim - 1 - ax)];
  return MSDA_SUCCESS;
}

static bool prologue_buffers_ok(const void* const* bufs, int n, int elem) {
  for (int i = 0; i < n; ++i)
    if (bufs[i] == nullptr || !msda::aligned(bufs[i], elem)) return false;
  return true;
}

int msda_prologue_fwd(int ndim, int64_t batch, int64_t num_queries, int64_t num_heads,
                      int64_t num_levels, int64_t num_points, const int32_t* spatial_shapes,
                      const void* reference_points, const void* sampling_offsets,
                      const void* attention_logits, int sampling_dtype,
                      void* sampling_locations, void* attention_weights, void* stream) {
  msda::PrologueArgs pa;
  const int st = prologue_args(ndim, batch, num_queries, num_heads, num_levels, num_points,
                               spatial_shapes, sampling_dtype, pa);
  if (st != MSDA_SUCCESS) return st;
  if (batch * num_queries * num_heads * num_levels * num_points == 0) return msda::ok();
  const void* bufs[5] = {reference_points, sampling_offsets, attention_logits, sampling_locations,
                         attention_weights};
  if (!prologue_buffers_ok(bufs, 5, msda::dtype_bytes(sampling_dtype)))
    return msda::fail(MSDA_ERROR_MISALIGNED, "NULL or unaligned prologue buffer");
  pa.ref = reference_points;
  pa.off = sampling_offsets;
  pa.logits = attention_logits;
  pa.loc = sampling_locations;
  pa.wout = attention_weights;
  const cudaError_t err = msda::prologue_fwd(pa, sampling_dtype, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? msda::ok() : msda::cuda_fail(err, "prologue forward launch");
}

int msda_prologue_bwd(int ndim, int64_t batch, int64_t num_queries, int64_t num_heads,
                      int64_t num_levels, int64_t num_points, const int32_t* spatial_shapes,
                      const void* attention_weights, const void* grad_sampling_locations,
                      const void* grad_attention_weights, int sampling_dtype,
                      float* grad_reference_partial, void* grad_sampling_offsets,
                      void* grad_attention_logits, void* stream) {
  msda::PrologueArgs pa;
  const int st = prologue_args(ndim, batch, num_queries, num_heads, num_levels, num_points,
                               spatial_shapes, sampling_dtype, pa);
  if (st != MSDA_SUCCESS) return st;
  if (batch * num_queries * num_heads * num_levels * num_points == 0) return msda::ok();
  const void* bufs[5] = {attention_weights, grad_sampling_locations, grad_attention_weights,
                         grad_sampling_offsets, grad_attention_logits};
  if (!prologue_buffers_ok(bufs, 5, msda::dtype_bytes(sampling_dtype)) ||
      grad_reference_partial == nullptr || !msda::aligned(grad_reference_partial, 4))
    return msda::fail(MSDA_ERROR_MISALIGNED, "NULL or unaligned prologue buffer");
  pa.weights = attention_weights;
  pa.gloc = grad_sampling_locations;
  pa.gattn = grad_attention_weights;
  pa.gref_partial = grad_reference_partial;
  pa.goff = grad_sampling_offsets;
  pa.glogits = grad_attention_logits;
  const cudaError_t err = msda::prologue_bwd(pa, sampling_dtype, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? msda::ok() : msda::cuda_fail(err, "prologue backward launch");
}

static size_t workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                              int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                              int spatial_shapes_on_device, int64_t num_levels,
                              int64_t num_queries, int64_t num_points, int fused,
                              bool scatter_only = false) {
  // Plan with 256-byte aligned stand-in pointers (never dereferenced).
  void* fake = reinterpret_cast<void*>(uintptr_t{256});
  const Args a = with_layout(Args{
      ndim, fake, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
      spatial_shapes_on_device, num_levels, fake, fake, value_dtype & ~MSDA_VALUE_HEAD_MAJOR,
      num_queries, num_points, 1, 1e-4, static_cast<const float*>(fake), fused, scatter_only});
  msda::Problem p;
  msda::LaunchShape ls;
  const void* bufs[2] = {fake, fake};
  if (msda::prepare(a, bufs, 2, p, ls) != MSDA_SUCCESS) return 0;
  msda::BwdPlan pl;
  msda::plan_bwd(a, p, ls, pl);
  return pl.ws_bytes;
}

size_t msda_bwd_workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                                int64_t num_heads, int64_t channels,
                                const int32_t* spatial_shapes, int spatial_shapes_on_device,
                                int64_t num_levels, int64_t num_queries, int64_t num_points) {
  return workspace_bytes(ndim, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
                         spatial_shapes_on_device, num_levels, num_queries, num_points, 0);
}

size_t msda_fused_bwd_workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                                      int64_t num_heads, int64_t channels,
                                      const int32_t* spatial_shapes, int spatial_shapes_on_device,
                                      int64_t num_levels, int64_t num_queries,
                                      int64_t num_points) {
  return workspace_bytes(ndim, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
                         spatial_shapes_on_device, num_levels, num_queries, num_points, 1);
}

}  // extern "C"

namespace msda {
// The static-scratch backward (msda_noalloc.cu) keeps the gather/scatter
// plan, whose workspace its fixed array was sized for.
size_t scatter_workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                               int spatial_shapes_on_device, int64_t num_levels,
                               int64_t num_queries, int64_t num_points) {
  return workspace_bytes(ndim, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
                         spatial_shapes_on_device, num_levels, num_queries, num_points, 0, true);
}

int bwd_scatter(int ndim, const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                int spatial_shapes_on_device, int64_t num_levels, const void* sampling_locations,
                const void* attention_weights, int sampling_dtype, int64_t num_queries,
                int64_t num_points, int clamp_grid, double clamp_eps, const void* grad_output,
                void* grad_value, void* grad_sampling_locations, void* grad_attention_weights,
                void* workspace, size_t workspace_bytes, void* stream) {
  MSDA_ARGS(ndim);
  a.scatter_only = true;
  return run_bwd(a, grad_output, grad_value, grad_sampling_locations, grad_attention_weights,
                 workspace, workspace_bytes, stream);
}
}  // namespace msda

extern "C" {

const char* msda_status_string(int status) {
  switch (status) {
    case MSDA_SUCCESS: return "MSDA_SUCCESS";
    case MSDA_ERROR_INVALID_ARGUMENT: return "MSDA_ERROR_INVALID_ARGUMENT";
    case MSDA_ERROR_UNSUPPORTED_DTYPE: return "MSDA_ERROR_UNSUPPORTED_DTYPE";
    case MSDA_ERROR_SHAPE_MISMATCH: return "MSDA_ERROR_SHAPE_MISMATCH";
    case MSDA_ERROR_TOO_MANY_LEVELS: return "MSDA_ERROR_TOO_MANY_LEVELS";
    case MSDA_ERROR_INT32_OVERFLOW: return "MSDA_ERROR_INT32_OVERFLOW";
    case MSDA_ERROR_MISALIGNED: return "MSDA_ERROR_MISALIGNED";
    case MSDA_ERROR_WORKSPACE: return "MSDA_ERROR_WORKSPACE";
    case MSDA_ERROR_UNSUPPORTED_CHANNELS: return "MSDA_ERROR_UNSUPPORTED_CHANNELS";
    case MSDA_ERROR_CUDA: return "MSDA_ERROR_CUDA";
    default: return "MSDA_ERROR_UNKNOWN";
  }
}

const char* msda_last_error(void) { return msda::g_last_error; }

int msda_abi_version(void) { return MSDA_B200_ABI_VERSION; }

#ifdef MSDA_CHECKED
// Checked build only (include/msda_b200_checked.h): the bounds-check bits
// recorded on the current device since the last clear; waits for the device.
MSDA_API unsigned int msda_checked_violations(int clear) {
  unsigned int* w = msda::check_word();
  if (w == nullptr) return 0xffffffffu;
  unsigned int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return 0xffffffffu;
  if (clear && cudaMemset(w, 0, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  return v;
}
#endif

}  // extern "C"
