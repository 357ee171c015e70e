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
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {

MSDA_DECLARE_PAIR(float, float)
MSDA_DECLARE_PAIR(__half, __half)
MSDA_DECLARE_PAIR(__half, float)
MSDA_DECLARE_PAIR(__nv_bfloat16, __nv_bfloat16)
MSDA_DECLARE_PAIR(__nv_bfloat16, float)
MSDA_DECLARE_BINNED(float, float)
MSDA_DECLARE_BINNED(__half, __half)
MSDA_DECLARE_BINNED(__half, float)
MSDA_DECLARE_BINNED(__nv_bfloat16, __nv_bfloat16)
MSDA_DECLARE_BINNED(__nv_bfloat16, float)

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
};

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
// The backward has two implementations: the gather/scatter kernel (any
// shape; fp32 atomics into grad_value or an fp32 workspace) and the binned
// tile kernel (msda_binned.cuh) for large problems with host-resident shapes
// and 16-byte channel rows.  The plan picks one and lays out the workspace.
constexpr int64_t kBinnedMinSamples = int64_t{1} << 18;
constexpr int kBinSmemBudget = 72 * 1024;    // three tile CTAs per SM
constexpr int64_t kAtomicLevelRecords = 8192;
constexpr int kMaxTilesPerBh = 24576;   // fill-pass histogram: 2 ints per tile in smem

// Gather path, 16-bit values: a level whose expected contributions per
// grad_value element (2^d corners x Q x P samples / voxels) stay at or below
// this bound reduces straight into grad_value in its own dtype -- the
// reference accumulates every level that way -- so its fp32 accumulator rows,
// their zero-fill and their cast disappear.  Busier levels keep fp32
// accumulation, which bounds their rounding error.
constexpr double kDirect16Contrib = 8.0;

struct BwdPlan {
  bool binned = false;
  BinPlan bp{};
  BinLaunch bl{};
  size_t off[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // counts, starts, cursor, item_start, item_counter, scan_tmp, records, acc
  size_t ws_bytes = 0;
  // gather path
  int32_t direct16 = 0;   // levels reduced straight into grad_value
  bool compact = false;   // fp32 accumulator holds only the other levels
  int64_t acc_keys = 0;   // keys per batch entry in the fp32 accumulator
  int32_t acc_start[kMaxLevels] = {};
};

// Gather-path value-gradient targets (see kDirect16Contrib).
void plan_gather_targets(const Args& a, const Problem& p, BwdPlan& pl) {
  pl.acc_keys = a.K;
  if (dtype_bytes(a.vdt) != 2 || p.shapes_dev != nullptr || a.K == 0) return;
  const char* env = std::getenv("MSDA_BWD_DIRECT16");
  if (env && std::strcmp(env, "0") == 0) return;
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

size_t align256(size_t x) { return (x + 255) & ~size_t{255}; }

// Shared memory of the tile kernel for a tile shape: value tile + halo + one
// zero row, and the tile's fp32 value gradient.
int64_t tile_smem_bytes(int ndim, const int32_t* t, int64_t row_bytes, int64_t C, int G) {
  const int64_t halo = int64_t{t[0] + 1} * (t[1] + 1) * (ndim == 3 ? t[2] + 1 : 1);
  const int64_t vox = int64_t{t[0]} * t[1] * t[2];
  (void)G;
  return (halo + 1) * row_bytes + vox * C * 4;
}

bool choose_tile(int ndim, int64_t row_bytes, int64_t C, int G, int budget, int32_t* tile,
                 int* smem) {
  static const int32_t c3[][3] = {{8, 8, 8}, {8, 8, 4}, {8, 4, 4}, {4, 4, 4}, {4, 4, 2}, {4, 2, 2}, {2, 2, 2}};
  static const int32_t c2[][3] = {{32, 16, 1}, {16, 16, 1}, {16, 8, 1}, {8, 8, 1}, {8, 4, 1}, {4, 4, 1}, {2, 2, 1}};
  const char* env = std::getenv("MSDA_BIN_TILE");
  int32_t forced[3] = {0, 0, 1};
  if (env && std::sscanf(env, "%d,%d,%d", &forced[0], &forced[1], &forced[2]) >= 2) {
    if (ndim == 2) forced[2] = 1;
  } else {
    forced[0] = 0;
  }
  for (int i = -1; i < 7; ++i) {
    const int32_t* t = i < 0 ? forced : (ndim == 3 ? c3[i] : c2[i]);
    if (t[0] <= 0 || t[1] <= 0 || t[2] <= 0) continue;
    const int64_t bytes = tile_smem_bytes(ndim, t, row_bytes, C, G);
    if (bytes <= budget || (i < 0 && bytes <= 200 * 1024)) {
      tile[0] = t[0]; tile[1] = t[1]; tile[2] = t[2];
      *smem = static_cast<int>(bytes);
      return true;
    }
  }
  return false;
}

void plan_bwd(const Args& a, const Problem& p, const LaunchShape& ls, BwdPlan& pl) {
  const int64_t e = dtype_bytes(a.vdt);
  const int64_t samples = a.B * a.Q * a.H * a.L * a.P;
  pl = BwdPlan{};
  const char* env = std::getenv("MSDA_BWD_PATH");
  // The binned path is opt-in (MSDA_BWD_PATH=binned) until it outruns the
  // gather/scatter kernel on the benchmark shapes.
  const bool force_binned = env && std::strcmp(env, "binned") == 0 && !a.fused;
  const bool force_gather = !force_binned;
  bool ok_binned = !force_gather && p.shapes_dev == nullptr && ls.vb == 16 && ls.vpl == 1 &&
                   samples > 0 && a.C > 0 && (force_binned || samples >= kBinnedMinSamples) &&
                   a.P <= 16 && a.Q < (int64_t{1} << 26) && a.L * a.P <= 512 &&
                   samples * (int64_t{1} << a.ndim) < INT32_MAX;
  for (int64_t l = 0; ok_binned && l < a.L; ++l)
    for (int ax = 0; ax < 3; ++ax) ok_binned = ok_binned && p.lv.size[l][ax] > 0;
  int smem = 0;
  BinPlan& bp = pl.bp;
  if (ok_binned) {
    const char* sb = std::getenv("MSDA_BIN_SMEM_KB");
    const int budget = sb ? std::atoi(sb) * 1024 : kBinSmemBudget;
    ok_binned = choose_tile(a.ndim, a.C * e, a.C, 1 << p.log2g, budget, bp.tile, &smem);
  }
  if (ok_binned) {
    int64_t ntl = 0;
    const double straddle = (1.0 + 1.0 / bp.tile[0]) * (1.0 + 1.0 / bp.tile[1]) *
                            (a.ndim == 3 ? 1.0 + 1.0 / bp.tile[2] : 1.0);
    int64_t acc_keys = 0;
    // Tuning / test knobs: records per tile above which a level reduces
    // through the fp32 accumulator, and records per work item there.
    const char* ar = std::getenv("MSDA_BIN_ATOMIC_RECORDS");
    const int64_t atomic_records = ar ? std::atoll(ar) : kAtomicLevelRecords;
    const char* sm = std::getenv("MSDA_BIN_SMAX");
    bp.s_max = sm && std::atoi(sm) > 0 ? std::atoi(sm) : 2048;
    for (int64_t l = 0; l < a.L; ++l) {
      int64_t nt = 1;
      for (int ax = 0; ax < 3; ++ax) {
        bp.ntile[l][ax] = (p.lv.size[l][ax] + bp.tile[ax] - 1) / bp.tile[ax];
        nt *= bp.ntile[l][ax];
      }
      bp.tile_base[l] = static_cast<int32_t>(ntl);
      ntl += nt;
      const double expect = static_cast<double>(a.Q * a.P) * straddle / static_cast<double>(nt);
      if (expect > static_cast<double>(atomic_records)) {
        bp.atomic_mask |= 1 << l;
        const int64_t nkey = int64_t{p.lv.size[l][0]} * p.lv.size[l][1] * p.lv.size[l][2];
        bp.acc_start[l] = static_cast<int32_t>(a.vdt == MSDA_FLOAT32 ? p.lv.start[l] : acc_keys);
        acc_keys += nkey;
      }
    }
    if (a.vdt == MSDA_FLOAT32) acc_keys = a.K;
    ok_binned = ntl <= kMaxTilesPerBh;
    bp.ntl = static_cast<int32_t>(ntl);
    bp.acc_keys = acc_keys;
    const int64_t rpc = std::max<int64_t>(1, 32768 / std::max<int64_t>(1, a.L * a.P));
    bp.rows_per_chunk = static_cast<int32_t>(rpc);
    bp.nchunk = static_cast<int32_t>((a.Q + rpc - 1) / rpc);
    bp.nlevels = static_cast<int32_t>(a.L);
  }
  if (!ok_binned) {
    pl.binned = false;
    plan_gather_targets(a, p, pl);
    pl.ws_bytes = (a.vdt == MSDA_FLOAT32)
                      ? 0 : static_cast<size_t>(a.B * pl.acc_keys * a.H * a.C) * sizeof(float);
    return;
  }
  pl.binned = true;
  const int64_t nb = a.B * a.H * bp.ntl;
  pl.bl.ndim = a.ndim;
  pl.bl.nb = nb;
  pl.bl.smem_main = smem;
  pl.bl.fp32_value = a.vdt == MSDA_FLOAT32;
  const int64_t scan_blocks = (nb + 1 + kScanThreads * kScanItems - 1) / (kScanThreads * kScanItems);
  const int64_t max_records = samples * (int64_t{1} << a.ndim);
  const size_t sizes[8] = {
      static_cast<size_t>(nb) * 4, static_cast<size_t>(nb + 1) * 4, static_cast<size_t>(nb) * 4,
      static_cast<size_t>(nb + 1) * 4, 4, static_cast<size_t>(scan_blocks + 1) * 4,
      static_cast<size_t>(max_records) * 4,
      (bp.atomic_mask && a.vdt != MSDA_FLOAT32)
          ? static_cast<size_t>(a.B * bp.acc_keys * a.H * a.C) * sizeof(float) : 0};
  size_t off = 0;
  for (int i = 0; i < 8; ++i) {
    pl.off[i] = off;
    off += align256(sizes[i]);
  }
  pl.ws_bytes = off;
}

cudaError_t dispatch_bwd_binned(int vdt, int sdt, const BinLaunch& bl, const Problem& p,
                                const BinPlan& bp, const BinBuffers& bb, const void* go, void* gv,
                                void* gl, void* ga, cudaStream_t st) {
  switch (vdt) {
    case MSDA_FLOAT32: return launch_bwd_binned<float, float>(bl, p, bp, bb, go, gv, gl, ga, st);
    case MSDA_FLOAT16:
      return sdt == MSDA_FLOAT32
                 ? launch_bwd_binned<__half, float>(bl, p, bp, bb, go, gv, gl, ga, st)
                 : launch_bwd_binned<__half, __half>(bl, p, bp, bb, go, gv, gl, ga, st);
    default:
      return sdt == MSDA_FLOAT32
                 ? launch_bwd_binned<__nv_bfloat16, float>(bl, p, bp, bb, go, gv, gl, ga, st)
                 : launch_bwd_binned<__nv_bfloat16, __nv_bfloat16>(bl, p, bp, bb, go, gv, gl,
                                                                   ga, st);
  }
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
  cudaError_t err;
  if (pl.binned) {
    char* w = static_cast<char*>(ws);
    BinBuffers bb;
    bb.counts = reinterpret_cast<int32_t*>(w + pl.off[0]);
    bb.starts = reinterpret_cast<int32_t*>(w + pl.off[1]);
    bb.cursor = reinterpret_cast<int32_t*>(w + pl.off[2]);
    bb.item_start = reinterpret_cast<int32_t*>(w + pl.off[3]);
    bb.item_counter = reinterpret_cast<int32_t*>(w + pl.off[4]);
    bb.scan_tmp = reinterpret_cast<int32_t*>(w + pl.off[5]);
    bb.records = reinterpret_cast<int32_t*>(w + pl.off[6]);
    bb.acc = a.vdt == MSDA_FLOAT32 ? static_cast<float*>(gv) : reinterpret_cast<float*>(w + pl.off[7]);
    err = dispatch_bwd_binned(a.vdt, a.sdt, pl.bl, p, pl.bp, bb, go, gv, gl, ga, st);
    if (err != cudaSuccess) return cuda_fail(err, "binned backward launch");
    return ok();
  }
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
    err = cudaMemset2DAsync(static_cast<char*>(gv) + p.lv.start[l] * row_bytes,
                            static_cast<size_t>(a.K * row_bytes), 0,
                            static_cast<size_t>(nvox * row_bytes), static_cast<size_t>(a.B), st);
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
  Args a{ND,    value, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes, \
         spatial_shapes_on_device, num_levels, sampling_locations, attention_weights,      \
         sampling_dtype, num_queries, num_points, clamp_grid, clamp_eps}

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
  Args a{ND,          value,           value_dtype,     batch,        num_keys,               \
         num_heads,   channels,        spatial_shapes,  spatial_shapes_on_device, num_levels, \
         sampling_offsets, attention_logits, sampling_dtype, num_queries, num_points,          \
         clamp_grid,  clamp_eps,       reference_points, 1}

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

static size_t workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                              int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                              int spatial_shapes_on_device, int64_t num_levels,
                              int64_t num_queries, int64_t num_points, int fused) {
  // Plan with 256-byte aligned stand-in pointers (never dereferenced).
  void* fake = reinterpret_cast<void*>(uintptr_t{256});
  Args a{ndim, fake, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
         spatial_shapes_on_device, num_levels, fake, fake, value_dtype, num_queries, num_points,
         1, 1e-4, static_cast<const float*>(fake), fused};
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
