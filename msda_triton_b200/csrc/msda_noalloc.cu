// msda_noalloc.cu -- the backward pass for callers that cannot allocate
// device memory.
//
// msda{2,3}d_bwd take their scratch (the fp32 value-gradient accumulator for
// fp16/bf16 inputs) from a caller-provided workspace.  Some callers cannot
// provide one: an inference-engine plugin whose enqueue step may not call
// cudaMalloc, code running while another framework owns the whole device
// memory pool, or a host language whose FFI has no access to a CUDA
// allocator.  msda_bwd_static_scratch serves them from a fixed array that is
// part of this library's device image instead: it allocates nothing.
//
// The array (kStaticScratchBytes) is reserved on every GPU that loads the
// library, for as long as the process lives (a device reset gives a new
// context and a new array, which the next call looks up).  Every call shares
// it, so calls whose GPU work overlaps -- on different streams, or from different host
// threads, on the same device -- race on it; serialise them (one stream) or
// use msda{2,3}d_bwd with separate workspaces.  The region a call uses is
// cleared by that call (the previous call's contents remain until then).
#include <cstdio>
#include <mutex>

#include "../../include/msda_b200.h"

namespace msda {
// msda_capi.cu: feeds msda_last_error(); the gather/scatter-plan backward
// and its workspace size.
int set_last_error(int code, const char* msg);
size_t scatter_workspace_bytes(int ndim, int value_dtype, int64_t batch, int64_t num_keys,
                               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                               int spatial_shapes_on_device, int64_t num_levels,
                               int64_t num_queries, int64_t num_points);
int bwd_scatter(int ndim, const void* value, int value_dtype, int64_t batch, int64_t num_keys,
                int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
                int spatial_shapes_on_device, int64_t num_levels, const void* sampling_locations,
                const void* attention_weights, int sampling_dtype, int64_t num_queries,
                int64_t num_points, int clamp_grid, double clamp_eps, const void* grad_output,
                void* grad_value, void* grad_sampling_locations, void* grad_attention_weights,
                void* workspace, size_t workspace_bytes, void* stream);
}  // namespace msda

namespace {

constexpr size_t kStaticScratchBytes = size_t{32} << 20;  // 32 MiB per device
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_setup_mutex;
// Per device: the driver context the address was looked up in, and the
// address.  A device reset or another context current on the device gives a
// new context, whose array has its own address: it is looked up again.
struct ScratchAddr {
  void* ctx = nullptr;
  void* addr = nullptr;
};
ScratchAddr g_scratch_addr[kMaxDevices];

int noalloc_fail(int code, const char* msg) { return msda::set_last_error(code, msg); }

// The driver context current on the calling thread (cuCtxGetCurrent through
// the runtime's entry-point lookup, so the library links no driver library).
void* current_context() {
  using GetCurrent = int (*)(void**);
  static GetCurrent fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<GetCurrent>(f);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in; the real address must come
// from cudaGetSymbolAddress with the device current.  Done once per device
// and context.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return noalloc_fail(MSDA_ERROR_CUDA, cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(MSDA_ERROR_INVALID_ARGUMENT, "device ordinal out of range");
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  ScratchAddr& c = g_scratch_addr[dev];
  if (c.addr == nullptr || ctx == nullptr || c.ctx != ctx) {
    void* p = nullptr;
    // with no context current yet, this makes the device's primary one current
    err = cudaGetSymbolAddress(&p, g_static_scratch);
    if (err != cudaSuccess || p == nullptr)
      return noalloc_fail(MSDA_ERROR_CUDA, err != cudaSuccess ? cudaGetErrorString(err)
                                                              : "null scratch address");
    c.ctx = current_context();
    c.addr = p;
  }
  *out = c.addr;
  return MSDA_SUCCESS;
}

}  // namespace

extern "C" MSDA_API int msda_bwd_static_scratch(
    int ndim, const void* value, int value_dtype, int64_t batch, int64_t num_keys,
    int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
    int spatial_shapes_on_device, int64_t num_levels, const void* sampling_locations,
    const void* attention_weights, int sampling_dtype, int64_t num_queries, int64_t num_points,
    int clamp_grid, double clamp_eps, const void* grad_output, void* grad_value,
    void* grad_sampling_locations, void* grad_attention_weights, void* stream) {
  if (ndim != 2 && ndim != 3) return noalloc_fail(MSDA_ERROR_INVALID_ARGUMENT, "ndim must be 2 or 3");
  const size_t need = msda::scatter_workspace_bytes(ndim, value_dtype, batch, num_keys,
                                                    num_heads, channels, spatial_shapes,
                                                    spatial_shapes_on_device, num_levels,
                                                    num_queries, num_points);
  if (need > kStaticScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "problem needs %zu bytes of backward scratch; the static scratch holds %zu bytes "
             "(use msda%dd_bwd with a caller workspace)",
             need, kStaticScratchBytes, ndim);
    return noalloc_fail(MSDA_ERROR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != MSDA_SUCCESS) return rc;
  // The regular backward zero-fills the part of the workspace it uses.
  rc = msda::bwd_scatter(
      ndim, value, value_dtype, batch, num_keys, num_heads, channels, spatial_shapes,
      spatial_shapes_on_device, num_levels, sampling_locations, attention_weights,
      sampling_dtype, num_queries, num_points, clamp_grid, clamp_eps, grad_output, grad_value,
      grad_sampling_locations, grad_attention_weights, scratch, kStaticScratchBytes, stream);
  return rc;  // on failure msda_last_error() already describes it
}
