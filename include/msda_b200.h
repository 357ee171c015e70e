/*
 * msda_b200.h -- C ABI of the B200 (sm_100a) multi-scale deformable attention
 * library, libmsda_b200.so.
 *
 * This is the drop-in boundary for the reference's hot path.  The reference
 * (mach9robotics/msda-triton) exposes the path as Python functions; each
 * entry point below replaces one of them, with the same tensor contract and
 * argument meaning:
 *
 *   msda2d_fwd  <- msda2d_fwd / _msda2d_fwd_prepared
 *                  (src/msda_triton/triton/msda_2d.py:654-718, :586-651)
 *   msda3d_fwd  <- msda3d_fwd / _msda3d_fwd_prepared
 *                  (src/msda_triton/triton/msda_3d.py:797-861, :729-794)
 *   msda2d_bwd  <- MSDA2DFn.backward (src/msda_triton/triton/msda_2d.py:777-853)
 *   msda3d_bwd  <- MSDA3DFn.backward (src/msda_triton/triton/msda_3d.py:920-996)
 *
 * Tensor contract (all buffers dense, row-major, on the current CUDA device):
 *   value               (B, K, H, C)        value_dtype
 *   spatial_shapes      (L, d) int32        rows (H, W) for 2D, (D, H, W) for 3D;
 *                                           host or device memory (see below)
 *   sampling_locations  (B, Q, H, L, P, d)  sampling_dtype, normalised to [0, 1]
 *   attention_weights   (B, Q, H, L, P)     sampling_dtype
 *   output              (B, Q, H*C)         value_dtype
 *   grad_value          like value; grad_sampling_locations / grad_attention_weights
 *                       like their inputs.
 * d = 2 for the msda2d_* entry points and 3 for msda3d_*.  K must equal
 * sum over levels of prod(shape); it is checked when the shapes are in host
 * memory (as the reference does, triton/msda_2d.py:53-74).  Device-resident
 * shapes are read by the kernels without a host synchronisation and are not
 * checked against K (reference: triton/msda_2d.py:76-82); a level that would
 * reach past K contributes nothing.
 *
 * Semantics: bilinear (2D) / trilinear (3D) sampling with align_corners=False
 * and zero padding, as torch.nn.functional.grid_sample; when clamp_grid is
 * non-zero the grid coordinate 2*loc-1 is clamped to [-1+eps, 1-eps] and the
 * location gradient is zero where the clamp is active.  Accumulation is fp32
 * for every dtype.
 *
 * Memory and threading: the caller owns every buffer.  The library allocates
 * nothing; the backward needs a workspace of msda_bwd_workspace_bytes() bytes
 * (256-byte aligned).  Every call is asynchronous
 * on `stream` (a cudaStream_t; NULL = legacy default stream) and keeps no
 * state between calls, so calls on different streams may run concurrently
 * (except msda_bwd_static_scratch, whose calls share one scratch array).
 * grad_* buffers need no initialisation: they are fully overwritten.
 *
 * Errors: every entry point returns MSDA_SUCCESS (0) or an msda_status code;
 * msda_status_string() names the code and msda_last_error() returns a
 * message describing the most recent failure on the calling thread.
 */
#ifndef MSDA_B200_H_
#define MSDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MSDA_API __attribute__((visibility("default")))
#else
#define MSDA_API
#endif

#define MSDA_B200_ABI_VERSION 3
#define MSDA_MAX_LEVELS 16

typedef enum msda_dtype {
  MSDA_FLOAT32 = 0,
  MSDA_FLOAT16 = 1,
  MSDA_BFLOAT16 = 2
} msda_dtype;

/* Flag ORed into any `value_dtype` argument: value (and grad_value) are laid
 * out head-major, (B, H, K, C) -- each head's keys contiguous -- instead of
 * the reference's (B, K, H, C).  This is the layout a value projection can
 * write per head (pytorch/msda_3d.py:302-305 views its output as
 * (B, K, H, C)); one head's slice of a level is then one contiguous range,
 * which stays in L2 while the kernels walk that head.  Every other argument
 * keeps its meaning; workspace sizes do not change.  No counterpart in the
 * reference. */
#define MSDA_VALUE_HEAD_MAJOR 0x100

typedef enum msda_status {
  MSDA_SUCCESS = 0,
  MSDA_ERROR_INVALID_ARGUMENT = 1,   /* null pointer, negative size, bad clamp_eps */
  MSDA_ERROR_UNSUPPORTED_DTYPE = 2,  /* dtype outside fp32/fp16/bf16, or an unsupported pairing */
  MSDA_ERROR_SHAPE_MISMATCH = 3,     /* K != sum of level sizes (host shapes only) */
  MSDA_ERROR_TOO_MANY_LEVELS = 4,    /* L > MSDA_MAX_LEVELS */
  MSDA_ERROR_INT32_OVERFLOW = 5,     /* K or B*Q*H exceeds the int32 range */
  MSDA_ERROR_MISALIGNED = 6,         /* a buffer is not aligned to its element size */
  MSDA_ERROR_WORKSPACE = 7,          /* workspace missing, too small or misaligned */
  MSDA_ERROR_UNSUPPORTED_CHANNELS = 8, /* C * sizeof(value_dtype) above 2048 bytes */
  MSDA_ERROR_CUDA = 9                /* a CUDA runtime call or launch failed */
} msda_status;

/* Forward pass.  sampling_dtype must equal value_dtype or be MSDA_FLOAT32.
 * Replaces msda2d_fwd (src/msda_triton/triton/msda_2d.py:654-718). */
MSDA_API int msda2d_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, void* output, void* stream);

/* Replaces msda3d_fwd (src/msda_triton/triton/msda_3d.py:797-861). */
MSDA_API int msda3d_fwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, void* output, void* stream);

/* Backward pass: all three gradients in one pass.
 * Replaces MSDA2DFn.backward (src/msda_triton/triton/msda_2d.py:777-853). */
MSDA_API int msda2d_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, void* grad_value,
               void* grad_sampling_locations, void* grad_attention_weights, void* workspace,
               size_t workspace_bytes, void* stream);

/* Replaces MSDA3DFn.backward (src/msda_triton/triton/msda_3d.py:920-996). */
MSDA_API int msda3d_bwd(const void* value, int value_dtype, int64_t batch, int64_t num_keys,
               int64_t num_heads, int64_t channels, const int32_t* spatial_shapes,
               int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, void* grad_value,
               void* grad_sampling_locations, void* grad_attention_weights, void* workspace,
               size_t workspace_bytes, void* stream);

/* Backward scatter only: ADDS the value gradient, in fp32, into
 * grad_value_accum (B, K, H, C) -- which the caller must have initialised
 * (zero, or a partial sum to extend) -- and writes grad_sampling_locations /
 * grad_attention_weights like msda{2,3}d_bwd.  No memset, no cast, no
 * workspace.  msda{2,3}d_bwd = zero-fill + this + msda_cast_from_f32; the split
 * lets a caller sum partial value gradients (e.g. queries sharded across GPUs
 * and reduced with NCCL) before one final cast.  grad_value_accum must be
 * 16-byte aligned.  Same reference counterpart as msda{2,3}d_bwd. */
MSDA_API int msda2d_bwd_accumulate(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, float* grad_value_accum,
               void* grad_sampling_locations, void* grad_attention_weights, void* stream);

MSDA_API int msda3d_bwd_accumulate(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, float* grad_value_accum,
               void* grad_sampling_locations, void* grad_attention_weights, void* stream);

/* Round `count` fp32 values to dst_dtype (float32 copies).  The final step of
 * the backward for fp16/bf16 values (the reference's grads are in the input
 * dtype, triton/msda_3d.py:941-944).  src 16-byte aligned. */
MSDA_API int msda_cast_from_f32(const float* src, void* dst, int dst_dtype, int64_t count,
                                void* stream);

/* Workspace bytes msda{2,3}d_bwd needs for this problem (it depends on the
 * level shapes, which must be the same pointer/residency as in the call).
 * The plan it sizes:
 *  - host-resident shapes and at least 2^20 samples: the cell-sorted
 *    backward -- bucket counts per cell of every level and (b, h), a rank
 *    and a 32-byte record per sample, 16 bytes per sample of the levels whose
 *    dot products run in sorted order, and (fp16/bf16 values) an fp32
 *    accumulator for the levels with more than 2 samples per cell;
 *  - otherwise the gather/scatter backward: none for fp32 values, an fp32
 *    accumulator of B*K*H*C*4 bytes for fp16/bf16 values.
 * Every value-gradient sum is carried in fp32 and rounded once.  The plan
 * assumes value, grad_output and grad_value are 16-byte aligned.  The
 * reference allocates its gradient buffers with torch.zeros_like
 * (triton/msda_3d.py:941-944); here the caller allocates.
 * Returns 0 when no workspace is needed or the arguments are invalid. */
MSDA_API size_t msda_bwd_workspace_bytes(int ndim, int value_dtype, int64_t batch,
                                         int64_t num_keys, int64_t num_heads, int64_t channels,
                                         const int32_t* spatial_shapes,
                                         int spatial_shapes_on_device, int64_t num_levels,
                                         int64_t num_queries, int64_t num_points);

/* Backward pass that allocates nothing, for callers that cannot allocate
 * device memory (an inference-engine plugin whose enqueue must not call
 * cudaMalloc, code running while another framework owns the device memory
 * pool, an FFI without access to a CUDA allocator).  No counterpart in the
 * reference: it is msda{2,3}d_bwd (ndim = 2 or 3) with the workspace taken
 * from a 32 MiB array inside the library's device image, reserved on every
 * GPU that loads the library until the process exits.  Problems needing more
 * than 32 MiB of scratch (msda_bwd_workspace_bytes) are rejected with
 * MSDA_ERROR_WORKSPACE.  The first call on a device, and the first call
 * after the current driver context changed (another context made current,
 * or a cudaDeviceReset that destroyed the old one), looks up the array's
 * device address (cudaGetSymbolAddress) and caches it for that context;
 * make such a call outside any stream capture.  All calls share the array:
 * calls whose GPU work overlaps on one device race; serialise them.  Each
 * call clears what it uses. */
MSDA_API int msda_bwd_static_scratch(int ndim, const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const void* sampling_locations, const void* attention_weights,
               int sampling_dtype, int64_t num_queries, int64_t num_points, int clamp_grid,
               double clamp_eps, const void* grad_output, void* grad_value,
               void* grad_sampling_locations, void* grad_attention_weights, void* stream);

/* Fused prologue: MSDA from the raw outputs of a deformable-attention
 * layer's two query projections instead of finished locations and weights
 * (the MSDA2D / MSDA3D modules, src/msda_triton/pytorch/msda_2d.py:325-339,
 * src/msda_triton/pytorch/msda_3d.py:325-350, compute them as separate
 * tensors first):
 *   reference_points  (B, Q, L, d) fp32, normalised
 *   sampling_offsets  (B, Q, H, L, P, d) sampling_dtype, in cells of the level
 *   attention_logits  (B, Q, H, L*P)     sampling_dtype
 * location = reference_points[b,q,l] + sampling_offsets[b,q,h,l,p] / (W, H[, D])_l
 * weight   = softmax over the L*P logits of row (b, q, h)
 * and then exactly msda{2,3}d_fwd.  The backward writes grad_value,
 * grad_sampling_offsets and grad_attention_logits (in the dtypes of their
 * inputs) and grad_reference_partial, fp32 (B, Q, H, L, d): the sum over the
 * row's points of the location gradient; the reference-point gradient is its
 * sum over H (one small reduction by the caller).  Workspace: see
 * msda_fused_bwd_workspace_bytes. */
MSDA_API int msda2d_fused_fwd(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const float* reference_points, const void* sampling_offsets,
               const void* attention_logits, int sampling_dtype, int64_t num_queries,
               int64_t num_points, int clamp_grid, double clamp_eps, void* output, void* stream);

MSDA_API int msda3d_fused_fwd(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const float* reference_points, const void* sampling_offsets,
               const void* attention_logits, int sampling_dtype, int64_t num_queries,
               int64_t num_points, int clamp_grid, double clamp_eps, void* output, void* stream);

MSDA_API int msda2d_fused_bwd(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const float* reference_points, const void* sampling_offsets,
               const void* attention_logits, int sampling_dtype, int64_t num_queries,
               int64_t num_points, int clamp_grid, double clamp_eps, const void* grad_output,
               void* grad_value, float* grad_reference_partial, void* grad_sampling_offsets,
               void* grad_attention_logits, void* workspace, size_t workspace_bytes,
               void* stream);

MSDA_API int msda3d_fused_bwd(const void* value, int value_dtype, int64_t batch,
               int64_t num_keys, int64_t num_heads, int64_t channels,
               const int32_t* spatial_shapes, int spatial_shapes_on_device, int64_t num_levels,
               const float* reference_points, const void* sampling_offsets,
               const void* attention_logits, int sampling_dtype, int64_t num_queries,
               int64_t num_points, int clamp_grid, double clamp_eps, const void* grad_output,
               void* grad_value, float* grad_reference_partial, void* grad_sampling_offsets,
               void* grad_attention_logits, void* workspace, size_t workspace_bytes,
               void* stream);

/* The same prologue as its own pass, for problems that run the unfused
 * entries (the cell-sorted backward has no fused form).  It replaces the
 * tensor operations of the modules (src/msda_triton/pytorch/msda_3d.py:
 * 336-350, src/msda_triton/pytorch/msda_2d.py:325-339).  spatial_shapes:
 * host, the reference's order per level; every tensor in sampling_dtype:
 *   reference_points (B, Q, L, d), sampling_offsets (B, Q, H, L, P, d),
 *   attention_logits (B, Q, H, L*P) ->
 *   sampling_locations (B, Q, H, L, P, d), attention_weights (B, Q, H, L, P)
 * A location has the rounding of `reference_points + sampling_offsets /
 * normalizer` in sampling_dtype (size converted to it, quotient rounded,
 * then the sum); the weights are the fused entries' row softmax.  The
 * backward takes the forward's attention_weights and the two gradients and
 * writes grad_sampling_offsets, grad_attention_logits (sampling_dtype) and
 * grad_reference_partial, fp32 (B, Q, H, L, d): the sum over points of the
 * location gradient (its sum over H is the reference-point gradient).
 * L*P is at most 2048 (MSDA_ERROR_INVALID_ARGUMENT above). */
MSDA_API int msda_prologue_fwd(int ndim, int64_t batch, int64_t num_queries, int64_t num_heads,
               int64_t num_levels, int64_t num_points, const int32_t* spatial_shapes,
               const void* reference_points, const void* sampling_offsets,
               const void* attention_logits, int sampling_dtype, void* sampling_locations,
               void* attention_weights, void* stream);

MSDA_API int msda_prologue_bwd(int ndim, int64_t batch, int64_t num_queries, int64_t num_heads,
               int64_t num_levels, int64_t num_points, const int32_t* spatial_shapes,
               const void* attention_weights, const void* grad_sampling_locations,
               const void* grad_attention_weights, int sampling_dtype,
               float* grad_reference_partial, void* grad_sampling_offsets,
               void* grad_attention_logits, void* stream);

/* Workspace bytes of msda{2,3}d_fused_bwd (always the gather/scatter plan). */
MSDA_API size_t msda_fused_bwd_workspace_bytes(int ndim, int value_dtype, int64_t batch,
                                               int64_t num_keys, int64_t num_heads,
                                               int64_t channels, const int32_t* spatial_shapes,
                                               int spatial_shapes_on_device, int64_t num_levels,
                                               int64_t num_queries, int64_t num_points);

/* Name of a status code ("MSDA_SUCCESS", ...). */
MSDA_API const char* msda_status_string(int status);

/* Human-readable detail of the last failure on the calling thread ("" if none). */
MSDA_API const char* msda_last_error(void);

/* MSDA_B200_ABI_VERSION of the loaded library. */
MSDA_API int msda_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MSDA_B200_H_ */
