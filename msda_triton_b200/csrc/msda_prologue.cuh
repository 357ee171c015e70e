// msda_prologue.cuh -- the sampling prologue of the MSDA modules as its own
// pass, for problems that run the unfused kernels (the cell-sorted backward
// has no fused variant):
//   forward:  sampling_locations = reference_points + sampling_offsets / size
//             attention_weights  = softmax over each (b, q, h) row's L*P logits
//   backward: the offsets', logits' and (summed over points) reference
//             points' gradients.
// Reference: MSDA2D/MSDA3D.forward (pytorch/msda_3d.py:325-350,
// pytorch/msda_2d.py:325-339), where these are separate tensor operations.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace msda {

struct PrologueArgs {
  int ndim;
  int64_t B, Q, H, L, P;
  int32_t size[16][3];   // per level and axis (x, y, z): W, H, D
  const void* ref;       // (B, Q, L, d)
  const void* off;       // (B, Q, H, L, P, d)
  const void* logits;    // (B, Q, H, L*P)
  const void* weights;   // backward: the forward's attention weights
  const void* gloc;      // backward: grad of sampling_locations
  const void* gattn;     // backward: grad of attention_weights
  void* loc;             // forward outputs
  void* wout;
  float* gref_partial;   // backward outputs: (B, Q, H, L, d) fp32, summed over points
  void* goff;
  void* glogits;
};

// dtype: MSDA_FLOAT32 / MSDA_FLOAT16 / MSDA_BFLOAT16 (every tensor in it).
cudaError_t prologue_fwd(const PrologueArgs& a, int dtype, cudaStream_t st);
cudaError_t prologue_bwd(const PrologueArgs& a, int dtype, cudaStream_t st);

}  // namespace msda
