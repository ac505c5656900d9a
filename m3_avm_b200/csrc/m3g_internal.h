// m3g_internal.h -- host/device interface between the C ABI and the kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace m3g {

// Status bits the kernels set in the per-device error word.
enum : uint32_t {
  kStatusCopyTimeout = 1u,  // a staged-copy wait gave up
};

// Arguments of the staged streaming GEMV (k_gemv_stream).
struct StreamArgs {
  const uint8_t* w;   // weight bytes of rows [0, rows), row-major, RB bytes per row, 16-byte aligned
  const float* x;     // x[in_dim]
  float* y;           // y[rows]
  uint32_t* status;   // per-device error word
  int rows;           // output rows handled by this launch
  int RB;             // bytes per row (multiple of 16)
  int U;              // units per row = in_dim / unit elements
  int TS;             // threads per row slot (multiple of 32, >= ceil(U / UPT))
  int RPI;            // row slots per CTA (blockDim = TS * RPI)
  int R;              // rows per stage (multiple of RPI, <= TS)
  int NS;             // pipeline stages
  int stage_stride;   // bytes between stage buffers (>= R*RB + 16, multiple of 128)
  int rows_per_cta;   // contiguous rows per CTA
};

cudaError_t launch_gemv_stream(int fmt, const StreamArgs& a, int threads, int grid, size_t smem, int upt,
                               cudaStream_t st);
cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, long long in_dim,
                                long long nblocks, int grid, cudaStream_t st);
cudaError_t launch_dequant(int fmt, const uint8_t* w, float* out, long long n_elems, int grid, cudaStream_t st);

}  // namespace m3g
