// m3g_vm.cu -- the VM's MATVEC and FFN opcodes on the device.
//
// exec_matvec (src/vm.rs:2643-2685): x [M, K] times W [K, N].  For M = 1 the
// reference calls matvec::matvec, the GGUF orientation y[j] = sum_i x[i] *
// W[i + j*K] -- the fused GEMV.  For M > 1 it reads the dequantised W as a
// row-major [K, N] array and multiplies with ndarray, y[m][j] = sum_k
// x[m][k] * W[k*N + j]; exec_ffn (src/vm.rs:2471-2576) always uses that
// row-major reading: hidden = x W1 + b1, gated = hidden * sigmoid(hidden),
// out = gated W2 + b2, a bias of length H (D_out) broadcast over the rows, of
// length M*H (M*D_out) per row, anything else zero.
//
// k_matvec_rowmajor computes the row-major form without dequantising W to
// memory: a CTA owns 256 consecutive output columns and a slice of k; each
// thread decodes its column's element of every row k in the slice exactly
// (the block decoders of src/quant.rs, blocks counted along the flat index
// k*N + j), multiplies it by x[m][k] for up to kVmRows rows of x held in
// shared memory, and adds its partials into y with one atomic per (row,
// column) -- y starts as the broadcast bias or zero.  The FFN's second product
// applies silu to its input as it loads it.
#include <algorithm>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/m3gemv.h"
#include "m3g_device.cuh"
#include "m3g_formats.cuh"
#include "m3g_internal.h"

namespace m3g {
int host_fail(int code, const char* fmt, ...);
bool block_geometry(uint32_t dtype, int* be, int* bb);
int gemv_device(int device, uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, float* y,
                long long in_dim, long long out_dim, cudaStream_t st);
}  // namespace m3g

namespace m3g {
namespace {

constexpr int kVmCols = 256;   // output columns per CTA (one thread each)
constexpr int kVmRows = 16;    // rows of x per launch
constexpr int kVmKSlice = 64;  // k values per CTA

__device__ __forceinline__ float elem_at(const uint8_t* w, int dtype, int be, int bb, long long idx) {
  if (dtype == 0) return reinterpret_cast<const float*>(w)[idx];
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(w)[idx]);
  const uint8_t* blk = w + (idx / be) * bb;
  const int off = static_cast<int>(idx % be);
  switch (dtype) {
    case 14: return q6k_elem(blk, off);
    case 8: return q8_0_elem(blk, off);
    case 2: return q4_0_elem(blk, off);
    default: return q4k_elem(blk, off);
  }
}

// y[m][j] += sum_{k in slice} f(x[m][k]) * W[k*sk + j*sj], m < rows (the
// row-major [K, N] reading is sk = N, sj = 1).
__global__ void __launch_bounds__(kVmCols) k_matvec_rowmajor(const float* __restrict__ x, int rows, int K,
                                                             const uint8_t* __restrict__ w, int dtype, int be,
                                                             int bb, int N, long long sk, long long sj,
                                                             float* __restrict__ y, int silu_x) {
  __shared__ float xs[kVmRows][kVmKSlice];
  const int j = blockIdx.x * kVmCols + threadIdx.x;
  const int k0 = blockIdx.y * kVmKSlice, k1 = min(K, k0 + kVmKSlice);
  for (int i = threadIdx.x; i < kVmRows * kVmKSlice; i += kVmCols) {
    const int m = i / kVmKSlice, k = k0 + i % kVmKSlice;
    float v = 0.f;
    if (m < rows && k < k1) {
      v = x[static_cast<long long>(m) * K + k];
      if (silu_x) v = v * (1.0f / (1.0f + expf(-v)));  // gated = v * sigmoid(v)
    }
    xs[m][i % kVmKSlice] = v;
  }
  __syncthreads();
  if (j >= N) return;
  float acc[kVmRows];
#pragma unroll
  for (int m = 0; m < kVmRows; ++m) acc[m] = 0.f;
  for (int k = k0; k < k1; ++k) {
    const float wv = elem_at(w, dtype, be, bb, static_cast<long long>(k) * sk + static_cast<long long>(j) * sj);
#pragma unroll
    for (int m = 0; m < kVmRows; ++m) acc[m] = fmaf(xs[m][k - k0], wv, acc[m]);
  }
  for (int m = 0; m < rows; ++m) atomicAdd(&y[static_cast<long long>(m) * N + j], acc[m]);
}

// y[m][j] = bias broadcast (len N), per row (len rows*N) or zero.
__global__ void k_bias_init(float* y, int rows, int N, const float* bias, long long bias_len) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(rows) * N) return;
  float v = 0.f;
  if (bias && bias_len == N) v = bias[i % N];
  else if (bias && bias_len == static_cast<long long>(rows) * N) v = bias[i];
  y[i] = v;
}

int rowmajor_product(const float* x, int M, int K, const uint8_t* w, uint32_t dtype, int N, const float* bias,
                     long long bias_len, bool silu_x, float* y, cudaStream_t st, bool gguf_orientation = false) {
  const long long sk = gguf_orientation ? 1 : N, sj = gguf_orientation ? K : 1;
  int be = 1, bb = 4;
  if (dtype == 1) bb = 2;
  else if (dtype != 0 && !block_geometry(dtype, &be, &bb)) return host_fail(M3G_ENONE, "dtype %u", dtype);
  const long long total = static_cast<long long>(M) * N;
  k_bias_init<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(y, M, N, bias, bias_len);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return host_fail(M3G_ECUDA, "bias init: %s", cudaGetErrorString(e));
  const dim3 grid(static_cast<unsigned>((N + kVmCols - 1) / kVmCols),
                  static_cast<unsigned>((K + kVmKSlice - 1) / kVmKSlice));
  for (int m0 = 0; m0 < M; m0 += kVmRows) {
    const int rows = std::min(kVmRows, M - m0);
    k_matvec_rowmajor<<<grid, kVmCols, 0, st>>>(x + static_cast<long long>(m0) * K, rows, K, w,
                                                 static_cast<int>(dtype), be, bb, N, sk, sj,
                                                 y + static_cast<long long>(m0) * N, silu_x ? 1 : 0);
    e = cudaGetLastError();
    if (e != cudaSuccess) return host_fail(M3G_ECUDA, "k_matvec_rowmajor: %s", cudaGetErrorString(e));
  }
  return M3G_OK;
}

// Bytes of n elements of a VM weight dtype (F32, F16 and the fused dtypes).
int weight_bytes(uint32_t dtype, uint64_t n, uint64_t* out) {
  if (dtype == 0) { *out = 4 * n; return M3G_OK; }
  if (dtype == 1) { *out = 2 * n; return M3G_OK; }
  int be = 0, bb = 0;
  if (!block_geometry(dtype, &be, &bb)) return host_fail(M3G_ENONE, "dtype %u has no decoder", dtype);
  if (n % static_cast<uint64_t>(be)) return host_fail(M3G_ENONE, "%llu elements are not whole blocks",
                                                     static_cast<unsigned long long>(n));
  *out = n / be * bb;
  return M3G_OK;
}

}  // namespace
}  // namespace m3g

extern "C" {

M3G_API int m3g_vm_matvec_dev(const float* x, uint64_t M, uint64_t K, const uint8_t* w, uint64_t w_len,
                              uint32_t dtype, uint64_t N, float* y, void* stream) {
  if (!x || !w || !y) return m3g::host_fail(M3G_EINVAL, "null argument");
  if (!M || !K || !N) return m3g::host_fail(M3G_ENONE, "zero dimension");
  if (M > (1u << 20) || K > 65535ull * 64 || N > (1u << 30) || K * N > (1ull << 40))
    return m3g::host_fail(M3G_EINVAL, "dimension too large");
  uint64_t need = 0;
  if (int rc = m3g::weight_bytes(dtype, K * N, &need)) return rc;
  if (w_len < need) return m3g::host_fail(M3G_ENONE, "W has %llu bytes, needs %llu",
                                          static_cast<unsigned long long>(w_len), static_cast<unsigned long long>(need));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  if (M == 1 && dtype != 0 && dtype != 1) {  // matvec::matvec: the GGUF orientation, the fused GEMV
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "no CUDA device");
    return m3g::gemv_device(dev, dtype, w, w_len, x, y, static_cast<long long>(K), static_cast<long long>(N), st);
  }
  // M = 1 with F32 / F16 weights keeps the GGUF orientation W[i + j*K]
  return m3g::rowmajor_product(x, static_cast<int>(M), static_cast<int>(K), w, dtype, static_cast<int>(N), nullptr,
                               0, false, y, st, M == 1);
}

M3G_API int m3g_vm_ffn_dev(const float* x, uint64_t M, uint64_t D, const uint8_t* w1, uint64_t w1_len,
                           uint32_t dtype1, uint64_t H, const uint8_t* w2, uint64_t w2_len, uint32_t dtype2,
                           uint64_t D_out, const float* b1, uint64_t b1_len, const float* b2, uint64_t b2_len,
                           float* y, void* stream) {
  if (!x || !w1 || !w2 || !y) return m3g::host_fail(M3G_EINVAL, "null argument");
  if (!M || !D || !H || !D_out) return m3g::host_fail(M3G_ENONE, "zero dimension");
  if (M > (1u << 20) || D > 65535ull * 64 || H > 65535ull * 64 || D_out > (1u << 30) || D * H > (1ull << 40) ||
      H * D_out > (1ull << 40))
    return m3g::host_fail(M3G_EINVAL, "dimension too large");
  uint64_t n1 = 0, n2 = 0;
  if (int rc = m3g::weight_bytes(dtype1, D * H, &n1)) return rc;
  if (int rc = m3g::weight_bytes(dtype2, H * D_out, &n2)) return rc;
  if (w1_len < n1 || w2_len < n2) return m3g::host_fail(M3G_ENONE, "weights shorter than their shapes");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  float* hidden = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&hidden), sizeof(float) * M * H, st);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ENOMEM, "FFN hidden: %s", cudaGetErrorString(e));
  int rc = m3g::rowmajor_product(x, static_cast<int>(M), static_cast<int>(D), w1, dtype1, static_cast<int>(H), b1,
                                 static_cast<long long>(b1_len), false, hidden, st);
  if (rc == M3G_OK)
    rc = m3g::rowmajor_product(hidden, static_cast<int>(M), static_cast<int>(H), w2, dtype2,
                               static_cast<int>(D_out), b2, static_cast<long long>(b2_len), true, y, st);
  cudaFreeAsync(hidden, st);
  return rc;
}

}  // extern "C"
