// m3g_kernels.cu -- sm_100a kernels of the fused dequantise-and-matvec path.
//
// k_gemv_stream<F, UPT>   the fast path: whole rows of GGUF blocks stream from
//                         HBM into a ring of shared-memory stages by 1-D TMA
//                         bulk copies (one elected thread, mbarrier
//                         completion), while every thread decodes its fixed
//                         units of each staged row against x held in
//                         registers; rows reduce with warp shuffles.
// k_gemv_generic<F>       any shape, including blocks that straddle two
//                         output rows (in_dim not a multiple of the block):
//                         one warp per block, exact decode, atomics per row.
// k_dequant<...>          bit-exact block decode to f32 (src/quant.rs:9-173).
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "m3g_device.cuh"
#include "m3g_formats.cuh"
#include "m3g_internal.h"

namespace m3g {

// Copy-wait limit of the staged pipeline: a stage normally lands within
// microseconds; after this long the kernel reports kStatusCopyTimeout.
constexpr uint64_t kCopyTimeoutNs = 2000000000ull;

template <class F, int UPT>
__global__ void __launch_bounds__(288) k_gemv_stream(const StreamArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int WPS = a.TS >> 5;               // consumer warps per row slot
  const int NC = a.TS * a.RPI;             // consumer threads
  const int NCW = NC >> 5;                 // consumer warps

  const long long row0 = static_cast<long long>(blockIdx.x) * a.rows_per_cta;
  long long row_end = row0 + a.rows_per_cta;
  if (row_end > a.rows) row_end = a.rows;
  if (row0 >= row_end) return;             // uniform across the CTA
  const int nrows = static_cast<int>(row_end - row0);
  const int nst = (nrows + a.R - 1) / a.R;

  float* xs = reinterpret_cast<float*>(smem + a.off_x);
  float* red = reinterpret_cast<float*>(smem + a.off_red);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + a.NS);
  const uint8_t* wbase = a.w + row0 * static_cast<long long>(a.RB);

  if (tid == 0) {
    for (int s = 0; s < a.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], static_cast<uint32_t>(NCW));
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------ producer warp
    uint64_t policy = 0;
    int issued = 0;
    auto issue = [&](int s) {
      const int rows_s = min(a.R, nrows - s * a.R);
      const uint32_t bytes = static_cast<uint32_t>(rows_s) * static_cast<uint32_t>(a.RB);
      const int b = s % a.NS;
      mbar_arrive_expect_tx(&full[b], bytes);
      bulk_g2s(smem + static_cast<size_t>(b) * a.stage_stride, wbase + static_cast<long long>(s) * a.R * a.RB,
               bytes, &full[b], policy);
    };
    if (lane == 0) {
      // Weights are never written by an earlier kernel, so their stream starts
      // before the grid dependency resolves.
      policy = l2_evict_first_policy();
      const int pre = min(a.NS, nst);
      for (int s = 0; s < pre; ++s) issue(s);
      issued = pre;
    }
    grid_dep_wait();
    grid_dep_launch();
    int buf = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int s = 0; s < nst; ++s) {
      ok = mbar_wait_bounded(&empty[buf], ph, kCopyTimeoutNs, abort_flag);
      if (!ok) break;
      const int rows_s = min(a.R, nrows - s * a.R);
      const float* rb = red + static_cast<size_t>(buf) * a.R * WPS;
      for (int r = lane; r < rows_s; r += 32) {
        float acc = 0.f;
        for (int w = 0; w < WPS; ++w) acc += rb[r * WPS + w];
        a.y[row0 + static_cast<long long>(s) * a.R + r] = acc;
      }
      __syncwarp();
      if (lane == 0 && s + a.NS < nst) {
        fence_proxy_async_smem();
        issue(s + a.NS);
        issued = s + a.NS + 1;
      }
      if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusCopyTimeout);
      // Let copies still in flight land (bounded) before the CTA exits.
      for (int s = max(0, issued - a.NS); s < issued; ++s)
        (void)mbar_wait_bounded(&full[s % a.NS], static_cast<uint32_t>(s / a.NS) & 1u, kCopyTimeoutNs);
    }
    return;
  }

  // -------------------------------------------------- consumer warps
  const int ctid = tid - 32;
  const int slot = ctid / a.TS;
  const int ls = ctid - slot * a.TS;
  const int wis = ls >> 5;
  grid_dep_wait();
  if (a.stage_x) {
    const float4* xg = reinterpret_cast<const float4*>(a.x);
    float4* xs4 = reinterpret_cast<float4*>(xs);
    for (int i = ctid; i < (a.in_dim >> 2); i += NC) xs4[i] = __ldg(xg + i);
    named_bar_sync(1, NC);
  }
  float xr[UPT][F::kUnitElems];
  float xe[UPT][F::kExtra];
  bool act[UPT];
#pragma unroll
  for (int k = 0; k < UPT; ++k) {
    const int u = ls + k * a.TS;
    act[k] = u < a.U;
    if (a.stage_x) {
#pragma unroll
      for (int i = 0; i < F::kUnitElems; i += 4) {
        const float4 v = act[k] ? *reinterpret_cast<const float4*>(xs + F::xpos(u, i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[k][i] = v.x; xr[k][i + 1] = v.y; xr[k][i + 2] = v.z; xr[k][i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < F::kUnitElems; i += 4) {
        const float4 v = act[k] ? __ldg(reinterpret_cast<const float4*>(a.x + F::xpos(u, i))) : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[k][i] = v.x; xr[k][i + 1] = v.y; xr[k][i + 2] = v.z; xr[k][i + 3] = v.w;
      }
    }
    F::prep(xr[k], xe[k]);
  }

  int buf = 0;
  uint32_t ph = 0;
  for (int i = 0; i < nst; ++i) {
    const bool ok = mbar_wait_bounded(&full[buf], ph, kCopyTimeoutNs, abort_flag);
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        atomicOr(a.status, kStatusCopyTimeout);
      }
      return;
    }
    const uint8_t* sb = smem + static_cast<size_t>(buf) * a.stage_stride;
    const int rows_here = min(a.R, nrows - i * a.R);
    float* rb = red + static_cast<size_t>(buf) * a.R * WPS;
    for (int rr = slot; rr < a.R; rr += a.RPI) {
      float acc = 0.f;
      if (rr < rows_here) {
        const uint8_t* rowp = sb + static_cast<size_t>(rr) * a.RB;
#pragma unroll
        for (int k = 0; k < UPT; ++k)
          if (act[k]) acc += F::dot(rowp, ls + k * a.TS, xr[k], xe[k]);
      }
      acc = warp_sum(acc);
      if (lane == 0) rb[rr * WPS + wis] = acc;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
    if (++buf == a.NS) { buf = 0; ph ^= 1u; }
  }
}

// Generic fallback: one warp per block, lane e-slices decode exactly, each
// block's products are reduced per output row it overlaps and added with one
// atomic per (block, row).  y must be zeroed first.
template <int FMT>
__device__ __forceinline__ float elem(const uint8_t* blk, int e) {
  if constexpr (FMT == 12) return q4k_elem(blk, e);
  else if constexpr (FMT == 14) return q6k_elem(blk, e);
  else if constexpr (FMT == 8) return q8_0_elem(blk, e);
  else return q4_0_elem(blk, e);
}

template <int FMT, int BE, int BB>
__global__ void __launch_bounds__(256) k_gemv_generic(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                                      float* __restrict__ y, long long in_dim, long long nblocks) {
  constexpr int EPL = BE / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long b = warp; b < nblocks; b += nwarps) {
    const uint8_t* blk = w + b * BB;
    const long long base = b * BE;
    const long long j0 = base / in_dim;
    const long long j_last = (base + BE - 1) / in_dim;
    float v[EPL];
    int rel[EPL];
#pragma unroll
    for (int t = 0; t < EPL; ++t) {
      const int e = lane * EPL + t;
      const long long k = base + e;
      const long long j = k / in_dim;
      v[t] = elem<FMT>(blk, e) * __ldg(x + (k - j * in_dim));
      rel[t] = static_cast<int>(j - j0);
    }
    for (long long r = 0; r <= j_last - j0; ++r) {
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < EPL; ++t)
        if (rel[t] == r) s += v[t];
      s = warp_sum(s);
      if (lane == 0) atomicAdd(y + j0 + r, s);
    }
  }
}

template <int FMT, int BE, int BB>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t* __restrict__ w, float* __restrict__ out,
                                                 long long nblocks) {
  constexpr int EPL = BE / 32;
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long b = warp; b < nblocks; b += nwarps) {
    const uint8_t* blk = w + b * BB;
#pragma unroll
    for (int t = 0; t < EPL; ++t) {
      const int e = t * 32 + lane;  // coalesced stores
      out[b * BE + e] = elem<FMT>(blk, e);
    }
  }
}

__global__ void k_dequant_f32(const uint8_t* __restrict__ w, float* __restrict__ out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint8_t* p = w + 4 * i;
    out[i] = __uint_as_float(static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
                             (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24));
  }
}

__global__ void k_dequant_f16(const uint8_t* __restrict__ w, float* __restrict__ out, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    out[i] = f16_to_f32(static_cast<uint32_t>(w[2 * i]) | (static_cast<uint32_t>(w[2 * i + 1]) << 8));
  }
}

// ---------------------------------------------------------------- launchers

// Raise a kernel's dynamic shared-memory limit once per device to the
// largest size requested so far (the attribute is per device context).
template <auto Kern>
static cudaError_t ensure_smem(size_t smem) {
  constexpr int kMaxDev = 64;
  static std::atomic<int> limit[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  if (static_cast<int>(smem) <= limit[dev].load(std::memory_order_relaxed)) return cudaSuccess;
  e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) {
    int cur = limit[dev].load();
    while (cur < static_cast<int>(smem) && !limit[dev].compare_exchange_weak(cur, static_cast<int>(smem))) {
    }
  }
  return e;
}

template <auto Kern>
static cudaError_t launch_pdl(const StreamArgs& a, int threads, int grid, size_t smem, cudaStream_t st, bool pdl) {
  cudaError_t e = ensure_smem<Kern>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, Kern, a);
}

template <class F>
static cudaError_t launch_stream_fmt(const StreamArgs& a, int threads, int grid, size_t smem, int upt,
                                     cudaStream_t st, bool pdl) {
  switch (upt) {
    case 1: return launch_pdl<k_gemv_stream<F, 1>>(a, threads, grid, smem, st, pdl);
    case 2: return launch_pdl<k_gemv_stream<F, 2>>(a, threads, grid, smem, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_stream(int fmt, const StreamArgs& a, int threads, int grid, size_t smem, int upt,
                               cudaStream_t st, bool pdl) {
  switch (fmt) {
    case 12: return launch_stream_fmt<FmtQ4K>(a, threads, grid, smem, upt, st, pdl);
    case 14: return launch_stream_fmt<FmtQ6K>(a, threads, grid, smem, upt, st, pdl);
    case 8: return launch_stream_fmt<FmtQ80>(a, threads, grid, smem, upt, st, pdl);
    case 2: return launch_stream_fmt<FmtQ40>(a, threads, grid, smem, upt, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, long long in_dim,
                                long long nblocks, int grid, cudaStream_t st) {
  switch (fmt) {
    case 12: k_gemv_generic<12, 256, 144><<<grid, 256, 0, st>>>(w, x, y, in_dim, nblocks); break;
    case 14: k_gemv_generic<14, 256, 210><<<grid, 256, 0, st>>>(w, x, y, in_dim, nblocks); break;
    case 8: k_gemv_generic<8, 32, 34><<<grid, 256, 0, st>>>(w, x, y, in_dim, nblocks); break;
    case 2: k_gemv_generic<2, 32, 18><<<grid, 256, 0, st>>>(w, x, y, in_dim, nblocks); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- host-buffer call I/O
// x for a host-buffer GEMV, read from mapped pinned host memory into device
// memory.  It releases the GEMV that follows (programmatic dependent launch)
// at once, so the GEMV's weight stream overlaps this copy; the GEMV reads x
// only after this grid has completed.
__global__ void __launch_bounds__(256) k_host_x_in(const float4* __restrict__ hx, float4* __restrict__ dx, int n4) {
  grid_dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) dx[i] = hx[i];
}

cudaError_t launch_host_x_in(const float* hx_dev, float* dx, long long n, cudaStream_t st) {
  const int n4 = static_cast<int>(n / 4);
  const int grid = std::max(1, std::min(16, (n4 + 255) / 256));
  k_host_x_in<<<grid, 256, 0, st>>>(reinterpret_cast<const float4*>(hx_dev), reinterpret_cast<float4*>(dx), n4);
  return cudaGetLastError();
}

cudaError_t launch_dequant(int fmt, const uint8_t* w, float* out, long long n_elems, int grid, cudaStream_t st) {
  switch (fmt) {
    case 0: k_dequant_f32<<<grid, 256, 0, st>>>(w, out, n_elems); break;
    case 1: k_dequant_f16<<<grid, 256, 0, st>>>(w, out, n_elems); break;
    case 12: k_dequant<12, 256, 144><<<grid, 256, 0, st>>>(w, out, n_elems / 256); break;
    case 14: k_dequant<14, 256, 210><<<grid, 256, 0, st>>>(w, out, n_elems / 256); break;
    case 8: k_dequant<8, 32, 34><<<grid, 256, 0, st>>>(w, out, n_elems / 32); break;
    case 2: k_dequant<2, 32, 18><<<grid, 256, 0, st>>>(w, out, n_elems / 32); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace m3g
