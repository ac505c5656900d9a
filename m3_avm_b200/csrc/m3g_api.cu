// m3g_api.cu -- C ABI of libm3gemv: argument rules, launch planning and the
// resident-offload context.  The rules follow the reference's Rust API for the
// path (src/matvec_quant.rs:51-109, src/quant.rs:120-173,
// src/inference_gpu.rs:58-237); the compute is the sm_100a kernels of
// m3g_kernels.cu.  There is no CPU fallback: without a device every compute
// entry point returns M3G_ECUDA.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/m3gemv.h"
#include "m3g_internal.h"

namespace {

thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? M3G_ENOMEM : M3G_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define M3G_CUDA(call)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

// ---------------------------------------------------------------- formats
struct FmtInfo {
  int fmt;         // kernel format id (13 maps to 12)
  int be;          // elements per block
  int bb;          // bytes per block
  int unit_elems;  // elements per thread unit in the streaming kernel
};

bool fmt_info(uint32_t dtype, FmtInfo& f) {
  switch (dtype) {
    case 12: case 13: f = {12, 256, 144, 64}; return true;
    case 14: f = {14, 256, 210, 64}; return true;
    case 8: f = {8, 32, 34, 32}; return true;
    case 2: f = {2, 32, 18, 32}; return true;
    default: return false;
  }
}

// quant_raw_len (src/matvec_quant.rs:51-83).
bool raw_len_rule(uint32_t dtype, uint64_t n, uint64_t& out) {
  FmtInfo f;
  if (!fmt_info(dtype, f)) return false;
  if (n % static_cast<uint64_t>(f.be)) return false;
  out = (n / f.be) * f.bb;
  return true;
}

// ---------------------------------------------------------------- tuning
struct Tuning {
  int64_t stage_bytes = 16384;  // target bytes per pipeline stage
  int64_t ctas_per_sm = 2;
  int64_t max_stages = 8;
  int64_t force_generic = 0;    // route every GEMV through the generic kernel (parity tests)
  int64_t pdl = 1;              // programmatic dependent launch of the streaming kernels
  int64_t mma = 1;              // tensor-core GEMV where the shape allows it
  int64_t mma_stages = 5;       // pipeline stages of the tensor-core GEMV
  int64_t mma_tps = 0;          // 16-row tiles per stage of 8-warp tiles (1, 2; 0: 2 for long runs of short rows)
  int64_t mma_kc = 16;          // super-blocks per k-chunk (<= 16)
  int64_t mma_ctas = 1;         // CTAs per SM the tensor-core GEMV is sized for
  int64_t mma_wk = 0;           // consumer warps splitting a tile's k-chunk (8, 16; 0 = by shape)
  int64_t mma_cg = 4;           // rows per bulk copy when rows are contiguous (1 or 4)
  int64_t mma_pre = 1;          // stages prefetched before the previous kernel finishes
  int64_t mma_coresident = 0;   // size CTAs for half an SM so consecutive GEMVs overlap
  int64_t decode_coresident = 1;  // the same for the GEMVs of a decode step
  int64_t decode_pre = 1;         // mma_pre for the GEMVs of a decode step
  int64_t mma_xfirst = 0;         // issue the ring past PRE only once x is loaded
  int64_t decode_xfirst = 0;      // the same for the GEMVs of a decode step
  int64_t decode_p2p = 1;         // sharded decode: peer stores over NVLink instead of NCCL all-gathers
  int64_t decode_shard_ffn = 1;   // sharded decode: FFN rows split over the ranks (0: only the vocab head)
  int64_t gemm8 = 1;              // batched Q4_K: 8 columns per launch (k_gemm8_q4k) instead of one GEMV each
  int64_t umma = 1;               // batched Q4_K on tcgen05 (k_umma_q4k), up to 64 columns per pass
  int64_t umma_chains = 8;        // independent accumulators per super-block (capped by TMEM)
  int64_t offload_graph = 1;      // host-buffer offload calls replay one CUDA graph (copy in, GEMV, copy out)
  int64_t peer_wait_us = 2000000; // limit of a kernel's wait for a counter bumped by other GPUs
  int64_t mma_tail_first = 1;     // tensor-core GEMV: a CTA's partial row group first
  int64_t offload_mapped = 1;     // batch-1 host-buffer calls: x, y, status through mapped pinned memory
  int64_t shard_p2p = -1;         // shard contexts: 1 rows exchanged by peer stores from the GEMV epilogue, 0 NCCL,
                                  // -1 peer stores from 8 ranks up (measured faster there, NCCL below)
  int64_t tc8 = 0;                // batch-1 Q4_K GEMV on tcgen05 kind::i8 (k_tc8_q4k, K <= 4096)
  int64_t tc8_pre = 0;            // k_tc8_q4k stages streamed before x is loaded (0: all)
};
Tuning g_tune;

// ---------------------------------------------------------------- per-device state
struct DevState {
  bool ready = false;
  int sms = 0;
  int smem_per_sm = 0;
  int smem_optin = 0;
  uint32_t* status = nullptr;
  // Set only in a per-call copy: the tensor-core GEMV's last CTA stores the
  // status word to *status_host (mapped host memory), counting CTAs in *fin_cnt.
  uint32_t* status_host = nullptr;
  unsigned int* fin_cnt = nullptr;
};
std::mutex g_dev_mu;
std::vector<DevState> g_dev;

int g_ndev = -1;

int dev_state(int device, DevState** out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_ndev <= 0) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n <= 0) return fail(M3G_ECUDA, "no CUDA device: %s", cudaGetErrorString(e));
    g_ndev = n;
    g_dev.resize(n);
  }
  if (device < 0 || device >= g_ndev) return fail(M3G_EINVAL, "device %d out of range [0,%d)", device, g_ndev);
  DevState& d = g_dev[device];
  if (!d.ready) {
    int prev = 0;
    M3G_CUDA(cudaGetDevice(&prev));
    M3G_CUDA(cudaSetDevice(device));
    M3G_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device));
    M3G_CUDA(cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device));
    M3G_CUDA(cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    void* p = nullptr;
    M3G_CUDA(cudaMalloc(&p, 256));
    M3G_CUDA(cudaMemset(p, 0, 256));
    d.status = static_cast<uint32_t*>(p);
    d.ready = true;
    M3G_CUDA(cudaSetDevice(prev));
  }
  *out = &d;
  return M3G_OK;
}

int current_dev_state(DevState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(M3G_ECUDA, "no CUDA device: %s", cudaGetErrorString(e));
  return dev_state(dev, out);
}

// ---------------------------------------------------------------- GEMV planning
struct StreamPlan {
  m3g::StreamArgs a{};
  int threads = 0, grid = 0, upt = 0;
  size_t smem = 0;
};

bool plan_stream(const FmtInfo& f, long long in_dim, long long rows, const uint8_t* w, const float* x,
                 const DevState& ds, StreamPlan& p) {
  if (g_tune.force_generic) return false;
  if (in_dim % f.be) return false;  // blocks straddle rows
  const long long RB = (in_dim / f.be) * f.bb;
  if (RB % 16 || reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16) return false;
  if (RB > (1 << 20) || rows > (1ll << 31) - 1) return false;
  const long long U = in_dim / f.unit_elems;
  int upt = 0, TS = 0;
  for (int cand = 1; cand <= 2; ++cand) {
    long long t = (U + cand - 1) / cand;
    t = (t + 31) / 32 * 32;
    if (t <= 256) { upt = cand; TS = static_cast<int>(t); break; }
  }
  if (!upt) return false;
  const int RPI = std::max(1, 256 / TS);
  const int WPS = TS / 32;
  const long long ctas_per_sm = std::max<int64_t>(1, g_tune.ctas_per_sm);
  const long long budget = std::min<long long>(ds.smem_optin, ds.smem_per_sm / ctas_per_sm - 1024);
  const long long x_bytes = 4 * in_dim;
  bool stage_x = x_bytes <= budget / 3;
  long long m = std::max<long long>(1, std::min<long long>(TS, g_tune.stage_bytes / (RPI * RB)));
  for (;;) {
    const long long R = RPI * m;
    const long long stride = (R * RB + 16 + 127) / 128 * 128;
    const long long xb = stage_x ? (x_bytes + 127) / 128 * 128 : 0;
    const long long per_stage_fixed = stride + R * WPS * 4 + 16;
    long long NS = std::min<long long>(g_tune.max_stages, (budget - xb - 16) / per_stage_fixed);
    if (NS >= 2) {
      p.a.R = static_cast<int>(R);
      p.a.NS = static_cast<int>(NS);
      p.a.stage_stride = static_cast<int>(stride);
      p.a.stage_x = stage_x ? 1 : 0;
      p.a.off_x = static_cast<int>(NS * stride);
      p.a.off_red = static_cast<int>(NS * stride + xb);
      p.a.off_bar = static_cast<int>((p.a.off_red + NS * R * WPS * 4 + 15) / 16 * 16);
      p.smem = static_cast<size_t>(p.a.off_bar + 16 * NS + 16);
      break;
    }
    if (m > 1) { --m; continue; }
    if (stage_x) { stage_x = false; continue; }
    return false;
  }
  const long long grid_target = static_cast<long long>(ds.sms) * ctas_per_sm;
  const long long rpc = std::max<long long>(1, (rows + grid_target - 1) / grid_target);
  p.a.in_dim = static_cast<int>(in_dim);
  p.a.rows = static_cast<int>(rows);
  p.a.RB = static_cast<int>(RB);
  p.a.U = static_cast<int>(U);
  p.a.TS = TS;
  p.a.RPI = RPI;
  p.a.rows_per_cta = static_cast<int>(rpc);
  p.threads = 32 + TS * RPI;
  p.grid = static_cast<int>((rows + rpc - 1) / rpc);
  p.upt = upt;
  return true;
}

struct MmaPlan {
  m3g::MmaArgs a{};
  int grid = 0, tps = 1, wk = 8;
  size_t smem = 0;
};

bool plan_mma(const FmtInfo& f, long long in_dim, long long rows, const uint8_t* w, const float* x,
              const DevState& ds, MmaPlan& p, bool coresident) {
  if (in_dim % 256) return false;
  const long long NSB = in_dim / 256;
  const int sbb = m3g::mma_sb_bytes(f.fmt);
  const long long RB = NSB * sbb;
  if (sbb == 0 || RB % 16 || reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16) return false;
  if (rows > (1ll << 31) - 1 || in_dim > (1 << 20)) return false;
  long long KC = std::min<long long>(NSB, std::min<int64_t>(16, g_tune.mma_kc));
  // Q8_0 rows take 4352 bytes per 4096 inputs, so a 16-row stage of 16
  // super-blocks is 70 KB and only two or three fit: half-width k-chunks keep
  // the ring deep (measured 4096x4096: 8.0 -> 6.45 us; 14336x4096: 18.1 ->
  // 17.6 us).  Q4_K, Q4_0 and Q6_K are slower with them.
  if (f.fmt == 8 && g_tune.mma_kc == 16 && NSB >= 16) KC = 8;
  // Consumer warps per tile: 16 when a k-chunk of 16 super-blocks covers the
  // whole row (one super-block per warp, x operands stay in registers), or
  // for the heavier Q6_K decode; 8 otherwise.  mma_wk = 8 / 16 forces it.
  const long long rows_per_sm = (rows + ds.sms - 1) / ds.sms;
  // Q6_K rows of 16 super-blocks with very many rows per SM (the 128256-row
  // vocab head: 867) run 3 % faster as two 8-warp tiles per stage; at 221
  // rows per SM (32768 rows) and below that form is slower.
  const bool q6k_many = f.fmt == 14 && NSB == 16 && KC == 16 && rows_per_sm >= 512;
  int wk = g_tune.mma_wk;
  if (wk != 8 && wk != 16)
    wk = q6k_many ? 8 : (((NSB == 16 && KC == 16) || (f.fmt == 14 && NSB >= 16)) ? 16 : 8);
  // Two 8-warp tiles per stage (16 consumer warps) pay off when each CTA
  // streams many short rows (measured: Q6_K 128256x2048 -31 %, Q4_K
  // 16384x2048 -10 %) and cost on small or long-row shapes (2048x2048 +19 %,
  // 28672x8192 +3 %).
  const int auto_tps = (NSB <= 8 && rows_per_sm >= 64) || q6k_many ? 2 : 1;
  const int tps = wk == 16 ? 1 : (g_tune.mma_tps == 0 ? auto_tps : static_cast<int>(std::min<int64_t>(2, g_tune.mma_tps)));
  if (f.fmt == 14) {  // 210-byte blocks: chunk sizes must stay multiples of 16 bytes
    if (NSB % 8) return false;
    KC = std::max<long long>(8, KC / 8 * 8);
    if (KC > NSB) KC = NSB;
  }
  const long long seg = KC * sbb;
  const long long NKC = (NSB + KC - 1) / KC;
  // Whole rows are contiguous when one k-chunk covers the row: copy 4 rows
  // per bulk copy then; otherwise one copy per row segment.
  const long long CG = (NKC == 1 && g_tune.mma_cg == 4) ? 4 : 1;
  // Row-group stride: the residue mod 128 that makes the tile's shared loads
  // conflict-free (Q4_K: 16-byte header + 8-byte quant loads of 8 rows; the
  // 2-byte aligned blocks of Q6_K and Q4_0: 4-byte loads across two words).
  const long long gs_mod = f.fmt == 12 ? 32 : 16;
  long long GS = (CG * seg + 15) / 16 * 16;
  while (GS % 128 != gs_mod) GS += 16;
  const long long xsl = 3 * in_dim, s32 = in_dim / 8, s16 = in_dim / 4, sc = NSB * 4;
  const long long fixed = xsl + s32 + s16 + sc + 4 * 128 + 16;
  const long long mctas = std::max<int64_t>(1, g_tune.mma_ctas);
  // mma_coresident sizes a CTA for half an SM without changing the grid, so
  // the next GEMV's CTAs (launched early by PDL) fit beside this one's.
  const long long div = std::max<long long>(mctas, coresident ? 2 : 1);
  const long long budget = std::min<long long>(ds.smem_optin, ds.smem_per_sm / div - 1024);
  const long long SR = 16 * tps;
  const long long per_stage = SR / CG * GS + SR * wk * 4 + 16;
  long long NS = std::min<long long>(g_tune.mma_stages, (budget - fixed) / per_stage);
  if (NS < 2) return false;
  long long off = NS * (SR / CG) * GS;
  p.a.off_xsl = static_cast<int>(off);
  off += (xsl + 127) / 128 * 128;
  p.a.off_sum32 = static_cast<int>(off);
  off += (s32 + 15) / 16 * 16;
  p.a.off_sum16 = static_cast<int>(off);
  off += (s16 + 15) / 16 * 16;
  p.a.off_scale = static_cast<int>(off);
  off += (sc + 15) / 16 * 16;
  p.a.off_red = static_cast<int>(off);
  off += NS * SR * wk * 4;
  p.a.off_bar = static_cast<int>(off);
  off += NS * 16 + 16;
  if (off > budget) return false;
  p.smem = static_cast<size_t>(off);
  p.a.rows = static_cast<int>(rows);
  p.a.RB = static_cast<int>(RB);
  p.a.NSB = static_cast<int>(NSB);
  p.a.KC = static_cast<int>(KC);
  p.a.NKC = static_cast<int>(NKC);
  p.a.CG = static_cast<int>(CG);
  p.a.GS = static_cast<int>(GS);
  p.a.SEG = static_cast<int>(seg);
  p.a.NS = static_cast<int>(NS);
  p.a.PRE = static_cast<int>(std::max<int64_t>(0, g_tune.mma_pre));
  p.a.peer_wait_ns = static_cast<unsigned long long>(g_tune.peer_wait_us) * 1000ull;
  p.a.tail_first = g_tune.mma_tail_first ? 1 : 0;
  p.tps = tps;
  p.wk = wk;
  const long long ctas = static_cast<long long>(ds.sms) * mctas;
  const long long rpc = std::max<long long>(1, (rows + ctas - 1) / ctas);
  p.a.rows_per_cta = static_cast<int>(rpc);
  p.grid = static_cast<int>((rows + rpc - 1) / rpc);
  return true;
}

// y[out_dim] = W x on `st`; w/x/y device pointers.
int gemv_launch(const DevState& ds, const FmtInfo& f, const uint8_t* w, const float* x, float* y,
                long long in_dim, long long out_dim, cudaStream_t st) {
  m3g::Tc8Plan tp;
  if (!g_tune.force_generic && g_tune.mma && g_tune.tc8 && f.fmt == 12 &&
      m3g::plan_tc8(in_dim, out_dim, w, x, ds.sms, ds.smem_optin, tp)) {
    tp.a.x = x;
    tp.a.y = y;
    tp.a.status = ds.status;
    tp.a.status_host = ds.status_host;
    tp.a.fin_cnt = ds.fin_cnt;
    if (g_tune.tc8_pre > 0 && g_tune.tc8_pre < tp.a.PRE) tp.a.PRE = static_cast<int>(g_tune.tc8_pre);
    cudaError_t e = m3g::launch_tc8(tp, w, st, g_tune.pdl != 0);
    if (e != cudaSuccess) return cuda_fail(e, "k_tc8_q4k launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M3G_OK;
  }
  MmaPlan mp;
  if (!g_tune.force_generic && g_tune.mma && plan_mma(f, in_dim, out_dim, w, x, ds, mp, g_tune.mma_coresident != 0)) {
    mp.a.w = w;
    mp.a.x = x;
    mp.a.y = y;
    mp.a.status = ds.status;
    mp.a.status_host = ds.status_host;
    mp.a.fin_cnt = ds.fin_cnt;
    mp.a.xfirst = static_cast<int>(g_tune.mma_xfirst);
    cudaError_t e = m3g::launch_gemv_mma(f.fmt, mp.a, mp.tps, mp.wk, mp.grid, mp.smem, st, g_tune.pdl != 0);
    if (e != cudaSuccess) return cuda_fail(e, "k_gemv_mma launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M3G_OK;
  }
  StreamPlan p;
  if (plan_stream(f, in_dim, out_dim, w, x, ds, p)) {
    p.a.w = w;
    p.a.x = x;
    p.a.y = y;
    p.a.status = ds.status;
    cudaError_t e = m3g::launch_gemv_stream(f.fmt, p.a, p.threads, p.grid, p.smem, p.upt, st, g_tune.pdl != 0);
    if (e != cudaSuccess) return cuda_fail(e, "k_gemv_stream launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return M3G_OK;
  }
  const long long nblocks = in_dim * out_dim / f.be;
  M3G_CUDA(cudaMemsetAsync(y, 0, sizeof(float) * static_cast<size_t>(out_dim), st));
  const long long want = (nblocks + 7) / 8;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(want, 8ll * ds.sms)));
  cudaError_t e = m3g::launch_gemv_generic(f.fmt, w, x, y, in_dim, nblocks, grid, st);
  if (e != cudaSuccess) return cuda_fail(e, "k_gemv_generic launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return M3G_OK;
}

struct Gemm8Plan {
  m3g::Gemm8Args a{};
  int grid = 0;
  size_t smem = 0;
};

// Batched Q4_K: chunks of KC <= 4 super-blocks (one prepared-x record each,
// double-buffered), stages of 8 / KC row tiles of one chunk, per-(row,
// column) sums; sized so two CTAs share an SM.
bool plan_gemm8(const FmtInfo& f, long long in_dim, long long rows, const uint8_t* w, const float* x,
                const DevState& ds, Gemm8Plan& p) {
  if (f.fmt != 12 || in_dim % 256) return false;
  if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16) return false;
  if (rows > (1ll << 31) - 1 || in_dim > (1 << 20)) return false;
  const long long NSB = in_dim / 256;
  long long KC = 4;
  while (KC > NSB) KC /= 2;  // 4, 2 or 1 super-blocks per chunk (8 / KC row tiles per stage)
  const long long NKC = (NSB + KC - 1) / KC;
  const long long SR = 16 * (8 / KC);
  long long GS = (KC * 144 + 15) / 16 * 16;
  while (GS % 128 != 32) GS += 16;
  const long long ctas = 2ll * ds.sms;
  const long long rpc = std::max<long long>(1, (rows + ctas - 1) / ctas);
  const long long xc = KC * m3g::kGemm8RecBytes;
  const long long off_stage = (2 * xc + 127) / 128 * 128;
  const long long per_stage = SR * GS + SR * 8 * KC * 4;
  const long long acc = (rpc * 8 * 4 + 15) / 16 * 16;
  const long long budget = std::min<long long>(ds.smem_optin, ds.smem_per_sm / 2 - 1024);
  long long NS = std::min<long long>(4, (budget - off_stage - acc - 256) / per_stage);
  if (NS < 2) return false;
  p.a.rows = static_cast<int>(rows);
  p.a.RB = static_cast<int>(NSB * 144);
  p.a.NSB = static_cast<int>(NSB);
  p.a.KC = static_cast<int>(KC);
  p.a.NKC = static_cast<int>(NKC);
  p.a.NS = static_cast<int>(NS);
  p.a.GS = static_cast<int>(GS);
  p.a.rows_per_cta = static_cast<int>(rpc);
  p.a.off_stage = static_cast<int>(off_stage);
  p.a.off_red = static_cast<int>(off_stage + NS * SR * GS);
  p.a.off_acc = static_cast<int>(p.a.off_red + NS * SR * 8 * KC * 4);
  p.a.off_bar = static_cast<int>(p.a.off_acc + acc);
  p.smem = static_cast<size_t>(p.a.off_bar + (2 * NS + 4) * 8 + 16);
  p.grid = static_cast<int>((rows + rpc - 1) / rpc);
  return static_cast<long long>(p.smem) <= budget;
}

// Batched Q4_K on tcgen05: NB accumulator columns for a pass of `cols`
// columns; weight stages of one 128-row super-block tile, X stages of one
// prepared super-block, as many of each as shared memory holds (the request is
// above half an SM, so one CTA -- and one 512-column TMEM allocation -- per SM).
struct UmmaPlan {
  m3g::UmmaArgs a{};
  int grid = 0, nb = 0;
  size_t smem = 0;
  size_t off_cnt = 0, off_xt = 0, off_part = 0, ws_bytes = 0;
};

bool plan_umma(const FmtInfo& f, long long in_dim, long long rows, const uint8_t* w, long long cols,
               const DevState& ds, UmmaPlan& p) {
  if (f.fmt != 12 || in_dim % 256 || in_dim > (1 << 22) || cols < 1 || cols > 64) return false;
  if (reinterpret_cast<uintptr_t>(w) % 16 || rows < 1 || rows > (1ll << 31) - 1) return false;
  const int nb = cols <= 8 ? 8 : cols <= 16 ? 16 : cols <= 32 ? 32 : 64;
  const long long XS = m3g::umma_xtile(nb), SW = 128 * 144;
  const long long avail = std::min<long long>(ds.smem_optin, 232448) - 8192 - 4096 - 256;
  long long NSX = 0, NSW = 0;
  for (long long nx = 4; nx >= 2 && !NSX; --nx) {
    const long long nw = std::min<long long>(8, (avail - nx * XS) / SW);
    if (nw >= 4 || (nx == 2 && nw >= 2)) NSX = nx, NSW = nw;
  }
  if (!NSX) return false;
  const long long NSB = in_dim / 256, tiles = (rows + 127) / 128;
  p.nb = nb;
  p.a.RB = NSB * 144;
  p.a.rows = rows;
  p.a.NSB = static_cast<int>(NSB);
  p.a.tiles = static_cast<int>(tiles);
  p.a.T = tiles * NSB;
  p.a.NSW = static_cast<int>(NSW);
  p.a.NSX = static_cast<int>(NSX);
  p.a.off_x = static_cast<int>(NSW * SW);
  p.a.off_am = static_cast<int>(p.a.off_x + NSX * XS);
  p.a.off_bar = p.a.off_am + 8192 + 4096;  // m operand stages, (d, dmin) ring
  p.smem = static_cast<size_t>(p.a.off_bar + (2 * NSW + NSX + 12) * 8 + 16);
  p.grid = static_cast<int>(std::min<long long>(ds.sms, p.a.T));
  p.off_cnt = static_cast<size_t>((NSB * 64 * 4 + 255) / 256 * 256);  // column scales [NSB][<= 64] first
  p.off_xt = p.off_cnt + static_cast<size_t>((tiles * 4 + 255) / 256 * 256);
  p.off_part = p.off_xt + static_cast<size_t>(NSB * XS);
  p.ws_bytes = p.off_part + static_cast<size_t>(p.grid) * 2 * nb * 128 * sizeof(float);
  return static_cast<long long>(p.smem) <= std::min<long long>(ds.smem_optin, 232448) &&
         static_cast<long long>(p.smem) > ds.smem_per_sm / 2;
}

int gemv_batch_launch(const DevState& ds, const FmtInfo& f, const uint8_t* w, const float* x, float* y,
                      long long in_dim, long long out_dim, long long batch, cudaStream_t st) {
  UmmaPlan up;
  if (batch >= 2 && !g_tune.force_generic && g_tune.mma && g_tune.umma &&
      plan_umma(f, in_dim, out_dim, w, std::min<long long>(batch, 64), ds, up)) {
    // one workspace sized for the widest pass: column scales | tile counters | X tiles | partial tiles
    uint8_t* ws = nullptr;
    M3G_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), up.ws_bytes, st));
    int rc = M3G_OK;
    for (long long p0 = 0; p0 < batch && rc == M3G_OK; p0 += 64) {
      const long long cols = std::min<long long>(64, batch - p0);
      UmmaPlan pp;
      if (!plan_umma(f, in_dim, out_dim, w, cols, ds, pp)) {
        rc = fail(M3G_EINVAL, "no tcgen05 plan for %lld columns", cols);
        break;
      }
      pp.a.w = w;
      pp.a.sig = reinterpret_cast<const float*>(ws);
      pp.a.cnt = reinterpret_cast<unsigned*>(ws + pp.off_cnt);
      pp.a.xt = ws + pp.off_xt;
      pp.a.part = reinterpret_cast<float*>(ws + pp.off_part);
      pp.a.y = y + p0 * out_dim;
      pp.a.status = ds.status;
      pp.a.cols = static_cast<int>(cols);
      pp.a.ldy = static_cast<int>(out_dim);
      cudaError_t e = m3g::launch_umma_q4k(pp.a, x + p0 * in_dim, in_dim, pp.nb,
                                           static_cast<int>(g_tune.umma_chains), pp.grid, pp.smem, st,
                                           g_tune.pdl != 0);
      if (e != cudaSuccess) rc = cuda_fail(e, "tcgen05 batched GEMV launch");
      else g_launches.fetch_add(3, std::memory_order_relaxed);
    }
    cudaFreeAsync(ws, st);
    return rc;
  }
  Gemm8Plan gp;
  if (batch >= 2 && !g_tune.force_generic && g_tune.mma && g_tune.gemm8 && plan_gemm8(f, in_dim, out_dim, w, x, ds, gp)) {
    // X is quantised once per pass of 8 columns into a stream-ordered workspace.
    uint8_t* ws = nullptr;
    const size_t ws_bytes = static_cast<size_t>(gp.a.NSB) * m3g::kGemm8RecBytes;
    M3G_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), ws_bytes, st));
    int rc = M3G_OK;
    for (long long p0 = 0; p0 < batch && rc == M3G_OK; p0 += m3g::kGemm8Cols) {
      const int cols = static_cast<int>(std::min<long long>(m3g::kGemm8Cols, batch - p0));
      cudaError_t e = m3g::launch_xprep8(x + p0 * in_dim, cols, static_cast<int>(in_dim), ws, st);
      if (e == cudaSuccess) {
        gp.a.w = w;
        gp.a.xq = ws;
        gp.a.y = y + p0 * out_dim;
        gp.a.status = ds.status;
        gp.a.cols = cols;
        gp.a.ldy = static_cast<int>(out_dim);
        e = m3g::launch_gemm8_q4k(gp.a, gp.grid, gp.smem, st);
      }
      if (e != cudaSuccess) rc = cuda_fail(e, "batched GEMV launch");
      else g_launches.fetch_add(2, std::memory_order_relaxed);
    }
    cudaFreeAsync(ws, st);
    return rc;
  }
  for (long long b = 0; b < batch; ++b) {
    int rc = gemv_launch(ds, f, w, x + b * in_dim, y + b * out_dim, in_dim, out_dim, st);
    if (rc) return rc;
  }
  return M3G_OK;
}

int check_status(const DevState& ds) {
  uint32_t s = 0;
  M3G_CUDA(cudaMemcpy(&s, ds.status, sizeof s, cudaMemcpyDeviceToHost));
  if (s & m3g::kStatusCopyTimeout) {
    cudaMemset(ds.status, 0, sizeof s);
    return fail(M3G_ETIMEOUT, "a staged weight copy did not complete in time");
  }
  return M3G_OK;
}

// Shape rules shared by the GEMV entry points (src/matvec_quant.rs:94-101).
int gemv_rules(uint32_t dtype, uint64_t raw_len, uint64_t in_dim, uint64_t out_dim, FmtInfo& f) {
  if (in_dim == 0 || out_dim == 0) return fail(M3G_ENONE, "zero dimension");
  if (in_dim > (1ull << 40) / out_dim) return fail(M3G_ENONE, "in_dim*out_dim overflows");
  uint64_t need = 0;
  if (!raw_len_rule(dtype, in_dim * out_dim, need))
    return fail(M3G_ENONE, "dtype %u has no fused kernel for %llu elements", dtype,
                static_cast<unsigned long long>(in_dim * out_dim));
  if (raw_len < need)
    return fail(M3G_ENONE, "raw has %llu bytes, needs %llu", static_cast<unsigned long long>(raw_len),
                static_cast<unsigned long long>(need));
  if (in_dim > (1ull << 31) || out_dim > (1ull << 31)) return fail(M3G_EINVAL, "dimension too large");
  fmt_info(dtype, f);
  return M3G_OK;
}

// RAII device buffer for the host-pointer entry points.
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  cudaError_t alloc(size_t n) { return cudaMalloc(&p, n ? n : 16); }
};

}  // namespace

// Entry points shared with the other translation units of the library.
namespace m3g {
int host_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

bool block_geometry(uint32_t dtype, int* be, int* bb) {
  FmtInfo f;
  if (!fmt_info(dtype, f)) return false;
  *be = f.be;
  *bb = f.bb;
  return true;
}

int gemv_fused(int device, uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, const float* x2,
               const float* gamma, const float* res, int xmode, float* y, long long in_dim, long long out_dim,
               cudaStream_t st, bool decode, unsigned long long* argmax_key, bool swiglu, long long key_row0,
               const PeerIO* peers, int* grid_out) {
  bool coresident = decode && g_tune.decode_coresident;
  if (swiglu && (out_dim % 16 || xmode == kXSiluMul || res || argmax_key))
    return fail(M3G_EINVAL, "SwiGLU epilogue needs gate/up rows in 16-row blocks and no other epilogue");
  FmtInfo f;
  if (int rc = gemv_rules(dtype, raw_len, static_cast<uint64_t>(in_dim), static_cast<uint64_t>(out_dim), f)) return rc;
  if (xmode < kXPlain || xmode > kXSiluMul) return fail(M3G_EINVAL, "unknown input transform %d", xmode);
  if (xmode == kXSiluMul && (!x2 || reinterpret_cast<uintptr_t>(x2) % 16))
    return fail(M3G_EINVAL, "silu input needs a 16-byte aligned second vector");
  if (gamma && reinterpret_cast<uintptr_t>(gamma) % 16) return fail(M3G_EINVAL, "norm weights not 16-byte aligned");
  DevState* ds = nullptr;
  if (int rc = dev_state(device, &ds)) return rc;
  // Half-SM CTAs let the next small GEMV start beside this one; a GEMV with
  // many rows per SM (the FFN gate|up, the vocab head) runs long enough to
  // prefer whole SMs and the deeper pipeline that goes with them.
  if (coresident && (out_dim + ds->sms - 1) / ds->sms >= 64) coresident = false;
  MmaPlan mp;
  // A half-SM CTA needs two stages of the row segment; wide Q6_K rows may not
  // fit, and then the CTA takes the whole SM.
  const bool planned = plan_mma(f, in_dim, out_dim, w, x, *ds, mp, coresident) ||
                       (coresident && plan_mma(f, in_dim, out_dim, w, x, *ds, mp, false));
  if (!planned)
    return fail(M3G_EINVAL, "no tensor-core plan for dtype %u, %lld x %lld (K %% 256, 16-byte rows and pointers)",
                dtype, out_dim, in_dim);
  mp.a.w = w;
  mp.a.x = x;
  mp.a.y = y;
  mp.a.status = ds->status;
  mp.a.x2 = x2;
  mp.a.gamma = gamma;
  mp.a.res = res;
  mp.a.xmode = xmode;
  mp.a.argmax_key = argmax_key;
  mp.a.swiglu = swiglu ? 1 : 0;
  mp.a.key_row0 = key_row0;
  if (swiglu) {  // tiles must start on 16-row (gate/up block) boundaries
    const long long rpc = (mp.a.rows_per_cta + 15) / 16 * 16;
    mp.a.rows_per_cta = static_cast<int>(rpc);
    mp.grid = static_cast<int>((out_dim + rpc - 1) / rpc);
  }
  mp.a.xfirst = static_cast<int>(decode ? g_tune.decode_xfirst : g_tune.mma_xfirst);
  if (decode) mp.a.PRE = static_cast<int>(g_tune.decode_pre);
  if (peers) {
    for (int p = 0; p < kMaxPeers; ++p) {
      mp.a.peer_y[p] = peers->peer_y[p];
      mp.a.peer_key[p] = peers->peer_key[p];
      mp.a.peer_cnt[p] = peers->peer_cnt[p];
    }
    mp.a.npeer = peers->npeer;
    mp.a.done_cnt = peers->done_cnt;
    mp.a.step = peers->step;
    mp.a.wait_cnt = peers->wait_cnt;
    mp.a.wait_mul = peers->wait_mul;
    mp.a.key_by_step = peers->key_by_step;
    mp.a.ystep = peers->ystep;
    mp.a.ystride = peers->ystride;
  }
  if (grid_out) *grid_out = mp.grid;
  cudaError_t e = launch_gemv_mma(f.fmt, mp.a, mp.tps, mp.wk, mp.grid, mp.smem, st, g_tune.pdl != 0);
  if (e != cudaSuccess) return cuda_fail(e, "k_gemv_mma launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return M3G_OK;
}

// The greedy-pick GEMV (argmax epilogue into *key) planned from device
// attributes alone, with a caller-provided status word: no per-device state
// is created, so nothing is allocated.
int gemv_greedy_on(uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, float* y, long long in_dim,
                   long long out_dim, cudaStream_t st, int sms, int smem_per_sm, int smem_optin, uint32_t* status,
                   unsigned long long* key) {
  FmtInfo f;
  if (int rc = gemv_rules(dtype, raw_len, static_cast<uint64_t>(in_dim), static_cast<uint64_t>(out_dim), f)) return rc;
  DevState ds;
  ds.ready = true;
  ds.sms = sms;
  ds.smem_per_sm = smem_per_sm;
  ds.smem_optin = smem_optin;
  ds.status = status;
  MmaPlan mp;
  if (!plan_mma(f, in_dim, out_dim, w, x, ds, mp, false))
    return fail(M3G_EINVAL, "no tensor-core plan for dtype %u, %lld x %lld (K %% 256, 16-byte rows and pointers)",
                dtype, out_dim, in_dim);
  mp.a.w = w;
  mp.a.x = x;
  mp.a.y = y;
  mp.a.status = status;
  mp.a.argmax_key = key;
  cudaError_t e = launch_gemv_mma(f.fmt, mp.a, mp.tps, mp.wk, mp.grid, mp.smem, st, g_tune.pdl != 0);
  if (e != cudaSuccess) return cuda_fail(e, "k_gemv_mma launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return M3G_OK;
}

bool decode_p2p_enabled() { return g_tune.decode_p2p != 0; }
bool shard_p2p_enabled(int world) { return g_tune.shard_p2p > 0 || (g_tune.shard_p2p < 0 && world >= 8); }

bool fused_plannable(int device, uint32_t dtype, long long in_dim, long long rows) {
  FmtInfo f;
  if (!fmt_info(dtype, f) || rows < 1) return false;
  DevState* ds = nullptr;
  if (dev_state(device, &ds)) return false;
  MmaPlan mp;
  alignas(16) static const float kAligned[4] = {0.f, 0.f, 0.f, 0.f};  // stands in for 16-byte aligned w and x
  const uint8_t* w16 = reinterpret_cast<const uint8_t*>(kAligned);
  return plan_mma(f, in_dim, rows, w16, kAligned, *ds, mp, false);
}
unsigned long long peer_wait_ns() { return static_cast<unsigned long long>(g_tune.peer_wait_us) * 1000ull; }
bool decode_shard_ffn_enabled() { return g_tune.decode_shard_ffn != 0; }

int status_word(int device, uint32_t** out) {
  DevState* ds = nullptr;
  if (int rc = dev_state(device, &ds)) return rc;
  *out = ds->status;
  return M3G_OK;
}

// y[out] = W x on `st` for device pointers, on `device` (the current one).
int gemv_device(int device, uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, float* y,
                long long in_dim, long long out_dim, cudaStream_t st) {
  FmtInfo f;
  if (int rc = gemv_rules(dtype, raw_len, static_cast<uint64_t>(in_dim), static_cast<uint64_t>(out_dim), f)) return rc;
  DevState* ds = nullptr;
  if (int rc = dev_state(device, &ds)) return rc;
  return gemv_launch(*ds, f, w, x, y, in_dim, out_dim, st);
}
}  // namespace m3g

// ================================================================ C ABI
extern "C" {

int m3g_abi_version(void) { return 1; }

const char* m3g_last_error(void) { return t_last_error.c_str(); }

uint64_t m3g_launch_count(void) { return g_launches.load(); }

int m3g_set_tuning(const char* key, int64_t value) {
  if (!key) return fail(M3G_EINVAL, "null key");
  if (!strcmp(key, "stage_bytes") && value >= 1024) g_tune.stage_bytes = value;
  else if (!strcmp(key, "ctas_per_sm") && value >= 1 && value <= 8) g_tune.ctas_per_sm = value;
  else if (!strcmp(key, "max_stages") && value >= 2 && value <= 32) g_tune.max_stages = value;
  else if (!strcmp(key, "force_generic")) g_tune.force_generic = value != 0;
  else if (!strcmp(key, "pdl")) g_tune.pdl = value != 0;
  else if (!strcmp(key, "mma")) g_tune.mma = value != 0;
  else if (!strcmp(key, "mma_stages") && value >= 2 && value <= 8) g_tune.mma_stages = value;
  else if (!strcmp(key, "mma_tps") && value >= 0 && value <= 2) g_tune.mma_tps = value;
  else if (!strcmp(key, "mma_kc") && value >= 1 && value <= 16) g_tune.mma_kc = value;
  else if (!strcmp(key, "mma_ctas") && value >= 1 && value <= 2) g_tune.mma_ctas = value;
  else if (!strcmp(key, "mma_wk") && (value == 0 || value == 8 || value == 16)) g_tune.mma_wk = value;
  else if (!strcmp(key, "mma_cg") && (value == 1 || value == 4)) g_tune.mma_cg = value;
  else if (!strcmp(key, "mma_pre") && value >= 0 && value <= 8) g_tune.mma_pre = value;
  else if (!strcmp(key, "mma_coresident")) g_tune.mma_coresident = value != 0;
  else if (!strcmp(key, "decode_coresident")) g_tune.decode_coresident = value != 0;
  else if (!strcmp(key, "decode_pre") && value >= 0 && value <= 8) g_tune.decode_pre = value;
  else if (!strcmp(key, "mma_xfirst")) g_tune.mma_xfirst = value != 0;
  else if (!strcmp(key, "decode_xfirst")) g_tune.decode_xfirst = value != 0;
  else if (!strcmp(key, "decode_p2p")) g_tune.decode_p2p = value != 0;
  else if (!strcmp(key, "decode_shard_ffn")) g_tune.decode_shard_ffn = value != 0;
  else if (!strcmp(key, "gemm8")) g_tune.gemm8 = value != 0;
  else if (!strcmp(key, "umma")) g_tune.umma = value != 0;
  else if (!strcmp(key, "offload_graph")) g_tune.offload_graph = value != 0;
  else if (!strcmp(key, "umma_chains") && value >= 1 && value <= 8) g_tune.umma_chains = value;
  else if (!strcmp(key, "peer_wait_us") && value >= 1 && value <= 60000000) g_tune.peer_wait_us = value;
  else if (!strcmp(key, "mma_tail_first")) g_tune.mma_tail_first = value != 0;
  else if (!strcmp(key, "offload_mapped")) g_tune.offload_mapped = value != 0;
  else if (!strcmp(key, "shard_p2p") && value >= -1 && value <= 1) g_tune.shard_p2p = value;
  else if (!strcmp(key, "tc8")) g_tune.tc8 = value != 0;
  else if (!strcmp(key, "tc8_pre") && value >= 0 && value <= 64) g_tune.tc8_pre = value;
  else return fail(M3G_ENONE, "unknown tuning key or value: %s=%lld", key, static_cast<long long>(value));
  return M3G_OK;
}

int m3g_quant_raw_len(uint32_t dtype, uint64_t n, uint64_t* out_len) {
  if (!out_len) return fail(M3G_EINVAL, "null out_len");
  uint64_t v = 0;
  if (!raw_len_rule(dtype, n, v)) return fail(M3G_ENONE, "no fused kernel for dtype %u, n %llu", dtype,
                                               static_cast<unsigned long long>(n));
  *out_len = v;
  return M3G_OK;
}

// ---------------------------------------------------------------- host helpers
// f32_to_bf16_bits (src/quant.rs:186-194): RNE, quiet-NaN guard.
uint16_t m3g_f32_to_bf16_bits(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint32_t bias = 0x7FFFu + ((b >> 16) & 1u);
  uint16_t bf = static_cast<uint16_t>((b + bias) >> 16);
  if (std::isnan(x)) bf |= 0x0040u;
  return bf;
}

float m3g_bf16_bits_to_f32(uint16_t b) {
  const uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

}  // extern "C"

namespace {
// binary32 -> binary16 round-to-nearest-even (the f16 the encoders store).
uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
  const uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) return man ? static_cast<uint16_t>(sign | 0x7E00u | (man >> 13)) : (sign | 0x7C00u);
  const int e = static_cast<int>(exp) - 127 + 15;
  if (e >= 31) return sign | 0x7C00u;
  if (e <= 0) {
    if (e < -10) return sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    uint32_t hm = man >> shift;
    const uint32_t rb = 1u << (shift - 1), rest = man & ((1u << shift) - 1u);
    if (rest > rb || (rest == rb && (hm & 1u))) hm += 1;
    return static_cast<uint16_t>(sign | hm);
  }
  const uint32_t hm = man >> 13, rest = man & 0x1FFFu;
  uint32_t out = (static_cast<uint32_t>(e) << 10) | hm;
  if (rest > 0x1000u || (rest == 0x1000u && (hm & 1u))) out += 1;
  return static_cast<uint16_t>(sign | out);
}

float f16_to_f32_host(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else {
      int e = -1;
      do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
      u = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7F800000u | (man << 13);
  } else {
    u = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Rust `f32 as i32` (saturating, NaN -> 0), then clamp.
int32_t sat_round_clamp(float v, int32_t lo, int32_t hi) {
  v = std::round(v);
  int32_t i;
  if (std::isnan(v)) i = 0;
  else if (v >= 2147483647.0f) i = INT32_MAX;
  else if (v <= -2147483648.0f) i = INT32_MIN;
  else i = static_cast<int32_t>(v);
  return i < lo ? lo : (i > hi ? hi : i);
}

int quantize_block(const float* src, uint64_t src_len, uint8_t* dst, uint64_t dst_len, int qmax, bool q4) {
  const uint64_t need = q4 ? 18 : 34;
  if (!src || !dst) return fail(M3G_EINVAL, "null pointer");
  if (src_len != 32 || dst_len < need) return fail(M3G_ENONE, "needs 32 floats and %llu bytes",
                                                   static_cast<unsigned long long>(need));
  float amax = 0.f;
  for (int i = 0; i < 32; ++i) {
    if (!std::isfinite(src[i])) return fail(M3G_ENONE, "non-finite input");
    amax = std::fmax(amax, std::fabs(src[i]));
  }
  const uint16_t db = f32_to_f16_rne(amax == 0.f ? 0.f : amax / static_cast<float>(qmax));
  const float ds = f16_to_f32_host(db);
  dst[0] = static_cast<uint8_t>(db & 0xFF);
  dst[1] = static_cast<uint8_t>(db >> 8);
  if (q4) {
    if (amax == 0.f) { memset(dst + 2, 0x88, 16); return M3G_OK; }
    for (int i = 0; i < 16; ++i) {
      const int32_t lo = sat_round_clamp(src[i] / ds, -8, 7) + 8;
      const int32_t hi = sat_round_clamp(src[i + 16] / ds, -8, 7) + 8;
      dst[2 + i] = static_cast<uint8_t>(static_cast<uint8_t>(lo) | static_cast<uint8_t>(hi << 4));
    }
  } else {
    if (amax == 0.f) { memset(dst + 2, 0, 32); return M3G_OK; }
    for (int i = 0; i < 32; ++i)
      dst[2 + i] = static_cast<uint8_t>(static_cast<int8_t>(sat_round_clamp(src[i] / ds, -127, 127)));
  }
  return M3G_OK;
}
}  // namespace

extern "C" {

// quantize_q4_0 (src/quant.rs:206-234).
int m3g_quantize_q4_0(const float* src, uint64_t src_len, uint8_t* dst, uint64_t dst_len) {
  return quantize_block(src, src_len, dst, dst_len, 7, true);
}

// quantize_q8_0 (src/quant.rs:239-264).
int m3g_quantize_q8_0(const float* src, uint64_t src_len, uint8_t* dst, uint64_t dst_len) {
  return quantize_block(src, src_len, dst, dst_len, 127, false);
}

// ---------------------------------------------------------------- decoders
// dequantize (src/quant.rs:120-173) on the device.
int m3g_dequantize_dev(const uint8_t* src, uint64_t src_len, uint32_t dtype, float* dst, uint64_t n,
                       void* stream) {
  if ((!src && src_len) || (!dst && n)) return fail(M3G_EINVAL, "null pointer");
  int fmt = -1;
  switch (dtype) {
    case 0: if (src_len < n * 4) return fail(M3G_ENONE, "F32 source too short"); fmt = 0; break;
    case 1: if (src_len < n * 2) return fail(M3G_ENONE, "F16 source too short"); fmt = 1; break;
    case 2:
      if (n % 32) return fail(M3G_ENONE, "Q4_0 needs n %% 32 == 0");
      if (src_len < n / 32 * 18) return fail(M3G_EPANIC, "Q4_0 source too short (reference assert!)");
      fmt = 2; break;
    case 12: case 13:
      if (n % 256) return fail(M3G_ENONE, "Q4_K needs n %% 256 == 0");
      if (src_len < n / 256 * 144) return fail(M3G_EPANIC, "Q4_K source too short (reference assert!)");
      fmt = 12; break;
    case 14:
      if (n % 256) return fail(M3G_ENONE, "Q6_K needs n %% 256 == 0");
      if (src_len < n / 256 * 210) return fail(M3G_ENONE, "Q6_K source too short");
      fmt = 14; break;
    case 8:
      if (n % 32) return fail(M3G_ENONE, "Q8_0 needs n %% 32 == 0");
      if (src_len < n / 32 * 34) return fail(M3G_ENONE, "Q8_0 source too short");
      fmt = 8; break;
    default:
      return fail(M3G_ENONE, "dequantize: unsupported dtype %u", dtype);
  }
  if (n == 0) return M3G_OK;
  DevState* ds = nullptr;
  if (int rc = current_dev_state(&ds)) return rc;
  const long long units = (fmt <= 1) ? static_cast<long long>(n) : static_cast<long long>(n) / (fmt == 12 || fmt == 14 ? 256 : 32) * 32;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((units + 255) / 256, 16ll * ds->sms)));
  cudaError_t e = m3g::launch_dequant(fmt, src, dst, static_cast<long long>(n), grid, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "k_dequant launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return M3G_OK;
}

int m3g_dequantize(const uint8_t* src, uint64_t src_len, uint32_t dtype, float* dst, uint64_t n) {
  if ((!src && src_len) || (!dst && n)) return fail(M3G_EINVAL, "null pointer");
  DevState* ds = nullptr;
  if (int rc = current_dev_state(&ds)) return rc;
  DevBuf ds_src, ds_dst;
  M3G_CUDA(ds_src.alloc(src_len));
  M3G_CUDA(ds_dst.alloc(n * sizeof(float)));
  if (src_len) M3G_CUDA(cudaMemcpy(ds_src.p, src, src_len, cudaMemcpyHostToDevice));
  int rc = m3g_dequantize_dev(static_cast<const uint8_t*>(ds_src.p), src_len, dtype, static_cast<float*>(ds_dst.p),
                              n, nullptr);
  if (rc) return rc;
  if (n) M3G_CUDA(cudaMemcpy(dst, ds_dst.p, n * sizeof(float), cudaMemcpyDeviceToHost));
  return M3G_OK;
}

// ---------------------------------------------------------------- fused GEMV
int m3g_matvec_quant_dev(const float* x, const uint8_t* raw, uint64_t raw_len, uint32_t dtype, uint64_t in_dim,
                         uint64_t out_dim, uint64_t batch, float* y, void* stream) {
  FmtInfo f;
  if (int rc = gemv_rules(dtype, raw_len, in_dim, out_dim, f)) return rc;
  if (!x || !raw || !y) return fail(M3G_EINVAL, "null pointer");
  if (batch == 0) return M3G_OK;
  DevState* ds = nullptr;
  if (int rc = current_dev_state(&ds)) return rc;
  return gemv_batch_launch(*ds, f, raw, x, y, static_cast<long long>(in_dim), static_cast<long long>(out_dim),
                           static_cast<long long>(batch), static_cast<cudaStream_t>(stream));
}

// matvec_quant (src/matvec_quant.rs:87-109) with host buffers.
int m3g_matvec_quant(const float* x, uint64_t x_len, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                     uint64_t in_dim, uint64_t out_dim, float* y) {
  if (x_len != in_dim) return fail(M3G_ENONE, "x has %llu elements, in_dim is %llu",
                                   static_cast<unsigned long long>(x_len), static_cast<unsigned long long>(in_dim));
  FmtInfo f;
  if (int rc = gemv_rules(dtype, raw_len, in_dim, out_dim, f)) return rc;
  if (!x || !raw || !y) return fail(M3G_EINVAL, "null pointer");
  DevState* ds = nullptr;
  if (int rc = current_dev_state(&ds)) return rc;
  uint64_t need = 0;
  raw_len_rule(dtype, in_dim * out_dim, need);
  DevBuf dw, dx, dy;
  M3G_CUDA(dw.alloc(need));
  M3G_CUDA(dx.alloc(in_dim * sizeof(float)));
  M3G_CUDA(dy.alloc(out_dim * sizeof(float)));
  M3G_CUDA(cudaMemcpy(dw.p, raw, need, cudaMemcpyHostToDevice));
  M3G_CUDA(cudaMemcpy(dx.p, x, in_dim * sizeof(float), cudaMemcpyHostToDevice));
  if (int rc = gemv_launch(*ds, f, static_cast<const uint8_t*>(dw.p), static_cast<const float*>(dx.p),
                           static_cast<float*>(dy.p), static_cast<long long>(in_dim),
                           static_cast<long long>(out_dim), nullptr))
    return rc;
  M3G_CUDA(cudaMemcpy(y, dy.p, out_dim * sizeof(float), cudaMemcpyDeviceToHost));
  return check_status(*ds);
}

int m3g_device_status(int device, uint32_t* out, int clear) {
  DevState* ds = nullptr;
  if (int rc = dev_state(device, &ds)) return rc;
  int prev = 0;
  M3G_CUDA(cudaGetDevice(&prev));
  M3G_CUDA(cudaSetDevice(device));
  uint32_t s = 0;
  cudaError_t e = cudaMemcpy(&s, ds->status, sizeof s, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(ds->status, 0, sizeof s);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "m3g_device_status");
  if (out) *out = s;
  return M3G_OK;
}

}  // extern "C"

// ================================================================ offload context
struct ResidentTensor {
  uint32_t dtype = 0;
  uint64_t in_dim = 0, out_dim = 0, raw_len = 0;
  uint8_t* d_raw = nullptr;
};

struct m3g_offload {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint64_t max_in = 0, max_out = 0;
  uint64_t cap_batch = 0;
  float* d_x = nullptr;
  // Host-buffer calls write y into d_out + 16 and report kernel status in the
  // context's own word at d_out, so one copy brings both back to h_out.
  uint8_t* d_out = nullptr;
  float* d_y = nullptr;           // d_out + 16
  uint32_t* d_status = nullptr;   // d_out
  float* h_x = nullptr;           // pinned staging
  uint8_t* h_out = nullptr;       // pinned: [status (16 bytes)][y]
  float* h_y = nullptr;           // h_out + 16
  uint32_t* h_status = nullptr;   // h_out
  // Batch-1 calls on the tensor-core plan move x, y and the status word
  // through mapped pinned memory instead of copy-engine transfers: a small
  // kernel pulls x in (the GEMV's weight stream overlaps it), the GEMV stores
  // y straight into host memory, and its last CTA stores the status word.
  float* hm_x = nullptr;
  float* hm_x_dev = nullptr;
  float* hm_y = nullptr;
  float* hm_y_dev = nullptr;
  uint32_t* hm_st = nullptr;      // [status, sequence number of the last call done]
  uint32_t* hm_st_dev = nullptr;
  uint32_t host_seq = 0;          // sequence number of the last mapped call (device copy at d_out + 8)
  uint64_t calls = 0;
  std::unordered_map<uint64_t, ResidentTensor> tensors;
  // Host-buffer calls: one captured graph per tensor (copy x in, GEMV, copy y
  // and the status word out), valid for the batch, weight and staging
  // buffers it was captured with.
  struct HostGraph {
    cudaGraphExec_t exec = nullptr;
    uint64_t batch = 0;
    const uint8_t* w = nullptr;
    bool mapped = false;
  };
  std::unordered_map<uint64_t, HostGraph> graphs;
  bool graphs_ok = true;  // cleared if a capture ever fails: calls then run eagerly
};

namespace {

// Makes `dev` current for the scope; a no-op (one query) when it already is.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev == dev) prev = -1;
    else cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

void drop_graphs(m3g_offload* c) {
  for (auto& kv : c->graphs)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  c->graphs.clear();
}

void free_io(m3g_offload* c) {
  if (c->stream) cudaStreamSynchronize(c->stream);  // mapped calls return before their kernels exit
  drop_graphs(c);
  if (c->d_x) cudaFree(c->d_x);
  if (c->d_out) cudaFree(c->d_out);
  if (c->h_x) cudaFreeHost(c->h_x);
  if (c->h_out) cudaFreeHost(c->h_out);
  c->d_x = c->d_y = c->h_x = c->h_y = nullptr;
  c->d_out = c->h_out = nullptr;
  c->d_status = c->h_status = nullptr;
  c->cap_batch = 0;
}

void free_mapped(m3g_offload* c) {
  for (void* p : {static_cast<void*>(c->hm_x), static_cast<void*>(c->hm_y), static_cast<void*>(c->hm_st)})
    if (p) cudaFreeHost(p);
  c->hm_x = c->hm_x_dev = c->hm_y = c->hm_y_dev = nullptr;
  c->hm_st = c->hm_st_dev = nullptr;
}

// Mapped pinned buffers of the batch-1 host call (allocated once, at create).
int ensure_mapped(m3g_offload* c) {
  if (c->hm_x) return M3G_OK;
  const size_t nx = static_cast<size_t>(std::max<uint64_t>(c->max_in, 16));
  const size_t ny = static_cast<size_t>(std::max<uint64_t>(c->max_out, 16));
  M3G_CUDA(cudaHostAlloc(&c->hm_x, nx * sizeof(float), cudaHostAllocMapped));
  M3G_CUDA(cudaHostAlloc(&c->hm_y, ny * sizeof(float), cudaHostAllocMapped));
  M3G_CUDA(cudaHostAlloc(&c->hm_st, 64, cudaHostAllocMapped));
  M3G_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->hm_x_dev), c->hm_x, 0));
  M3G_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->hm_y_dev), c->hm_y, 0));
  M3G_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->hm_st_dev), c->hm_st, 0));
  c->hm_st[0] = c->hm_st[1] = 0u;
  return M3G_OK;
}

int ensure_io(m3g_offload* c, uint64_t batch) {
  if (batch <= c->cap_batch) return M3G_OK;
  free_io(c);
  const size_t nx = static_cast<size_t>(std::max<uint64_t>(c->max_in, 16) * batch);
  const size_t ny = static_cast<size_t>(std::max<uint64_t>(c->max_out, 16) * batch);
  M3G_CUDA(cudaMalloc(&c->d_x, nx * sizeof(float)));
  M3G_CUDA(cudaMalloc(&c->d_out, 16 + ny * sizeof(float)));
  M3G_CUDA(cudaMemset(c->d_out, 0, 16));
  // The device's sequence word at d_out + 8 starts again at 0, and so do the
  // host's count and the mapped copy (no kernel is in flight: free_io synced).
  c->host_seq = 0;
  if (c->hm_st) c->hm_st[1] = 0u;
  M3G_CUDA(cudaMallocHost(&c->h_x, nx * sizeof(float)));
  M3G_CUDA(cudaMallocHost(&c->h_out, 16 + ny * sizeof(float)));
  c->d_status = reinterpret_cast<uint32_t*>(c->d_out);
  c->d_y = reinterpret_cast<float*>(c->d_out + 16);
  c->h_status = reinterpret_cast<uint32_t*>(c->h_out);
  c->h_y = reinterpret_cast<float*>(c->h_out + 16);
  c->cap_batch = batch;
  return M3G_OK;
}

}  // namespace

extern "C" {

// GpuOffload::try_new (src/inference_gpu.rs:58-127).
int m3g_offload_create(int device, uint64_t max_in, uint64_t max_out, m3g_offload** out) {
  if (!out) return fail(M3G_EINVAL, "null out");
  *out = nullptr;
  DevState* ds = nullptr;
  if (int rc = dev_state(device, &ds)) return rc;
  DeviceGuard g(device);
  auto* c = new m3g_offload();
  c->device = device;
  c->max_in = max_in;
  c->max_out = max_out;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return cuda_fail(e, "cudaStreamCreate");
  }
  int rc = ensure_io(c, 1);
  if (!rc && g_tune.offload_mapped) {
    rc = ensure_mapped(c);
    if (rc) {  // no mapped memory here: every call takes the copy path
      free_mapped(c);
      rc = M3G_OK;
    }
  }
  if (rc) {
    free_io(c);
    cudaStreamDestroy(c->stream);
    delete c;
    return rc;
  }
  *out = c;
  return M3G_OK;
}

void m3g_offload_destroy(m3g_offload* c) {
  if (!c) return;
  DeviceGuard g(c->device);
  cudaDeviceSynchronize();
  drop_graphs(c);
  for (auto& kv : c->tensors) cudaFree(kv.second.d_raw);
  free_io(c);
  free_mapped(c);
  cudaStreamDestroy(c->stream);
  delete c;
}

// GpuOffload::upload (src/inference_gpu.rs:131-177).
int m3g_offload_upload(m3g_offload* c, uint64_t tidx, uint32_t dtype, const uint8_t* raw, uint64_t raw_len,
                       uint64_t in_dim, uint64_t out_dim) {
  if (!c) return fail(M3G_EINVAL, "null context");
  FmtInfo f;
  if (!fmt_info(dtype, f)) return fail(M3G_ENONE, "upload: dtype %u has no fused kernel", dtype);
  if (in_dim == 0 || out_dim == 0) return fail(M3G_ENONE, "upload: zero dimension");
  if (in_dim > (1ull << 31) || out_dim > (1ull << 31)) return fail(M3G_EINVAL, "upload: dimension too large");
  uint64_t expect = 0;
  if (!raw_len_rule(dtype, in_dim * out_dim, expect) || expect != raw_len)
    return fail(M3G_ENONE, "upload: raw_len %llu != quant_raw_len %llu", static_cast<unsigned long long>(raw_len),
                static_cast<unsigned long long>(expect));
  if (!raw) return fail(M3G_EINVAL, "null raw");
  DeviceGuard g(c->device);
  ResidentTensor t;
  t.dtype = dtype;
  t.in_dim = in_dim;
  t.out_dim = out_dim;
  t.raw_len = raw_len;
  M3G_CUDA(cudaMalloc(&t.d_raw, raw_len + 16));
  cudaError_t e = cudaMemcpy(t.d_raw, raw, raw_len, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(t.d_raw);
    return cuda_fail(e, "upload copy");
  }
  auto it = c->tensors.find(tidx);
  if (it != c->tensors.end()) {
    cudaDeviceSynchronize();  // the old bytes may be in use on any stream
    auto gi = c->graphs.find(tidx);
    if (gi != c->graphs.end()) {
      if (gi->second.exec) cudaGraphExecDestroy(gi->second.exec);
      c->graphs.erase(gi);
    }
    cudaFree(it->second.d_raw);
    it->second = t;
  } else {
    c->tensors.emplace(tidx, t);
  }
  return M3G_OK;
}

int m3g_offload_offloaded(const m3g_offload* c, uint64_t tidx) { return c && c->tensors.count(tidx) ? 1 : 0; }

uint64_t m3g_offload_tensor_count(const m3g_offload* c) { return c ? c->tensors.size() : 0; }

uint64_t m3g_offload_calls(const m3g_offload* c) { return c ? c->calls : 0; }

const uint8_t* m3g_offload_tensor_ptr(const m3g_offload* c, uint64_t tidx) {
  if (!c) return nullptr;
  auto it = c->tensors.find(tidx);
  return it == c->tensors.end() ? nullptr : it->second.d_raw;
}

int m3g_offload_matvec_dev(m3g_offload* c, uint64_t tidx, const float* x, uint64_t batch, float* y, void* stream) {
  if (!c) return fail(M3G_EINVAL, "null context");
  auto it = c->tensors.find(tidx);
  if (it == c->tensors.end()) return fail(M3G_ENOTFOUND, "tensor %llu not resident", static_cast<unsigned long long>(tidx));
  if (!x || !y) return fail(M3G_EINVAL, "null pointer");
  const ResidentTensor& t = it->second;
  FmtInfo f;
  fmt_info(t.dtype, f);
  DevState* ds = nullptr;
  if (int rc = dev_state(c->device, &ds)) return rc;
  DeviceGuard g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL: the legacy default stream
  int rc = gemv_batch_launch(*ds, f, t.d_raw, x, y, static_cast<long long>(t.in_dim),
                             static_cast<long long>(t.out_dim), static_cast<long long>(batch), st);
  if (!rc) ++c->calls;
  return rc;
}

// GpuOffload::matvec (src/inference_gpu.rs:188-237), host x and y, batched.
int m3g_offload_matvec_batch(m3g_offload* c, uint64_t tidx, const float* x, uint64_t batch, uint64_t in_dim,
                             uint64_t out_dim, float* y) {
  if (!c) return fail(M3G_EINVAL, "null context");
  auto it = c->tensors.find(tidx);
  if (it == c->tensors.end()) return fail(M3G_ENOTFOUND, "tensor %llu not resident", static_cast<unsigned long long>(tidx));
  const ResidentTensor& t = it->second;
  if (t.in_dim != in_dim || t.out_dim != out_dim)
    return fail(M3G_ENONE, "matvec dims %llux%llu differ from upload %llux%llu",
                static_cast<unsigned long long>(in_dim), static_cast<unsigned long long>(out_dim),
                static_cast<unsigned long long>(t.in_dim), static_cast<unsigned long long>(t.out_dim));
  if (in_dim > c->max_in || out_dim > c->max_out) return fail(M3G_ENONE, "matvec exceeds max_in/max_out");
  if (!x || !y) return fail(M3G_EINVAL, "null pointer");
  if (batch == 0) return M3G_OK;
  DeviceGuard g(c->device);
  if (int rc = ensure_io(c, batch)) return rc;
  const size_t bx = static_cast<size_t>(in_dim * batch) * sizeof(float);
  const size_t by = static_cast<size_t>(out_dim * batch) * sizeof(float);
  DevState* ds = nullptr;
  if (int rc = dev_state(c->device, &ds)) return rc;
  // The kernels of this call report into the context's status word.
  DevState dsc = *ds;
  dsc.status = c->d_status;
  FmtInfo f;
  fmt_info(t.dtype, f);
  DevState dsm = dsc;  // mapped path: the GEMV's last CTA returns the status word itself
  dsm.status_host = c->hm_st_dev;
  dsm.fin_cnt = reinterpret_cast<unsigned int*>(c->d_out + 4);
  // Batch 1 on the tensor-core plan (plain stores of y, no atomics): x, y and
  // the status word go through mapped pinned memory.  Otherwise: copy in,
  // GEMV, one copy out of [status | y].
  MmaPlan probe;
  const bool mapped = batch == 1 && c->hm_x && g_tune.offload_mapped && in_dim % 4 == 0 && !g_tune.force_generic &&
                      g_tune.mma && plan_mma(f, static_cast<long long>(in_dim), static_cast<long long>(out_dim),
                                             t.d_raw, c->d_x, *ds, probe, g_tune.mma_coresident != 0);
  memcpy(mapped ? c->hm_x : c->h_x, x, bx);
  auto enqueue = [&]() -> int {
    if (mapped) {
      cudaError_t e = m3g::launch_host_x_in(c->hm_x_dev, c->d_x, static_cast<long long>(in_dim), c->stream);
      if (e != cudaSuccess) return cuda_fail(e, "x copy-in kernel");
      if (int rc = gemv_batch_launch(dsm, f, t.d_raw, c->d_x, c->hm_y_dev, static_cast<long long>(t.in_dim),
                                     static_cast<long long>(t.out_dim), 1, c->stream))
        return rc;
      ++c->calls;
      g_launches.fetch_add(1, std::memory_order_relaxed);
      return M3G_OK;
    }
    M3G_CUDA(cudaMemcpyAsync(c->d_x, c->h_x, bx, cudaMemcpyHostToDevice, c->stream));
    if (int rc = gemv_batch_launch(dsc, f, t.d_raw, c->d_x, c->d_y, static_cast<long long>(t.in_dim),
                                   static_cast<long long>(t.out_dim), static_cast<long long>(batch), c->stream))
      return rc;
    ++c->calls;
    M3G_CUDA(cudaMemcpyAsync(c->h_out, c->d_out, 16 + by, cudaMemcpyDeviceToHost, c->stream));
    return M3G_OK;
  };
  m3g_offload::HostGraph* hg = nullptr;
  if (g_tune.offload_graph && c->graphs_ok) {
    auto gi = c->graphs.find(tidx);
    if (gi != c->graphs.end() &&
        (gi->second.batch != batch || gi->second.w != t.d_raw || gi->second.mapped != mapped)) {
      if (gi->second.exec) cudaGraphExecDestroy(gi->second.exec);
      c->graphs.erase(gi);
      gi = c->graphs.end();
    }
    if (gi == c->graphs.end()) {
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      const uint64_t calls0 = c->calls;  // capturing is not a call
      bool ok = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
      const int rc = ok ? enqueue() : M3G_OK;
      c->calls = calls0;
      ok = (cudaStreamEndCapture(c->stream, &graph) == cudaSuccess) && ok && rc == M3G_OK;
      if (ok) ok = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();  // a failed capture leaves no sticky error; clear the last one
      if (ok) {
        gi = c->graphs.emplace(tidx, m3g_offload::HostGraph{exec, batch, t.d_raw, mapped}).first;
      } else {
        if (exec) cudaGraphExecDestroy(exec);
        c->graphs_ok = false;  // run this and later calls eagerly
      }
    }
    if (gi != c->graphs.end()) hg = &gi->second;
  }
  if (hg) {
    M3G_CUDA(cudaGraphLaunch(hg->exec, c->stream));
    ++c->calls;
  } else if (int rc = enqueue()) {
    return rc;
  }
  if (mapped) {
    // The GEMV's last CTA publishes this call's sequence number after y and
    // the status word (system-scope fences); wait for it on the host, bounded,
    // instead of synchronising the stream.  On time-out fall back to the sync,
    // which also surfaces a launch error.
    const uint32_t want = c->host_seq + 1u;
    volatile uint32_t* seq = c->hm_st + 1;
    bool seen = *seq == want;
    if (!seen) {
      const auto t0 = std::chrono::steady_clock::now();
      for (uint32_t it = 1; !(seen = *seq == want); ++it)
        if ((it & 1023u) == 0u && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2)) break;
    }
    if (!seen) {
      M3G_CUDA(cudaStreamSynchronize(c->stream));
      seen = *seq == want;
    }
    if (!seen) return fail(M3G_ECUDA, "host-buffer GEMV did not report completion");
    c->host_seq = want;
  } else {
    M3G_CUDA(cudaStreamSynchronize(c->stream));
  }
  memcpy(y, mapped ? c->hm_y : c->h_y, by);
  const uint32_t bits = mapped ? *static_cast<volatile uint32_t*>(c->hm_st) : *c->h_status;
  if (bits) {
    cudaMemset(c->d_status, 0, sizeof(uint32_t));
    if (mapped) *static_cast<volatile uint32_t*>(c->hm_st) = 0u;
    return fail(M3G_ETIMEOUT, "a bounded wait in the GEMV gave up (status 0x%x)", bits);
  }
  return M3G_OK;
}

int m3g_offload_matvec(m3g_offload* c, uint64_t tidx, const float* x, uint64_t in_dim, uint64_t out_dim,
                       float* y) {
  return m3g_offload_matvec_batch(c, tidx, x, 1, in_dim, out_dim, y);
}

}  // extern "C"
