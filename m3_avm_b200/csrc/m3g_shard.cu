// m3g_shard.cu -- output-row sharding of a GEMV across the GPUs of one node.
//
// Each rank (one process per GPU) keeps rows [r*RPR, min(out, (r+1)*RPR)) of
// a weight tensor resident, RPR = ceil(out_dim / world).  A matvec computes
// the local rows straight into this rank's slot of the gather buffer, and the
// other ranks' slots arrive in one of two ways:
//
//  * peer stores (tuning key shard_p2p, when every rank can map every other
//    rank's exchange region over NVLink): the GEMV's epilogue stores each row into
//    every peer's exchange region as well, and the CTA that completes the
//    rank's rows adds 1 to every peer's arrival counter after a system-scope
//    fence -- the all-gather is fused into the GEMV, tile by tile.  A small
//    kernel then waits (bounded) for all ranks' arrivals and copies the
//    peers' slots into the caller's buffer.  The regions are double-buffered
//    by call parity, so a rank one call ahead never overwrites rows a peer
//    still copies;
//  * otherwise (the default) one in-place NCCL all-gather of the fp32 slices.
//
// Measured on 2 B200s (Q4_K 14336 x 4096 per call): the local rows alone take
// 6.0 us, with the NCCL all-gather 16.4-18.2 us, with peer stores 19.3 us.
// A stamped copy shows where the peer-store form goes: each CTA's
// system-scope fence after its remote stores takes ~3.4 us, the last CTA's
// fence and arrival atomics ~3.7 us (a release reduction instead waited as
// long), then the gather.  NCCL stays the default.
//
// Communicator creation is non-blocking with a wall-clock limit: a rank that
// never joins makes create() abort the communicator and return M3G_ETIMEOUT
// instead of hanging.
#include <chrono>
#include <cstring>
#include <thread>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/m3gemv.h"
#include "m3g_device.cuh"
#include "m3g_internal.h"

namespace m3g {
int host_fail(int code, const char* fmt, ...);
int gemv_device(int device, uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, float* y,
                long long in_dim, long long out_dim, cudaStream_t st);
bool block_geometry(uint32_t dtype, int* be, int* bb);
}  // namespace m3g

namespace {

struct ShardTensor {
  uint32_t dtype = 0;
  uint64_t in_dim = 0, out_dim = 0;
  uint64_t rpr = 0, row_begin = 0, rows_local = 0;
  uint64_t bytes_local = 0;
  uint8_t* d_raw = nullptr;
};

int nccl_fail(ncclResult_t r, const char* what) {
  return m3g::host_fail(M3G_ENCCL, "%s: %s", what, ncclGetErrorString(r));
}

}  // namespace

namespace m3g {

// The communicator is non-blocking (so that a missing rank cannot hang
// creation): a call may return ncclInProgress, which is completed here by
// polling the communicator's state for at most timeout_s seconds.
int nccl_settle(ncclComm_t comm, ncclResult_t r, const char* what, double timeout_s) {
  if (r == ncclSuccess) return M3G_OK;
  if (r != ncclInProgress) return nccl_fail(r, what);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) return nccl_fail(ncclInternalError, what);
    if (st == ncclSuccess) return M3G_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s)
      return m3g::host_fail(M3G_ETIMEOUT, "%s did not complete within %.1f s", what, timeout_s);
    std::this_thread::yield();
  }
}

// A non-blocking communicator on the current device; a rank that never joins
// makes creation abort after timeout_s with M3G_ETIMEOUT.
int nccl_comm_create(int rank, int world, const uint8_t* id128, double timeout_s, ncclComm_t* out) {
  *out = nullptr;
  ncclUniqueId id;
  memcpy(id.internal, id128, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress || (r == ncclSuccess && comm)) {
    ncclResult_t st = ncclInProgress;
    if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) {
      r = ncclInternalError;
      break;
    }
    if (st == ncclSuccess) {
      r = ncclSuccess;
      break;
    }
    if (st != ncclInProgress) {
      r = st;
      break;
    }
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > timeout_s) {
      ncclCommAbort(comm);
      return m3g::host_fail(M3G_ETIMEOUT, "NCCL communicator init did not complete within %.1f s", timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess) {
    if (comm) ncclCommAbort(comm);
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  *out = comm;
  return M3G_OK;
}

// Finalize (bounded) then destroy; abort when finalising does not complete.
void nccl_comm_close(ncclComm_t comm, double timeout_s) {
  if (!comm) return;
  if (nccl_settle(comm, ncclCommFinalize(comm), "ncclCommFinalize", timeout_s) == M3G_OK)
    ncclCommDestroy(comm);
  else
    ncclCommAbort(comm);
}

}  // namespace m3g

using m3g::nccl_settle;

struct m3g_shard {
  int device = 0, rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;
  uint64_t max_in = 0, max_out = 0;
  std::unordered_map<uint64_t, ShardTensor> tensors;
  float* d_x = nullptr;    // [batch][max_in]
  float* d_ws = nullptr;   // gather buffer [world][batch][RPR]
  uint64_t cap_x = 0, cap_ws = 0;
  float* h_x = nullptr;    // pinned staging of the host-buffer call: x
  float* h_ws = nullptr;   // and the gathered y, [world][batch][RPR]
  uint64_t cap_hx = 0, cap_hws = 0;
  uint64_t calls = 0;
  double timeout_s = 60.0;
  // Peer-store exchange: this rank's region (counters, then two halves of
  // world * rpr_cap floats) and every rank's region mapped here.
  bool p2p = false;
  uint8_t* region = nullptr;
  uint8_t* peer_base[m3g::kMaxPeers] = {};
  uint64_t rpr_cap = 0;  // rows per rank the region holds
};

namespace {

// Exchange region layout: counters first (a peer adds to arr), then the two
// halves of the gathered rows.
constexpr size_t kArrOff = 0;     // u32: arrivals (every rank adds 1 per call)
constexpr size_t kDoneOff = 64;   // u32: this rank's GEMV CTAs done in this call
constexpr size_t kStepOff = 128;  // i32: calls completed (parity of the halves)
constexpr size_t kZeroOff = 192;  // i32: constant 0 (the GEMV's per-call count base)
constexpr size_t kFinOff = 256;   // u32: gather CTAs finished in this call
constexpr size_t kRowsOff = 512;  // f32 [2][world * rpr_cap]

// Waits (bounded) until every rank's rows of this call have arrived, copies
// the other ranks' slots from this call's half of the region into y (this
// rank's slot is already there), and closes the call: the last CTA clears the
// per-call counts and advances the step.
__global__ void __launch_bounds__(256) k_shard_gather(uint8_t* region, unsigned world, int rank, long long rpr,
                                                      long long rpr_cap, float* __restrict__ y, long long n,
                                                      uint32_t* status, unsigned long long wait_ns) {
  m3g::grid_dep_wait();
  // The next call's GEMV may start streaming its weights; it reads this
  // region's step and writes peers' rows only after its own grid dependency.
  m3g::grid_dep_launch();
  const unsigned* arr = reinterpret_cast<const unsigned*>(region + kArrOff);
  int* step = reinterpret_cast<int*>(region + kStepOff);
  __shared__ int s_step;
  if (threadIdx.x == 0) {
    const int s = *reinterpret_cast<volatile int*>(step);
    const unsigned target = static_cast<unsigned>(s + 1) * world;
    if (!m3g::wait_count_bounded(arr, target, wait_ns)) atomicOr(status, m3g::kStatusPeerTimeout);
    s_step = s;
  }
  __syncthreads();
  const int s = s_step;
  const float* src = reinterpret_cast<const float*>(region + kRowsOff) + static_cast<long long>(s & 1) * world * rpr_cap;
  const long long mine0 = static_cast<long long>(rank) * rpr, mine1 = mine0 + rpr;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (i >= mine0 && i < mine1) continue;
    y[i] = __ldcg(src + (i / rpr) * rpr_cap + i % rpr);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned* fin = reinterpret_cast<unsigned*>(region + kFinOff);
    if (atomicAdd(fin, 1u) == gridDim.x - 1) {
      *fin = 0u;
      *reinterpret_cast<unsigned*>(region + kDoneOff) = 0u;
      *step = s + 1;
      __threadfence();
    }
  }
}

// Maps every rank's exchange region (CUDA IPC over NVLink): handles are
// swapped with one NCCL all-gather and the ranks agree (MIN all-reduce) that
// every mapping opened; otherwise every rank keeps the NCCL path.
int open_peer_regions(m3g_shard* c) {
  c->p2p = false;
  c->peer_base[c->rank] = c->region;
  constexpr int kRec = 72;  // 64-byte handle + ok flag
  uint8_t rec[kRec] = {};
  cudaIpcMemHandle_t mine;
  memset(&mine, 0, sizeof mine);
  int ok = c->region && cudaIpcGetMemHandle(&mine, c->region) == cudaSuccess ? 1 : 0;
  cudaGetLastError();
  memcpy(rec, &mine, sizeof mine);
  memcpy(rec + 64, &ok, sizeof ok);
  uint8_t* dev = nullptr;
  cudaError_t e = cudaMalloc(&dev, static_cast<size_t>(kRec) * c->world + 16);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ENOMEM, "peer handles: %s", cudaGetErrorString(e));
  std::vector<uint8_t> all(static_cast<size_t>(kRec) * c->world);
  int rc = M3G_OK;
  e = cudaMemcpy(dev + kRec * c->rank, rec, kRec, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = nccl_settle(c->comm, ncclAllGather(dev + kRec * c->rank, dev, kRec, ncclUint8, c->comm, c->stream),
                     "ncclAllGather(ipc handles)", c->timeout_s);
    if (!rc) e = cudaStreamSynchronize(c->stream);
    if (!rc && e == cudaSuccess) e = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost);
  }
  if (rc || e != cudaSuccess) {
    cudaFree(dev);
    return rc ? rc : m3g::host_fail(M3G_ECUDA, "peer handle exchange: %s", cudaGetErrorString(e));
  }
  int mine_ok = 1;
  for (int p = 0; p < c->world; ++p) {
    int okp = 0;
    memcpy(&okp, all.data() + kRec * p + 64, sizeof okp);
    if (!okp) mine_ok = 0;
  }
  for (int p = 0; p < c->world && mine_ok; ++p) {
    if (p == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, all.data() + kRec * p, sizeof h);
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      mine_ok = 0;
      break;
    }
    c->peer_base[p] = static_cast<uint8_t*>(ptr);
  }
  int* flag = reinterpret_cast<int*>(dev);
  e = cudaMemcpy(flag, &mine_ok, sizeof mine_ok, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = nccl_settle(c->comm, ncclAllReduce(flag, flag, 1, ncclInt, ncclMin, c->comm, c->stream),
                     "ncclAllReduce(peer agreement)", c->timeout_s);
    if (!rc) e = cudaStreamSynchronize(c->stream);
  }
  int all_ok = 0;
  if (!rc && e == cudaSuccess) e = cudaMemcpy(&all_ok, flag, sizeof all_ok, cudaMemcpyDeviceToHost);
  cudaFree(dev);
  if (!rc && e == cudaSuccess && all_ok) {
    c->p2p = true;
    return M3G_OK;
  }
  for (int p = 0; p < c->world; ++p)
    if (p != c->rank && c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  for (int p = 0; p < c->world; ++p) c->peer_base[p] = p == c->rank ? c->region : nullptr;
  if (rc) return rc;
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "peer agreement: %s", cudaGetErrorString(e));
  return M3G_OK;
}

struct Dev {
  int prev = -1;
  explicit Dev(int d) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(d);
  }
  ~Dev() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int grow(float** p, uint64_t* cap, uint64_t n) {
  if (n <= *cap) return M3G_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(p, n * sizeof(float));
  if (e != cudaSuccess) return m3g::host_fail(M3G_ENOMEM, "shard buffer: %s", cudaGetErrorString(e));
  *cap = n;
  return M3G_OK;
}

// Pinned host staging, grown on demand: the copies are then one DMA each.
int grow_pinned(float** p, uint64_t* cap, uint64_t n) {
  if (n <= *cap) return M3G_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMallocHost(p, n * sizeof(float));
  if (e != cudaSuccess) return m3g::host_fail(M3G_ENOMEM, "shard staging: %s", cudaGetErrorString(e));
  *cap = n;
  return M3G_OK;
}

}  // namespace

extern "C" {

// Row partition of a sharded tensor: pure host arithmetic, no device.
int m3g_shard_plan(uint32_t dtype, uint64_t in_dim, uint64_t out_dim, int world, int rank, uint64_t* row_begin,
                   uint64_t* rows_local, uint64_t* rows_per_rank, uint64_t* byte_begin, uint64_t* byte_len) {
  int be = 0, bb = 0;
  if (!m3g::block_geometry(dtype, &be, &bb)) return m3g::host_fail(M3G_ENONE, "shard: dtype %u has no fused kernel", dtype);
  if (world < 1 || rank < 0 || rank >= world) return m3g::host_fail(M3G_EINVAL, "shard: rank %d of %d", rank, world);
  if (in_dim == 0 || out_dim == 0) return m3g::host_fail(M3G_ENONE, "shard: zero dimension");
  if (in_dim % static_cast<uint64_t>(be))
    return m3g::host_fail(M3G_ENONE, "shard: rows must hold whole blocks (in_dim %% %d != 0)", be);
  const uint64_t rb = in_dim / be * bb;
  const uint64_t rpr = (out_dim + world - 1) / world;
  const uint64_t b0 = std::min<uint64_t>(out_dim, rpr * rank);
  const uint64_t b1 = std::min<uint64_t>(out_dim, rpr * (rank + 1));
  if (row_begin) *row_begin = b0;
  if (rows_local) *rows_local = b1 - b0;
  if (rows_per_rank) *rows_per_rank = rpr;
  if (byte_begin) *byte_begin = b0 * rb;
  if (byte_len) *byte_len = (b1 - b0) * rb;
  return M3G_OK;
}

int m3g_shard_unique_id(uint8_t* out128) {
  if (!out128) return m3g::host_fail(M3G_EINVAL, "null id buffer");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(out128, id.internal, NCCL_UNIQUE_ID_BYTES);
  return M3G_OK;
}

int m3g_shard_create(int device, int rank, int world, const uint8_t* id128, uint64_t max_in, uint64_t max_out,
                     double timeout_s, m3g_shard** out) {
  if (!out || !id128) return m3g::host_fail(M3G_EINVAL, "null argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return m3g::host_fail(M3G_EINVAL, "rank %d of %d", rank, world);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return m3g::host_fail(M3G_ECUDA, "no CUDA device %d", device);
  Dev g(device);
  auto* c = new m3g_shard();
  c->device = device;
  c->rank = rank;
  c->world = world;
  c->max_in = max_in;
  c->max_out = max_out;
  c->timeout_s = timeout_s;
  if (int rc = m3g::nccl_comm_create(rank, world, id128, timeout_s, &c->comm)) {
    delete c;
    return rc;
  }
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    ncclCommAbort(c->comm);
    delete c;
    return m3g::host_fail(M3G_ECUDA, "cudaStreamCreate: %s", cudaGetErrorString(e));
  }
  // The device's kernel state (status word, SM count) is made now, so that a
  // later matvec may be captured into a CUDA graph (no allocation inside it).
  uint32_t* status = nullptr;
  if (int rc = m3g::status_word(device, &status)) {
    cudaStreamDestroy(c->stream);
    ncclCommAbort(c->comm);
    delete c;
    return rc;
  }
  // Peer-store exchange region.  Every rank makes the same decision (the
  // tuning key is process-wide) and joins the collective agreement, even one
  // whose allocation failed: it then votes no and every rank keeps NCCL.
  if (world > 1 && world <= m3g::kMaxPeers && m3g::shard_p2p_enabled(world)) {
    c->rpr_cap = (max_out + world - 1) / world;
    const size_t bytes = kRowsOff + 2 * static_cast<size_t>(world) * c->rpr_cap * sizeof(float);
    cudaError_t ea = cudaMalloc(&c->region, bytes);
    if (ea == cudaSuccess) ea = cudaMemset(c->region, 0, kRowsOff);
    if (ea != cudaSuccess) {
      cudaGetLastError();
      if (c->region) cudaFree(c->region);
      c->region = nullptr;
    }
    if (int rc = open_peer_regions(c)) {
      m3g_shard_destroy(c);
      return rc;
    }
  }
  *out = c;
  return M3G_OK;
}

void m3g_shard_destroy(m3g_shard* c) {
  if (!c) return;
  Dev g(c->device);
  cudaDeviceSynchronize();
  if (c->p2p && c->comm) {
    // no rank may unmap or free a region while another still stores into it
    int* one = nullptr;
    if (cudaMalloc(&one, sizeof(int)) == cudaSuccess) {
      if (nccl_settle(c->comm, ncclAllReduce(one, one, 1, ncclInt, ncclSum, c->comm, c->stream),
                      "ncclAllReduce(teardown barrier)", c->timeout_s) == M3G_OK)
        cudaStreamSynchronize(c->stream);
      cudaFree(one);
    }
  }
  for (int p = 0; p < c->world && p < m3g::kMaxPeers; ++p)
    if (p != c->rank && c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  if (c->region) cudaFree(c->region);
  for (auto& kv : c->tensors) cudaFree(kv.second.d_raw);
  if (c->d_x) cudaFree(c->d_x);
  if (c->d_ws) cudaFree(c->d_ws);
  if (c->h_x) cudaFreeHost(c->h_x);
  if (c->h_ws) cudaFreeHost(c->h_ws);
  if (c->comm) {
    ncclResult_t r = ncclCommFinalize(c->comm);
    if (nccl_settle(c->comm, r, "ncclCommFinalize", c->timeout_s) == M3G_OK) ncclCommDestroy(c->comm);
    else ncclCommAbort(c->comm);
  }
  cudaStreamDestroy(c->stream);
  delete c;
}

// Keep this rank's rows of a full GGUF tensor resident.
int m3g_shard_upload(m3g_shard* c, uint64_t tidx, uint32_t dtype, const uint8_t* raw, uint64_t raw_len,
                     uint64_t in_dim, uint64_t out_dim) {
  if (!c || !raw) return m3g::host_fail(M3G_EINVAL, "null argument");
  uint64_t need = 0;
  if (m3g_quant_raw_len(dtype, in_dim * out_dim, &need) != M3G_OK || need != raw_len)
    return m3g::host_fail(M3G_ENONE, "shard upload: raw_len %llu != quant_raw_len %llu",
                          static_cast<unsigned long long>(raw_len), static_cast<unsigned long long>(need));
  ShardTensor t;
  uint64_t b0 = 0;
  if (int rc = m3g_shard_plan(dtype, in_dim, out_dim, c->world, c->rank, &t.row_begin, &t.rows_local, &t.rpr, &b0,
                              &t.bytes_local))
    return rc;
  t.dtype = dtype;
  t.in_dim = in_dim;
  t.out_dim = out_dim;
  Dev g(c->device);
  cudaError_t e = cudaMalloc(&t.d_raw, t.bytes_local + 16);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ENOMEM, "shard upload: %s", cudaGetErrorString(e));
  if (t.bytes_local) e = cudaMemcpy(t.d_raw, raw + b0, t.bytes_local, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(t.d_raw);
    return m3g::host_fail(M3G_ECUDA, "shard upload copy: %s", cudaGetErrorString(e));
  }
  auto it = c->tensors.find(tidx);
  if (it != c->tensors.end()) {
    cudaDeviceSynchronize();  // the old bytes may be in use on any stream
    cudaFree(it->second.d_raw);
    it->second = t;
  } else {
    c->tensors.emplace(tidx, t);
  }
  return M3G_OK;
}

// Y[b][out] for device x [b][in]: local rows, then one in-place all-gather.
// y must hold batch * rows_per_rank * world floats; with batch == 1 the
// result is y[0 .. out_dim), with batch > 1 it is y[rank][b][rows_per_rank]
// (use m3g_shard_matvec for the [b][out] layout).
int m3g_shard_matvec_dev(m3g_shard* c, uint64_t tidx, const float* x, uint64_t batch, float* y, void* stream) {
  if (!c || !x || !y) return m3g::host_fail(M3G_EINVAL, "null argument");
  auto it = c->tensors.find(tidx);
  if (it == c->tensors.end()) return m3g::host_fail(M3G_ENOTFOUND, "tensor %llu not resident",
                                                    static_cast<unsigned long long>(tidx));
  const ShardTensor& t = it->second;
  if (batch == 0) return M3G_OK;
  Dev g(c->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL: the legacy default stream
  float* slot = y + static_cast<uint64_t>(c->rank) * batch * t.rpr;
  // The peer-store form needs every rank to hold rows and a tensor-core plan
  // for the shape; both depend only on the tensor, so every rank decides alike.
  const bool p2p = c->p2p && batch == 1 && t.rpr <= c->rpr_cap &&
                   static_cast<uint64_t>(c->world - 1) * t.rpr < t.out_dim &&
                   m3g::fused_plannable(c->device, t.dtype, static_cast<long long>(t.in_dim),
                                        static_cast<long long>(t.rows_local));
  if (p2p) {
    const float* xin = x;
    if (reinterpret_cast<uintptr_t>(x) % 16) {  // the tensor-core plan reads x 16 bytes at a time
      if (int rc = grow(&c->d_x, &c->cap_x, t.in_dim)) return rc;
      cudaError_t e = cudaMemcpyAsync(c->d_x, x, t.in_dim * sizeof(float), cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "shard x copy: %s", cudaGetErrorString(e));
      xin = c->d_x;
    }
    m3g::PeerIO io;
    for (int p = 0; p < c->world; ++p) {
      io.peer_cnt[p] = reinterpret_cast<unsigned int*>(c->peer_base[p] + kArrOff);
      if (p != c->rank)
        io.peer_y[p] = reinterpret_cast<float*>(c->peer_base[p] + kRowsOff) + static_cast<uint64_t>(c->rank) * c->rpr_cap;
    }
    io.npeer = c->world;
    io.done_cnt = reinterpret_cast<unsigned int*>(c->region + kDoneOff);
    io.step = reinterpret_cast<const int*>(c->region + kZeroOff);
    io.ystep = reinterpret_cast<const int*>(c->region + kStepOff);
    io.ystride = static_cast<long long>(c->world) * static_cast<long long>(c->rpr_cap);
    if (int rc = m3g::gemv_fused(c->device, t.dtype, t.d_raw, t.bytes_local, xin, nullptr, nullptr, nullptr,
                                 m3g::kXPlain, slot, static_cast<long long>(t.in_dim),
                                 static_cast<long long>(t.rows_local), st, false, nullptr, false, 0, &io))
      return rc;
    uint32_t* status = nullptr;
    if (int rc = m3g::status_word(c->device, &status)) return rc;
    const long long n = static_cast<long long>(c->world) * static_cast<long long>(t.rpr);
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(512, (n + 255) / 256)));
    // Programmatic dependent launch: the gather's CTAs (256 threads, no
    // shared memory) fit beside the GEMV's and wait in griddepcontrol.wait,
    // so no launch gap separates the two.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_shard_gather, c->region, static_cast<unsigned>(c->world), c->rank,
                                       static_cast<long long>(t.rpr), static_cast<long long>(c->rpr_cap), y, n,
                                       status, m3g::peer_wait_ns());
    if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "shard gather launch: %s", cudaGetErrorString(e));
    ++c->calls;
    return M3G_OK;
  }
  if (t.rows_local) {
    for (uint64_t b = 0; b < batch; ++b) {
      int rc = m3g::gemv_device(c->device, t.dtype, t.d_raw, t.bytes_local, x + b * t.in_dim, slot + b * t.rpr,
                                static_cast<long long>(t.in_dim), static_cast<long long>(t.rows_local), st);
      if (rc) return rc;
    }
  }
  ncclResult_t r = ncclAllGather(slot, y, batch * t.rpr, ncclFloat, c->comm, st);
  if (int rc = nccl_settle(c->comm, r, "ncclAllGather", c->timeout_s)) return rc;
  ++c->calls;
  return M3G_OK;
}

// Host x [batch][in] -> host y [batch][out], full output on every rank.
int m3g_shard_matvec(m3g_shard* c, uint64_t tidx, const float* x, uint64_t batch, uint64_t in_dim, uint64_t out_dim,
                     float* y) {
  if (!c || !x || !y) return m3g::host_fail(M3G_EINVAL, "null argument");
  auto it = c->tensors.find(tidx);
  if (it == c->tensors.end()) return m3g::host_fail(M3G_ENOTFOUND, "tensor %llu not resident",
                                                    static_cast<unsigned long long>(tidx));
  const ShardTensor& t = it->second;
  if (t.in_dim != in_dim || t.out_dim != out_dim) return m3g::host_fail(M3G_ENONE, "shard matvec: dims differ");
  if (batch == 0) return M3G_OK;
  Dev g(c->device);
  const uint64_t ws = static_cast<uint64_t>(c->world) * batch * t.rpr;
  if (int rc = grow(&c->d_x, &c->cap_x, batch * in_dim)) return rc;
  if (int rc = grow(&c->d_ws, &c->cap_ws, ws)) return rc;
  if (int rc = grow_pinned(&c->h_x, &c->cap_hx, batch * in_dim)) return rc;
  if (int rc = grow_pinned(&c->h_ws, &c->cap_hws, ws)) return rc;
  // one pinned copy in, the GEMV and the exchange, one pinned copy of the
  // whole gather buffer out; the host then reorders [rank][b][rpr] -> [b][out]
  memcpy(c->h_x, x, batch * in_dim * sizeof(float));
  cudaError_t e = cudaMemcpyAsync(c->d_x, c->h_x, batch * in_dim * sizeof(float), cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "shard x copy: %s", cudaGetErrorString(e));
  if (int rc = m3g_shard_matvec_dev(c, tidx, c->d_x, batch, c->d_ws, c->stream)) return rc;
  e = cudaMemcpyAsync(c->h_ws, c->d_ws, ws * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "shard y copy: %s", cudaGetErrorString(e));
  e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return m3g::host_fail(M3G_ECUDA, "shard sync: %s", cudaGetErrorString(e));
  for (uint64_t b = 0; b < batch; ++b) {
    for (int r = 0; r < c->world; ++r) {
      const uint64_t r0 = std::min<uint64_t>(out_dim, t.rpr * r), r1 = std::min<uint64_t>(out_dim, t.rpr * (r + 1));
      if (r1 > r0)
        memcpy(y + b * out_dim + r0, c->h_ws + (static_cast<uint64_t>(r) * batch + b) * t.rpr,
               (r1 - r0) * sizeof(float));
    }
  }
  return M3G_OK;
}

int m3g_shard_info(const m3g_shard* c, uint64_t tidx, uint64_t* row_begin, uint64_t* rows_local,
                   uint64_t* rows_per_rank) {
  if (!c) return m3g::host_fail(M3G_EINVAL, "null context");
  auto it = c->tensors.find(tidx);
  if (it == c->tensors.end()) return m3g::host_fail(M3G_ENOTFOUND, "tensor not resident");
  if (row_begin) *row_begin = it->second.row_begin;
  if (rows_local) *rows_local = it->second.rows_local;
  if (rows_per_rank) *rows_per_rank = it->second.rpr;
  return M3G_OK;
}

uint64_t m3g_shard_calls(const m3g_shard* c) { return c ? c->calls : 0; }

int m3g_shard_exchange(const m3g_shard* c) {
  if (!c) return 0;
  if (c->world == 1) return 0;
  return c->p2p ? 2 : 1;
}

}  // extern "C"
