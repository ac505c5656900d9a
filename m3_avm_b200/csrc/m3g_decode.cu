// m3g_decode.cu -- device-resident greedy decode of a Llama-style model.
//
// The decode step of RealInference::forward_one (src/inference.rs:953-1152)
// with every MATVEC on the fused tensor-core GEMV, everything else on small
// kernels, and no host round trip between tokens:
//
//   k_embed           token_embd row of tokens[pos] -> hidden (exact block decode)
//   per layer:
//     GEMV  qkv       rms_norm(hidden) * attn_norm, fused into the GEMV input;
//                     q|k|v rows concatenated into one weight when they share a dtype
//     k_attention_split  RoPE of q and k, K/V appended at pos, softmax attention
//                     over positions [0, pos], one 8-CTA cluster per query head
//                     (GQA: head hh reads KV head hh / (n_heads / n_kv_heads))
//     GEMV  o         hidden += W_o att (residual fused in the epilogue)
//     GEMV  gate|up   rms_norm(hidden) * ffn_norm input, gate and up rows
//                     interleaved in blocks of 8 so the epilogue writes silu(g) * u
//     GEMV  down      hidden += W_down (silu(g) * u)
//   GEMV  head        rms_norm(hidden) * output_norm -> logits
//                     whose epilogue also reduces (logit, row) to the greedy
//                     pick with one 64-bit atomicMax per CTA
//   k_pick_step       the pick (lowest index of the largest logit) into
//                     tokens[pos + 1] unless that slot holds a given prompt
//                     token, then pos += 1
//
// Sharded over the GPUs of a node (one process per GPU, one NCCL
// communicator), each rank keeps the attention weights whole and only its
// rows of gate/up, down and the vocab head: after gate|up one in-place
// all-gather assembles silu(g) * u, after down one assembles the hidden
// state, and one 64-bit MAX all-reduce merges the ranks' greedy keys.  Every
// row is computed exactly as on one GPU, so the ranks hold identical state.
//
// The position and the token stream live in device memory, so one captured
// CUDA graph replays every step; kernels chain with programmatic dependent
// launch so each GEMV starts streaming its weights while the previous kernel
// finishes.  The KV cache is compact (n_kv_heads * head_dim floats per
// position and layer); the reference stores it repeated to the full hidden
// width, which holds the same values.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/m3gemv.h"
#include "m3g_device.cuh"
#include "m3g_formats.cuh"
#include "m3g_internal.h"

namespace m3g {
int host_fail(int code, const char* fmt, ...);
bool block_geometry(uint32_t dtype, int* be, int* bb);
int nccl_settle(ncclComm_t comm, ncclResult_t r, const char* what, double timeout_s);
int nccl_comm_create(int rank, int world, const uint8_t* id128, double timeout_s, ncclComm_t* out);
void nccl_comm_close(ncclComm_t comm, double timeout_s);
}  // namespace m3g

namespace cg = cooperative_groups;

namespace m3g {
namespace {

struct AttnArgs {
  const float* qkv;   // [q: n_heads*HD][k: kvd][v: kvd]
  float* kc;          // this layer's K cache [max_pos][kvd]
  float* vc;          // this layer's V cache [max_pos][kvd]
  const float* rope;  // [max_pos][HD/2][cos, sin]
  const int* pos;
  float* out;         // [n_heads*HD]
  uint32_t* status;
  int groups;         // n_heads / n_kv_heads
  int kvd;            // n_kv_heads * HD
  int qd;             // n_heads * HD
  int max_pos;
  float scale;        // 1 / sqrt(HD)
};

// Attention of one step, one thread-block cluster of kAttnSplit CTAs per
// query head: RoPE of q and of the head's KV-group k (split-half pairs,
// rounded as the reference's apply_rope), the first CTA of the group's first
// head appends K/V at pos, and each CTA takes a contiguous slice of the
// positions with a local softmax (max m, sum l, weighted V o).  Scores are
// the reference's sequential dot products (bit-identical for identical q and
// k).  CTA 0 of the cluster reads the others' partials through distributed
// shared memory and combines them, out = sum_p e^(m_p - M) o_p / sum_p
// e^(m_p - M) l_p (GQA: query head hh reads KV head hh / groups).
constexpr int kAttnSplit = 8;
constexpr int kAttnSplitThreads = 128;

template <int HD>
__global__ void __launch_bounds__(kAttnSplitThreads) k_attention_split(const AttnArgs a) {
  constexpr int HALF = HD / 2, DPL = HD / 32, NW = kAttnSplitThreads / 32;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                  // [HD]
  float* kn = qs + HD;             // [HD]
  float* vn = kn + HD;             // [HD]
  float* part = vn + HD;           // [NW][HD]
  float* red = part + NW * HD;     // [64]
  float* res = red + 64;           // [2 + HD]: m, l, o of this CTA (read by CTA 0)
  float* sc = res + 2 + HD;        // [chunk] scores, then weights
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hh = blockIdx.x / kAttnSplit, kv = hh / a.groups;
  // The position, its RoPE row and the cached K/V rows before it were written
  // by kernels that completed before this step's q|k|v GEMV began, so they are
  // loaded (into registers) before that GEMV -- the grid dependency -- ends.
  const int pos = *a.pos;
  const bool pos_ok = pos >= 0 && pos < a.max_pos;
  const int npos = pos_ok ? pos + 1 : 0;
  const int chunk = (npos + kAttnSplit - 1) / kAttnSplit;
  const int i0 = min(npos, rank * chunk), i1 = min(npos, i0 + chunk);
  const int ic = min(i1, pos);  // cached rows are i0 .. ic-1
  constexpr bool kPre = HD == 64;
  constexpr int VP = kPre ? 16 : 1;  // V rows per warp held in registers
  float4 kreg[kPre ? HD / 4 : 1];
  float vreg[VP][DPL];
  const bool kpre = kPre && i0 + tid < ic;
  if (kpre) {
    const float4* kr = reinterpret_cast<const float4*>(a.kc + static_cast<size_t>(i0 + tid) * a.kvd + kv * HD);
#pragma unroll
    for (int j = 0; j < (kPre ? HD / 4 : 1); ++j) kreg[j] = kr[j];
  }
  if (kPre) {
#pragma unroll
    for (int j = 0; j < VP; ++j) {
      const int i = i0 + warp + NW * j;
      if (i < ic) {
        const float* vr = a.vc + static_cast<size_t>(i) * a.kvd + kv * HD + DPL * lane;
#pragma unroll
        for (int d = 0; d < DPL; ++d) vreg[j][d] = vr[d];
      }
    }
  }
  float cs_c = 0.f, cs_s = 0.f;
  if (pos_ok && tid < HALF) {
    cs_c = a.rope[static_cast<size_t>(pos) * HD + 2 * tid];
    cs_s = a.rope[static_cast<size_t>(pos) * HD + 2 * tid + 1];
  }
  grid_dep_wait();
  grid_dep_launch();
  if (!pos_ok && tid == 0 && rank == 0 && hh == 0) atomicOr(a.status, kStatusBadPos);
  if (pos_ok) {
    const float* q = a.qkv + hh * HD;
    const float* k = a.qkv + a.qd + kv * HD;
    static_assert(HALF <= kAttnSplitThreads, "one RoPE pair per thread");
    for (int i = tid; i < HALF; i += kAttnSplitThreads) {
      const float c = cs_c, s = cs_s;
      float x0 = q[i], x1 = q[i + HALF];
      qs[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      qs[i + HALF] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
      x0 = k[i];
      x1 = k[i + HALF];
      kn[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      kn[i + HALF] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    for (int i = tid; i < HD; i += kAttnSplitThreads) vn[i] = a.qkv[a.qd + a.kvd + kv * HD + i];
  }
  __syncthreads();
  if (pos_ok && rank == 0 && hh % a.groups == 0) {
    for (int i = tid; i < HD; i += kAttnSplitThreads) {
      a.kc[static_cast<size_t>(pos) * a.kvd + kv * HD + i] = kn[i];
      a.vc[static_cast<size_t>(pos) * a.kvd + kv * HD + i] = vn[i];
    }
  }
  float lmax = -INFINITY;
  for (int i = i0 + tid; i < i1; i += kAttnSplitThreads) {
    const float* kr = i == pos ? kn : a.kc + static_cast<size_t>(i) * a.kvd + kv * HD;
    const bool inreg = kpre && i == i0 + tid;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < HD; j += 4) {
      const float4 k4 = inreg ? kreg[kPre ? j / 4 : 0] : *reinterpret_cast<const float4*>(kr + j);
      const float4 q4 = *reinterpret_cast<const float4*>(qs + j);
      dot = __fadd_rn(dot, __fmul_rn(q4.x, k4.x));
      dot = __fadd_rn(dot, __fmul_rn(q4.y, k4.y));
      dot = __fadd_rn(dot, __fmul_rn(q4.z, k4.z));
      dot = __fadd_rn(dot, __fmul_rn(q4.w, k4.w));
    }
    const float s = __fmul_rn(dot, a.scale);
    sc[i - i0] = s;
    lmax = fmaxf(lmax, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, o));
  if (lane == 0) red[warp] = lmax;
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) mx = fmaxf(mx, red[w]);
  float lsum = 0.f;
  for (int i = i0 + tid; i < i1; i += kAttnSplitThreads) {
    const float e = expf(__fsub_rn(sc[i - i0], mx));
    sc[i - i0] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) red[32 + warp] = lsum;
  __syncthreads();
  float acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; ++d) acc[d] = 0.f;
  int vfirst = i0 + warp;  // rows still to read from memory start here
  if (kPre) {
#pragma unroll
    for (int j = 0; j < VP; ++j) {
      const int i = i0 + warp + NW * j;
      if (i < ic) {
        const float w = sc[i - i0];
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[d] += w * vreg[j][d];
        vfirst = i + NW;
      }
    }
  }
#pragma unroll 4
  for (int i = vfirst; i < i1; i += NW) {
    const float w = sc[i - i0];
    const float* vr = (i == pos ? vn : a.vc + static_cast<size_t>(i) * a.kvd + kv * HD) + DPL * lane;
    if (DPL == 2) {
      const float2 v2 = *reinterpret_cast<const float2*>(vr);
      acc[0] += w * v2.x;
      acc[1] += w * v2.y;
    } else {
#pragma unroll
      for (int d = 0; d < DPL; d += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vr + d);
        acc[d] += w * v4.x;
        acc[d + 1] += w * v4.y;
        acc[d + 2] += w * v4.z;
        acc[d + 3] += w * v4.w;
      }
    }
  }
#pragma unroll
  for (int d = 0; d < DPL; ++d) part[warp * HD + DPL * lane + d] = acc[d];
  __syncthreads();
  for (int i = tid; i < HD; i += kAttnSplitThreads) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) o += part[w * HD + i];
    res[2 + i] = o;
  }
  if (tid == 0) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) l += red[32 + w];
    res[0] = i1 > i0 ? mx : -INFINITY;
    res[1] = l;
  }
  cluster.sync();  // every CTA's partial is in its shared memory
  if (rank == 0) {
    for (int i = tid; i < HD; i += kAttnSplitThreads) {
      float M = -INFINITY;
#pragma unroll
      for (int p = 0; p < kAttnSplit; ++p) M = fmaxf(M, cluster.map_shared_rank(res, p)[0]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int p = 0; p < kAttnSplit; ++p) {
        const float* r = cluster.map_shared_rank(res, p);
        const float f = r[0] == -INFINITY ? 0.f : expf(__fsub_rn(r[0], M));
        L = fmaf(f, r[1], L);
        O = fmaf(f, r[2 + i], O);
      }
      if (pos_ok) a.out[hh * HD + i] = __fdiv_rn(O, L);
    }
  }
  cluster.sync();  // the partials stay readable until CTA 0 has combined them
}

// hidden = row tokens[pos] of the embedding, decoded exactly as the
// reference's dequantize does (embedding_row, src/inference.rs:903-944).
__global__ void __launch_bounds__(256) k_embed(const uint8_t* __restrict__ w, int dtype, int be, int bb,
                                               const int* tokens, const int* pos, float* hidden, int h, int vocab,
                                               int max_pos, uint32_t* status) {
  grid_dep_wait();
  grid_dep_launch();
  const int p = *pos;
  int tok = (p >= 0 && p < max_pos) ? tokens[p] : -1;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, kStatusBadToken);
    tok = 0;
  }
  const int e = blockIdx.x * 256 + threadIdx.x;
  if (e >= h) return;
  const long long idx = static_cast<long long>(tok) * h + e;
  float v;
  if (dtype == 0) {
    v = reinterpret_cast<const float*>(w)[idx];
  } else if (dtype == 1) {
    v = __half2float(reinterpret_cast<const __half*>(w)[idx]);
  } else {
    const uint8_t* blk = w + (idx / be) * bb;
    const int off = static_cast<int>(idx % be);
    switch (dtype) {
      case 14: v = q6k_elem(blk, off); break;
      case 8: v = q8_0_elem(blk, off); break;
      case 2: v = q4_0_elem(blk, off); break;
      default: v = q4k_elem(blk, off); break;
    }
  }
  hidden[e] = v;
}

// Greedy pick (sample_with_params with top_k = 1: the first index holding
// the largest logit) from the key the head GEMV's epilogue reduced with
// atomicMax, and the step's bookkeeping; the key is cleared for the next step.
__global__ void __launch_bounds__(32) k_pick_step(unsigned long long* key, int* pos, int* tokens, const int* nfixed,
                                                  int max_pos, int* last, int* step, const unsigned int* wait_cnt,
                                                  unsigned int wait_mul, int key_by_step, uint32_t* status,
                                                  unsigned long long wait_ns) {
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x != 0) return;
  if (wait_cnt) {  // sharded with peer stores: every rank's head CTAs have merged their keys
    const unsigned int target = static_cast<unsigned int>(*step + 1) * wait_mul;
    if (!wait_count_bounded(wait_cnt, target, wait_ns)) atomicOr(status, kStatusPeerTimeout);
  }
  if (key_by_step) key += *step & 1;  // this step's slot (a rank one step ahead merges into the other)
  const unsigned long long k = *key;
  const int pick = k ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k)) : 0;  // 0: every logit NaN
  const int p = *pos, next = p + 1;
  *last = pick;
  if (next <= max_pos && next >= *nfixed) tokens[next] = pick;
  *pos = next;
  *key = 0ull;
  *step += 1;
}

template <class Kern, class... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <class Kern, class... Args>
cudaError_t launch_pdl_cluster(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace
}  // namespace m3g

// ================================================================ engine
namespace {

using m3g::host_fail;

#define DEC_CUDA(call)                                                                            \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return host_fail(M3G_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

constexpr int kSlotEmbd = 0, kSlotOutNorm = 1, kSlotOut = 2, kSlotLayer0 = 3, kPerLayer = 9;
enum { kAttnNorm = 0, kQ, kK, kV, kO, kFfnNorm, kGate, kUp, kDown };

struct Tensor {
  uint8_t* d = nullptr;  // device bytes (norms: f32)
  uint64_t len = 0;
  uint32_t dtype = 0;
  int in = 0, out = 0;   // matrix shape held here (a row shard's rows); norms: in = out = hidden
  int row0 = 0;          // first row of the full tensor held here
  bool set = false;
};

// A GEMV of the step: rows [0, out) of `w` (possibly several tensors' rows
// concatenated) applied to in_dim inputs.
struct Gemv {
  const uint8_t* w = nullptr;
  uint64_t len = 0;
  uint32_t dtype = 0;
  int in = 0, out = 0;
};

}  // namespace

struct m3g_decoder {
  int device = 0;
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  double timeout_s = 60.0;
  int Fr = 0, hr = 0, Vr = 0;  // rows per rank of gate/up (each), down, head
  m3g_decoder_config cfg{};
  int hd = 0, kvd = 0;
  cudaStream_t st = nullptr;
  std::vector<Tensor> t;
  // Concatenated weights built at the first step (q|k|v and gate|up per layer).
  std::vector<uint8_t*> fused;
  std::vector<Gemv> qkv, gu;  // per layer; .w == nullptr: launch the parts separately
  bool prepared = false;
  // Activations and state.
  float *hidden = nullptr, *qkvb = nullptr, *att = nullptr, *gub = nullptr, *logits = nullptr;
  float *rope = nullptr, *kc = nullptr, *vc = nullptr;
  int *dpos = nullptr, *tokens = nullptr, *nfixed = nullptr, *last = nullptr;
  unsigned long long* key = nullptr;  // greedy pick of the step (argmax epilogue of the head GEMV)
  // One allocation holds what other ranks write into: hidden, the FFN
  // activation, the greedy key, the arrival counters (2 per layer + head) and
  // the step counter.  With peer stores its IPC mapping is opened by every rank.
  uint8_t* xregion = nullptr;
  size_t xregion_bytes = 0, off_hidden = 0, off_gub = 0, off_key = 0, off_cnt = 0;
  unsigned int* cnt = nullptr;   // arrivals of every rank, per exchange: [layer][ffn, hidden], head
  unsigned int* done = nullptr;  // this rank's finished CTAs, same slots
  int* dstep = nullptr;          // steps completed (advanced by k_pick_step)
  bool p2p = false;
  bool shard_ffn = false;  // world > 1: FFN rows split too (else every rank keeps the layers, the head is split)
  uint8_t* peer_base[m3g::kMaxPeers] = {};
  int* h_io = nullptr;  // pinned: [0] token / nfixed staging, [1] last token
  uint32_t* status = nullptr;
  int pos = 0;           // host mirror of the device position
  bool pending = false;  // tokens[pos] holds the greedy pick of the last step
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // Prompt steps before the last need no logits: one GPU replays this graph,
  // the step without the vocab head, for them.
  cudaGraph_t graph_nohead = nullptr;
  cudaGraphExec_t exec_nohead = nullptr;
  bool use_graph = true;
  uint64_t steps = 0;
};

namespace {

// Shared memory of k_attention_split: q, k, v of this position, per-warp
// partials, reductions, the CTA's (m, l, o) and its slice of the scores.
size_t attn_split_smem(const m3g_decoder* d) {
  const size_t hd = static_cast<size_t>(d->hd), nw = m3g::kAttnSplitThreads / 32;
  const size_t chunk = (d->cfg.max_pos + m3g::kAttnSplit - 1) / m3g::kAttnSplit;
  return sizeof(float) * (3 * hd + nw * hd + 64 + 2 + hd + chunk);
}

// Rank p's copy of a region offset (this rank's own region for p == rank).
template <class T>
T* peer_at(const m3g_decoder* d, int p, size_t off) {
  return reinterpret_cast<T*>(d->peer_base[p] + off);
}

int slot_shape(const m3g_decoder* d, int slot, int* in, int* out, bool* is_norm) {
  const int h = static_cast<int>(d->cfg.hidden), F = static_cast<int>(d->cfg.ffn);
  *is_norm = false;
  if (slot == kSlotEmbd || slot == kSlotOut) {
    *in = h;
    *out = static_cast<int>(d->cfg.vocab);
    return M3G_OK;
  }
  if (slot == kSlotOutNorm) {
    *in = *out = h;
    *is_norm = true;
    return M3G_OK;
  }
  const int kind = (slot - kSlotLayer0) % kPerLayer;
  switch (kind) {
    case kAttnNorm: case kFfnNorm: *in = *out = h; *is_norm = true; break;
    case kQ: case kO: *in = h; *out = h; break;
    case kK: case kV: *in = h; *out = d->kvd; break;
    case kGate: case kUp: *in = h; *out = F; break;
    default: *in = F; *out = h; break;
  }
  return M3G_OK;
}

bool gemv_dtype(uint32_t dt) { return dt == 2 || dt == 8 || dt == 12 || dt == 13 || dt == 14; }

// Rows [row0, row0 + rows) of a slot's full tensor that this rank keeps.
void shard_rows(const m3g_decoder* d, int slot, int full_out, int* row0, int* rows) {
  *row0 = 0;
  *rows = full_out;
  if (d->world == 1 || slot < kSlotLayer0) {
    if (slot == kSlotOut && d->world > 1) {
      *row0 = d->rank * d->Vr;
      *rows = std::max(0, std::min(full_out, *row0 + d->Vr) - *row0);
    }
    return;
  }
  const int kind = (slot - kSlotLayer0) % kPerLayer;
  if (!d->shard_ffn) return;
  if (kind == kGate || kind == kUp) {
    *row0 = d->rank * d->Fr;
    *rows = d->Fr;
  } else if (kind == kDown) {
    *row0 = d->rank * d->hr;
    *rows = d->hr;
  }
}

Gemv part(const Tensor& x) { return Gemv{x.d, x.len, x.dtype, x.in, x.out}; }

// Concatenate the rows of tensors that share dtype and in_dim into one
// weight so that a single GEMV launch covers them.
int concat_rows(m3g_decoder* d, const std::vector<const Tensor*>& parts, Gemv& g) {
  g = Gemv{};
  for (const Tensor* p : parts)
    if (p->dtype != parts[0]->dtype || p->in != parts[0]->in) return M3G_OK;  // launched separately
  uint64_t total = 0;
  int rows = 0;
  for (const Tensor* p : parts) {
    uint64_t need = 0;
    if (m3g_quant_raw_len(p->dtype, static_cast<uint64_t>(p->in) * p->out, &need)) return M3G_OK;
    if (need % 16) return M3G_OK;  // rows of the next part would start unaligned
    total += need;
    rows += p->out;
  }
  uint8_t* buf = nullptr;
  DEC_CUDA(cudaMalloc(&buf, total));
  d->fused.push_back(buf);
  uint64_t off = 0;
  for (const Tensor* p : parts) {
    uint64_t need = 0;
    m3g_quant_raw_len(p->dtype, static_cast<uint64_t>(p->in) * p->out, &need);
    DEC_CUDA(cudaMemcpy(buf + off, p->d, need, cudaMemcpyDeviceToDevice));
    off += need;
  }
  g = Gemv{buf, total, parts[0]->dtype, parts[0]->in, rows};
  return M3G_OK;
}

// gate|up rows interleaved in blocks of 8 (8 gate rows, then the same 8 up
// rows) for the GEMV's SwiGLU epilogue, which then writes silu(g) * u.
int interleave_gate_up(m3g_decoder* d, const Tensor& gate, const Tensor& up, Gemv& g) {
  g = Gemv{};
  if (gate.dtype != up.dtype || gate.in != up.in || gate.out != up.out || gate.out % 8) return M3G_OK;
  uint64_t need = 0;
  if (m3g_quant_raw_len(gate.dtype, static_cast<uint64_t>(gate.in) * gate.out, &need)) return M3G_OK;
  const uint64_t rb = need / static_cast<uint64_t>(gate.out);
  if (rb * gate.out != need || rb % 16) return M3G_OK;  // rows must be whole, 16-byte multiples
  uint8_t* buf = nullptr;
  DEC_CUDA(cudaMalloc(&buf, 2 * need));
  d->fused.push_back(buf);
  const size_t blk = 8 * rb, nblk = static_cast<size_t>(gate.out / 8);
  DEC_CUDA(cudaMemcpy2D(buf, 2 * blk, gate.d, blk, blk, nblk, cudaMemcpyDeviceToDevice));
  DEC_CUDA(cudaMemcpy2D(buf + blk, 2 * blk, up.d, blk, blk, nblk, cudaMemcpyDeviceToDevice));
  g = Gemv{buf, 2 * need, gate.dtype, gate.in, 2 * gate.out};
  return M3G_OK;
}

int prepare(m3g_decoder* d) {
  if (d->prepared) return M3G_OK;
  for (size_t s = 0; s < d->t.size(); ++s)
    if (!d->t[s].set) return host_fail(M3G_EINVAL, "decoder tensor slot %zu was never uploaded", s);
  const int L = static_cast<int>(d->cfg.n_layers);
  d->qkv.assign(L, Gemv{});
  d->gu.assign(L, Gemv{});
  for (int l = 0; l < L; ++l) {
    const Tensor* T = &d->t[kSlotLayer0 + kPerLayer * l];
    if (int rc = concat_rows(d, {&T[kQ], &T[kK], &T[kV]}, d->qkv[l])) return rc;
    if (int rc = interleave_gate_up(d, T[kGate], T[kUp], d->gu[l])) return rc;
    if (d->shard_ffn && !d->gu[l].w)
      return host_fail(M3G_EINVAL, "sharded decode needs gate and up of one dtype with 16-byte rows (layer %d)", l);
  }
  d->prepared = true;
  return M3G_OK;
}

int gemv(m3g_decoder* d, const Gemv& g, const float* x, const float* x2, const float* gamma, const float* res,
         int xmode, float* y, unsigned long long* key = nullptr, bool swiglu = false) {
  return m3g::gemv_fused(d->device, g.dtype, g.w, g.len, x, x2, gamma, res, xmode, y, g.in, g.out, d->st, true, key,
                         swiglu);
}

// Enqueue one decode step on d->st (also the body the graph captures).
// head = false (one GPU only) leaves out the vocab head GEMV: the pick then
// reads the cleared key and, the next token being a prompt token, writes none.
int enqueue_step(m3g_decoder* d, bool head = true) {
  const int h = static_cast<int>(d->cfg.hidden), F = static_cast<int>(d->cfg.ffn);
  const int L = static_cast<int>(d->cfg.n_layers), V = static_cast<int>(d->cfg.vocab);
  const int mp = static_cast<int>(d->cfg.max_pos);
  const bool pp = d->world > 1 && d->p2p;  // greedy keys merge by peer atomics
  const bool pp_ffn = pp && d->shard_ffn;   // FFN rows exchanged by peer stores too
  // Exchange slots: 2l = silu(g)*u of layer l, 2l+1 = hidden after layer l, 2L = greedy key.
  auto exchange = [&](int slot, size_t region_off, size_t elem_off, bool rows) {
    m3g::PeerIO io;
    io.npeer = d->world;
    for (int p = 0; p < d->world; ++p) {
      if (rows && p != d->rank) io.peer_y[p] = peer_at<float>(d, p, region_off) + elem_off;
      io.peer_cnt[p] = peer_at<unsigned int>(d, p, d->off_cnt) + slot;
    }
    io.done_cnt = d->done + slot;
    io.step = d->dstep;
    return io;
  };
  auto wait_on = [&](m3g::PeerIO& io, int slot) {
    io.wait_cnt = d->cnt + slot;
    io.wait_mul = static_cast<unsigned int>(d->world);
    io.step = d->dstep;
  };
  const Tensor& E = d->t[kSlotEmbd];
  int be = 1, bb = 4;
  if (E.dtype == 1) bb = 2;
  else if (E.dtype != 0) m3g::block_geometry(E.dtype, &be, &bb);
  DEC_CUDA(m3g::launch_pdl(m3g::k_embed, dim3((h + 255) / 256), dim3(256), 0, d->st, static_cast<const uint8_t*>(E.d),
                           static_cast<int>(E.dtype), be, bb, static_cast<const int*>(d->tokens),
                           static_cast<const int*>(d->dpos), d->hidden, h, V, mp, d->status));
  const size_t split_smem = attn_split_smem(d);
  for (int l = 0; l < L; ++l) {
    const Tensor* T = &d->t[kSlotLayer0 + kPerLayer * l];
    const float* g_attn = reinterpret_cast<const float*>(T[kAttnNorm].d);
    const float* g_ffn = reinterpret_cast<const float*>(T[kFfnNorm].d);
    // q|k|v reads hidden, which holds every rank's rows of the previous layer
    m3g::PeerIO wq;
    const m3g::PeerIO* pq = nullptr;
    if (pp_ffn && l > 0) {
      wait_on(wq, 2 * (l - 1) + 1);
      pq = &wq;
    }
    auto gq = [&](const Gemv& g, float* y) {
      return m3g::gemv_fused(d->device, g.dtype, g.w, g.len, d->hidden, nullptr, g_attn, nullptr, m3g::kXRmsNorm, y,
                             g.in, g.out, d->st, true, nullptr, false, 0, pq);
    };
    if (d->qkv[l].w) {
      if (int rc = gq(d->qkv[l], d->qkvb)) return rc;
    } else {
      if (int rc = gq(part(T[kQ]), d->qkvb)) return rc;
      if (int rc = gq(part(T[kK]), d->qkvb + h)) return rc;
      if (int rc = gq(part(T[kV]), d->qkvb + h + d->kvd)) return rc;
    }
    m3g::AttnArgs a{};
    a.qkv = d->qkvb;
    a.kc = d->kc + static_cast<size_t>(l) * mp * d->kvd;
    a.vc = d->vc + static_cast<size_t>(l) * mp * d->kvd;
    a.rope = d->rope;
    a.pos = d->dpos;
    a.out = d->att;
    a.status = d->status;
    a.groups = static_cast<int>(d->cfg.n_heads / d->cfg.n_kv_heads);
    a.kvd = d->kvd;
    a.qd = h;
    a.max_pos = mp;
    a.scale = 1.0f / sqrtf(static_cast<float>(d->hd));
    const dim3 sgrid(static_cast<unsigned>(d->cfg.n_heads * m3g::kAttnSplit));
    const dim3 sblock(m3g::kAttnSplitThreads);
    if (d->hd == 64) {
      DEC_CUDA(m3g::launch_pdl_cluster(m3g::k_attention_split<64>, sgrid, sblock, split_smem, d->st, m3g::kAttnSplit,
                                       a));
    } else {
      DEC_CUDA(m3g::launch_pdl_cluster(m3g::k_attention_split<128>, sgrid, sblock, split_smem, d->st,
                                       m3g::kAttnSplit, a));
    }
    if (int rc = gemv(d, part(T[kO]), d->att, nullptr, nullptr, d->hidden, m3g::kXPlain, d->hidden)) return rc;
    if (pp_ffn) {  // this rank's rows, stored into every rank's buffers by the GEMV epilogues
      float* hslot = d->gub + static_cast<size_t>(d->rank) * d->Fr;
      const m3g::PeerIO gio = exchange(2 * l, d->off_gub, static_cast<size_t>(d->rank) * d->Fr, true);
      const Gemv& gu = d->gu[l];
      if (int rc = m3g::gemv_fused(d->device, gu.dtype, gu.w, gu.len, d->hidden, nullptr, g_ffn, nullptr,
                                   m3g::kXRmsNorm, hslot, gu.in, gu.out, d->st, true, nullptr, true, 0, &gio))
        return rc;
      float* yslot = d->hidden + static_cast<size_t>(d->rank) * d->hr;
      m3g::PeerIO dio = exchange(2 * l + 1, d->off_hidden, static_cast<size_t>(d->rank) * d->hr, true);
      wait_on(dio, 2 * l);
      const Tensor& Dn = T[kDown];
      if (int rc = m3g::gemv_fused(d->device, Dn.dtype, Dn.d, Dn.len, d->gub, nullptr, nullptr, yslot, m3g::kXPlain,
                                   yslot, Dn.in, Dn.out, d->st, true, nullptr, false, 0, &dio))
        return rc;
    } else if (d->shard_ffn) {  // this rank's rows, then NCCL all-gathers of silu(g) * u and of hidden
      float* hslot = d->gub + static_cast<size_t>(d->rank) * d->Fr;
      if (int rc = gemv(d, d->gu[l], d->hidden, nullptr, g_ffn, nullptr, m3g::kXRmsNorm, hslot, nullptr, true))
        return rc;
      if (int rc = m3g::nccl_settle(d->comm, ncclAllGather(hslot, d->gub, d->Fr, ncclFloat, d->comm, d->st),
                                    "ncclAllGather(ffn)", d->timeout_s))
        return rc;
      float* yslot = d->hidden + static_cast<size_t>(d->rank) * d->hr;
      if (int rc = gemv(d, part(T[kDown]), d->gub, nullptr, nullptr, yslot, m3g::kXPlain, yslot)) return rc;
      if (int rc = m3g::nccl_settle(d->comm, ncclAllGather(yslot, d->hidden, d->hr, ncclFloat, d->comm, d->st),
                                    "ncclAllGather(hidden)", d->timeout_s))
        return rc;
    } else if (d->gu[l].w) {  // interleaved gate|up: the epilogue writes silu(g) * u
      if (int rc = gemv(d, d->gu[l], d->hidden, nullptr, g_ffn, nullptr, m3g::kXRmsNorm, d->gub, nullptr, true))
        return rc;
      if (int rc = gemv(d, part(T[kDown]), d->gub, nullptr, nullptr, d->hidden, m3g::kXPlain, d->hidden)) return rc;
    } else {  // separate launches; the down GEMV applies SwiGLU to its input
      if (int rc = gemv(d, part(T[kGate]), d->hidden, nullptr, g_ffn, nullptr, m3g::kXRmsNorm, d->gub)) return rc;
      if (int rc = gemv(d, part(T[kUp]), d->hidden, nullptr, g_ffn, nullptr, m3g::kXRmsNorm, d->gub + F)) return rc;
      if (int rc = gemv(d, part(T[kDown]), d->gub, d->gub + F, nullptr, d->hidden, m3g::kXSiluMul, d->hidden))
        return rc;
    }
  }
  const float* g_out = reinterpret_cast<const float*>(d->t[kSlotOutNorm].d);
  const Tensor& H = d->t[kSlotOut];
  m3g::PeerIO hio;
  const m3g::PeerIO* ph = nullptr;
  if (pp) {  // the ranks' greedy keys merge into every rank's key
    hio = exchange(2 * L, 0, 0, false);
    for (int p = 0; p < d->world; ++p)
      if (p != d->rank) hio.peer_key[p] = peer_at<unsigned long long>(d, p, d->off_key);
    hio.key_by_step = 1;
    // with the FFN split the head's input holds every rank's rows of the last
    // layer; with only the head split every rank computed all of it itself
    if (pp_ffn) wait_on(hio, 2 * (L - 1) + 1);
    ph = &hio;
  }
  if (H.out > 0 && (head || d->world > 1)) {  // the last rank of a small vocabulary may hold no rows (NCCL path only)
    if (int rc = m3g::gemv_fused(d->device, H.dtype, H.d, H.len, d->hidden, nullptr, g_out, nullptr, m3g::kXRmsNorm,
                                 d->logits + H.row0, H.in, H.out, d->st, true, d->key, false, H.row0, ph))
      return rc;
  }
  if (d->world > 1 && !pp) {  // the greedy pick over all ranks' rows
    if (int rc = m3g::nccl_settle(d->comm, ncclAllReduce(d->key, d->key, 1, ncclUint64, ncclMax, d->comm, d->st),
                                  "ncclAllReduce(greedy key)", d->timeout_s))
      return rc;
  }
  const unsigned int* pick_wait = pp ? d->cnt + 2 * L : nullptr;
  DEC_CUDA(m3g::launch_pdl(m3g::k_pick_step, dim3(1), dim3(32), 0, d->st, d->key, d->dpos, d->tokens,
                           static_cast<const int*>(d->nfixed), mp, d->last, d->dstep, pick_wait,
                           static_cast<unsigned int>(d->world), pp ? 1 : 0, d->status, m3g::peer_wait_ns()));
  return M3G_OK;
}

void drop_graph(m3g_decoder* d) {
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  if (d->exec_nohead) cudaGraphExecDestroy(d->exec_nohead);
  if (d->graph_nohead) cudaGraphDestroy(d->graph_nohead);
  d->exec = nullptr;
  d->graph = nullptr;
  d->exec_nohead = nullptr;
  d->graph_nohead = nullptr;
}

// Run `n` steps.  The first step of a decoder runs eagerly (it also sets up
// every kernel's shared-memory limit); later ones replay the captured graph.
// prompt: the steps feed prompt tokens, and only the last one's logits are
// wanted.
int run_steps(m3g_decoder* d, uint64_t n, bool prompt = false) {
  if (int rc = prepare(d)) return rc;
  if (d->pos + n > d->cfg.max_pos)
    return host_fail(M3G_EINVAL, "%llu steps from position %d overflow the KV cache of %llu positions",
                     static_cast<unsigned long long>(n), d->pos, static_cast<unsigned long long>(d->cfg.max_pos));
  for (uint64_t i = 0; i < n; ++i) {
    const bool head = !(prompt && d->world == 1 && d->steps > 0 && i + 1 < n);
    cudaGraph_t& graph = head ? d->graph : d->graph_nohead;
    cudaGraphExec_t& exec = head ? d->exec : d->exec_nohead;
    if (d->use_graph && d->steps > 0 && !exec) {
      DEC_CUDA(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal));
      const int rc = enqueue_step(d, head);
      cudaGraph_t g = nullptr;
      const cudaError_t e = cudaStreamEndCapture(d->st, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (e != cudaSuccess) return host_fail(M3G_ECUDA, "decode step capture: %s", cudaGetErrorString(e));
      graph = g;
      DEC_CUDA(cudaGraphInstantiate(&exec, graph, 0));
    }
    if (exec) {
      DEC_CUDA(cudaGraphLaunch(exec, d->st));
    } else if (int rc = enqueue_step(d, head)) {
      return rc;
    }
    ++d->steps;
    ++d->pos;
  }
  d->pending = true;
  return M3G_OK;
}

int check_status(m3g_decoder* d) {
  DEC_CUDA(cudaStreamSynchronize(d->st));
  uint32_t s = 0;
  DEC_CUDA(cudaMemcpy(&s, d->status, sizeof s, cudaMemcpyDeviceToHost));
  if (s & (m3g::kStatusBadPos | m3g::kStatusBadToken | m3g::kStatusCopyTimeout)) {
    cudaMemset(d->status, 0, sizeof s);
    if (s & m3g::kStatusCopyTimeout) return host_fail(M3G_ETIMEOUT, "a staged weight copy did not complete in time");
    return host_fail(M3G_EINVAL, "decode step saw %s", (s & m3g::kStatusBadPos) ? "a position outside the KV cache"
                                                                             : "a token outside the vocabulary");
  }
  return M3G_OK;
}

// Peer stores need every rank to map every other rank's exchange region
// (CUDA IPC over NVLink).  The ranks swap handles with one all-gather and
// agree (MIN all-reduce) on whether all mappings opened; otherwise every rank
// keeps the NCCL all-gathers.
int setup_peers(m3g_decoder* d) {
  d->p2p = false;
  d->peer_base[d->rank] = d->xregion;
  // With the FFN split, peer stores carry the rows and keep the ranks in step
  // through the per-layer exchanges.  With only the head split, the ranks
  // merge their greedy keys by peer atomics and may drift one step apart, so
  // the key has one slot per step parity (a rank one step ahead can only have
  // reached the next step's head: its pick waited for this rank's head).
  if (d->world < 2 || d->world > m3g::kMaxPeers || !m3g::decode_p2p_enabled()) return M3G_OK;
  if (static_cast<long long>(d->cfg.vocab) - static_cast<long long>(d->world - 1) * d->Vr < 1) return M3G_OK;
  constexpr int kRec = 72;  // 64-byte handle + ok flag
  uint8_t rec[kRec] = {};
  cudaIpcMemHandle_t mine;
  int ok = cudaIpcGetMemHandle(&mine, d->xregion) == cudaSuccess ? 1 : 0;
  memcpy(rec, &mine, sizeof mine);
  memcpy(rec + 64, &ok, sizeof ok);
  uint8_t* dev = nullptr;
  DEC_CUDA(cudaMalloc(&dev, static_cast<size_t>(kRec) * d->world + 16));
  std::vector<uint8_t> all(static_cast<size_t>(kRec) * d->world);
  int rc = M3G_OK;
  cudaError_t e = cudaMemcpy(dev + kRec * d->rank, rec, kRec, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = m3g::nccl_settle(d->comm, ncclAllGather(dev + kRec * d->rank, dev, kRec, ncclUint8, d->comm, d->st),
                          "ncclAllGather(ipc handles)", d->timeout_s);
    if (!rc) e = cudaStreamSynchronize(d->st);
    if (!rc && e == cudaSuccess) e = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost);
  }
  if (rc || e != cudaSuccess) {
    cudaFree(dev);
    return rc ? rc : host_fail(M3G_ECUDA, "peer handle exchange: %s", cudaGetErrorString(e));
  }
  int mine_ok = 1;
  for (int p = 0; p < d->world; ++p) {
    int okp = 0;
    memcpy(&okp, all.data() + kRec * p + 64, sizeof okp);
    if (!okp) mine_ok = 0;
  }
  for (int p = 0; p < d->world && mine_ok; ++p) {
    if (p == d->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, all.data() + kRec * p, sizeof h);
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      mine_ok = 0;
      break;
    }
    d->peer_base[p] = static_cast<uint8_t*>(ptr);
  }
  // agree: peer stores only if every rank mapped every peer
  int* flag = reinterpret_cast<int*>(dev);
  e = cudaMemcpy(flag, &mine_ok, sizeof mine_ok, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = m3g::nccl_settle(d->comm, ncclAllReduce(flag, flag, 1, ncclInt, ncclMin, d->comm, d->st),
                          "ncclAllReduce(peer agreement)", d->timeout_s);
    if (!rc) e = cudaStreamSynchronize(d->st);
  }
  int all_ok = 0;
  if (!rc && e == cudaSuccess) e = cudaMemcpy(&all_ok, flag, sizeof all_ok, cudaMemcpyDeviceToHost);
  cudaFree(dev);
  if (rc) return rc;
  if (e != cudaSuccess) return host_fail(M3G_ECUDA, "peer agreement: %s", cudaGetErrorString(e));
  if (!all_ok) {
    for (int p = 0; p < d->world; ++p)
      if (p != d->rank && d->peer_base[p]) cudaIpcCloseMemHandle(d->peer_base[p]);
    for (int p = 0; p < d->world; ++p) d->peer_base[p] = p == d->rank ? d->xregion : nullptr;
    return M3G_OK;
  }
  d->p2p = true;
  return M3G_OK;
}

// Sharded: every rank assembles the full logits of the last step (only when
// the caller asks for them; the greedy loop needs only the merged key).
int gather_logits(m3g_decoder* d, bool want) {
  if (d->world == 1 || !want) return M3G_OK;
  float* slot = d->logits + static_cast<size_t>(d->rank) * d->Vr;
  return m3g::nccl_settle(d->comm, ncclAllGather(slot, d->logits, d->Vr, ncclFloat, d->comm, d->st),
                          "ncclAllGather(logits)", d->timeout_s);
}

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DevGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

M3G_API int m3g_decoder_create(int device, const m3g_decoder_config* cfg, m3g_decoder** out) {
  return m3g_decoder_create_sharded(device, cfg, 0, 1, nullptr, 0.0, out);
}

M3G_API int m3g_decoder_create_sharded(int device, const m3g_decoder_config* cfg, int rank, int world,
                                       const uint8_t* nccl_id128, double timeout_s, m3g_decoder** out) {
  if (!cfg || !out) return host_fail(M3G_EINVAL, "null argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return host_fail(M3G_EINVAL, "rank %d of %d", rank, world);
  if (world > 1 && !nccl_id128) return host_fail(M3G_EINVAL, "sharded decoder needs an NCCL unique id");
  const bool shard_ffn = world > 1 && m3g::decode_shard_ffn_enabled();
  if (world > 1 && cfg->vocab < static_cast<uint64_t>(world))
    return host_fail(M3G_EINVAL, "sharding needs vocab >= world");
  if (shard_ffn && (cfg->ffn % (8ull * world) || cfg->hidden % world))
    return host_fail(M3G_EINVAL, "FFN sharding needs ffn %% (8 * world) == 0 and hidden %% world == 0");
  const m3g_decoder_config& c = *cfg;
  if (!c.n_layers || !c.hidden || !c.ffn || !c.n_heads || !c.n_kv_heads || !c.vocab || !c.max_pos)
    return host_fail(M3G_EINVAL, "zero dimension in the decoder shape");
  if (c.hidden % c.n_heads || c.n_heads % c.n_kv_heads) return host_fail(M3G_EINVAL, "heads do not divide");
  const uint64_t hd = c.hidden / c.n_heads;
  if (hd != 64 && hd != 128) return host_fail(M3G_EINVAL, "head_dim %llu (64 and 128 are supported)",
                                             static_cast<unsigned long long>(hd));
  if (c.hidden % 256 || c.ffn % 256) return host_fail(M3G_EINVAL, "hidden and ffn must be multiples of 256");
  if (c.vocab > (1u << 30) || c.max_pos > (1u << 20) || c.hidden > (1u << 16) || c.ffn > (1u << 20) ||
      c.n_layers > 4096)
    return host_fail(M3G_EINVAL, "decoder shape too large");
  if (c.max_pos * sizeof(float) + 4096 > 200 * 1024)
    return host_fail(M3G_EINVAL, "max_pos %llu exceeds the attention kernel's shared memory",
                     static_cast<unsigned long long>(c.max_pos));
  DevGuard g(device);
  auto* d = new m3g_decoder();
  d->device = device;
  d->cfg = c;
  d->rank = rank;
  d->world = world;
  d->timeout_s = timeout_s > 0 ? timeout_s : 60.0;
  d->shard_ffn = shard_ffn;
  d->Fr = static_cast<int>(shard_ffn ? c.ffn / world : c.ffn);
  d->hr = static_cast<int>(shard_ffn ? c.hidden / world : c.hidden);
  d->Vr = static_cast<int>((c.vocab + world - 1) / world);
  d->hd = static_cast<int>(hd);
  d->kvd = static_cast<int>(c.n_kv_heads * hd);
  d->t.resize(kSlotLayer0 + kPerLayer * c.n_layers);
  for (size_t s = 0; s < d->t.size(); ++s) {
    bool norm = false;
    slot_shape(d, static_cast<int>(s), &d->t[s].in, &d->t[s].out, &norm);
  }
  auto fail = [&](int rc) {
    m3g_decoder_destroy(d);
    return rc;
  };
  const size_t h = c.hidden, F = c.ffn, mp = c.max_pos;
  if (int rc = m3g::status_word(device, &d->status)) return fail(rc);
  cudaError_t e = cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking);
  auto up256 = [](size_t n) { return (n + 255) / 256 * 256; };
  d->off_hidden = 0;
  d->off_gub = up256(4 * h);
  d->off_key = d->off_gub + up256(4 * 2 * F);
  d->off_cnt = d->off_key + 256;
  d->xregion_bytes = d->off_cnt + up256(4 * (2 * (2 * c.n_layers + 1) + 1));
  if (e == cudaSuccess) e = cudaMalloc(&d->xregion, d->xregion_bytes);
  if (e == cudaSuccess) e = cudaMemset(d->xregion, 0, d->xregion_bytes);
  if (e == cudaSuccess) {
    d->hidden = reinterpret_cast<float*>(d->xregion + d->off_hidden);
    d->gub = reinterpret_cast<float*>(d->xregion + d->off_gub);
    d->key = reinterpret_cast<unsigned long long*>(d->xregion + d->off_key);
    d->cnt = reinterpret_cast<unsigned int*>(d->xregion + d->off_cnt);
    d->done = d->cnt + (2 * c.n_layers + 1);
    d->dstep = reinterpret_cast<int*>(d->done + (2 * c.n_layers + 1));
  }
  if (e == cudaSuccess) e = cudaMalloc(&d->qkvb, 4 * (h + 2 * d->kvd));
  if (e == cudaSuccess) e = cudaMalloc(&d->att, 4 * h);
  if (e == cudaSuccess) e = cudaMalloc(&d->logits, 4 * static_cast<size_t>(d->Vr) * world);
  if (e == cudaSuccess) e = cudaMalloc(&d->rope, 4 * mp * hd);
  if (e == cudaSuccess) e = cudaMalloc(&d->kc, 4 * c.n_layers * mp * d->kvd);
  if (e == cudaSuccess) e = cudaMalloc(&d->vc, 4 * c.n_layers * mp * d->kvd);
  if (e == cudaSuccess) e = cudaMalloc(&d->dpos, 4 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d->tokens, 4 * (mp + 1));
  if (e == cudaSuccess) e = cudaHostAlloc(&d->h_io, 4 * 4, cudaHostAllocDefault);
  if (e != cudaSuccess) {
    const int rc = host_fail(e == cudaErrorMemoryAllocation ? M3G_ENOMEM : M3G_ECUDA, "decoder setup: %s",
                             cudaGetErrorString(e));
    return fail(rc);
  }
  d->nfixed = d->dpos + 1;
  d->last = d->dpos + 2;
  // RoPE table: (cos, sin) of pos * theta^(-2i / head_dim) in f32, the
  // arithmetic of src/inference.rs:1000-1007, computed once on the host.
  std::vector<float> rope(mp * hd);
  for (size_t p = 0; p < mp; ++p)
    for (size_t i = 0; i < hd / 2; ++i) {
      const float f = static_cast<float>(p) * powf(c.rope_theta, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
      rope[p * hd + 2 * i] = cosf(f);
      rope[p * hd + 2 * i + 1] = sinf(f);
    }
  e = cudaMemcpy(d->rope, rope.data(), 4 * mp * hd, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(d->dpos, 0, 4 * 4);
  if (e == cudaSuccess) e = cudaMemset(d->tokens, 0, 4 * (mp + 1));
  if (e == cudaSuccess) {
    const int split_smem = static_cast<int>(attn_split_smem(d));
    e = hd == 64 ? cudaFuncSetAttribute(m3g::k_attention_split<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        split_smem)
                 : cudaFuncSetAttribute(m3g::k_attention_split<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        split_smem);
  }
  if (e != cudaSuccess) return fail(host_fail(M3G_ECUDA, "decoder setup: %s", cudaGetErrorString(e)));
  if (world > 1) {
    if (int rc = m3g::nccl_comm_create(rank, world, nccl_id128, d->timeout_s, &d->comm)) return fail(rc);
    if (int rc = setup_peers(d)) return fail(rc);
  }
  *out = d;
  return M3G_OK;
}

M3G_API int m3g_decoder_upload(m3g_decoder* d, uint32_t slot, uint32_t dtype, const void* raw, uint64_t raw_len) {
  if (!d || !raw) return host_fail(M3G_EINVAL, "null argument");
  if (slot >= d->t.size()) return host_fail(M3G_EINVAL, "slot %u out of range", slot);
  int in = 0, out = 0;
  bool norm = false;
  slot_shape(d, static_cast<int>(slot), &in, &out, &norm);
  uint64_t need = 0;
  if (norm) {
    if (dtype != 0) return host_fail(M3G_EINVAL, "norm weights of slot %u must be f32 (dtype 0)", slot);
    need = 4ull * in;
  } else if (slot == kSlotEmbd && (dtype == 0 || dtype == 1)) {
    need = (dtype == 0 ? 4ull : 2ull) * in * out;
  } else {
    if (!gemv_dtype(dtype)) return host_fail(M3G_EINVAL, "slot %u: dtype %u has no fused GEMV", slot, dtype);
    if (m3g_quant_raw_len(dtype, static_cast<uint64_t>(in) * out, &need))
      return host_fail(M3G_EINVAL, "slot %u: %d x %d is not whole blocks of dtype %u", slot, out, in, dtype);
  }
  if (raw_len < need)
    return host_fail(M3G_EINVAL, "slot %u: %llu bytes, needs %llu", slot, static_cast<unsigned long long>(raw_len),
                     static_cast<unsigned long long>(need));
  int row0 = 0, rows = out;
  shard_rows(d, static_cast<int>(slot), out, &row0, &rows);
  const uint64_t rb = norm ? need : need / static_cast<uint64_t>(out);
  if (!norm && rb * static_cast<uint64_t>(out) != need && rows != out)
    return host_fail(M3G_EINVAL, "slot %u: rows of dtype %u straddle blocks and cannot be sharded", slot, dtype);
  const uint64_t off = norm ? 0 : rb * static_cast<uint64_t>(row0);
  const uint64_t len = norm ? need : (rows == out ? need : rb * static_cast<uint64_t>(rows));
  DevGuard g(d->device);
  if (cudaStreamSynchronize(d->st) != cudaSuccess) return host_fail(M3G_ECUDA, "decoder stream failed");
  drop_graph(d);
  for (uint8_t* f : d->fused) cudaFree(f);
  d->fused.clear();
  d->prepared = false;
  Tensor& t = d->t[slot];
  if (t.d) cudaFree(t.d);
  t.d = nullptr;
  t.set = false;
  DEC_CUDA(cudaMalloc(&t.d, len ? len : 16));
  if (len) DEC_CUDA(cudaMemcpy(t.d, static_cast<const uint8_t*>(raw) + off, len, cudaMemcpyHostToDevice));
  t.len = len;
  t.dtype = dtype;
  t.row0 = row0;
  if (!norm) t.out = rows;
  t.set = true;
  return M3G_OK;
}

M3G_API int m3g_decoder_forward(m3g_decoder* d, uint32_t token, float* logits) {
  if (!d) return host_fail(M3G_EINVAL, "null decoder");
  if (token >= d->cfg.vocab) return host_fail(M3G_EINVAL, "token %u outside the vocabulary", token);
  if (d->pos >= static_cast<int>(d->cfg.max_pos)) return host_fail(M3G_EINVAL, "KV cache full");
  DevGuard g(d->device);
  DEC_CUDA(cudaStreamSynchronize(d->st));
  d->h_io[0] = static_cast<int>(token);
  d->h_io[1] = 0;
  DEC_CUDA(cudaMemcpyAsync(d->tokens + d->pos, &d->h_io[0], 4, cudaMemcpyHostToDevice, d->st));
  DEC_CUDA(cudaMemcpyAsync(d->nfixed, &d->h_io[1], 4, cudaMemcpyHostToDevice, d->st));
  if (int rc = run_steps(d, 1)) return rc;
  if (int rc = gather_logits(d, logits != nullptr)) return rc;
  if (logits) DEC_CUDA(cudaMemcpyAsync(logits, d->logits, 4 * d->cfg.vocab, cudaMemcpyDeviceToHost, d->st));
  return check_status(d);
}

M3G_API int m3g_decoder_prefill(m3g_decoder* d, const uint32_t* tokens, uint64_t n, float* logits) {
  if (!d || (!tokens && n)) return host_fail(M3G_EINVAL, "null argument");
  if (n == 0) return M3G_OK;
  if (d->pos + n > d->cfg.max_pos) return host_fail(M3G_EINVAL, "prompt overflows the KV cache");
  for (uint64_t i = 0; i < n; ++i)
    if (tokens[i] >= d->cfg.vocab) return host_fail(M3G_EINVAL, "token %u outside the vocabulary", tokens[i]);
  DevGuard g(d->device);
  DEC_CUDA(cudaStreamSynchronize(d->st));
  DEC_CUDA(cudaMemcpy(d->tokens + d->pos, tokens, 4 * n, cudaMemcpyHostToDevice));
  const int nfixed = d->pos + static_cast<int>(n);
  DEC_CUDA(cudaMemcpy(d->nfixed, &nfixed, 4, cudaMemcpyHostToDevice));
  if (int rc = run_steps(d, n, true)) return rc;
  if (int rc = gather_logits(d, logits != nullptr)) return rc;
  if (logits) DEC_CUDA(cudaMemcpyAsync(logits, d->logits, 4 * d->cfg.vocab, cudaMemcpyDeviceToHost, d->st));
  return check_status(d);
}

M3G_API int m3g_decoder_generate(m3g_decoder* d, uint64_t n_gen, uint32_t* out_tokens) {
  if (!d || (!out_tokens && n_gen)) return host_fail(M3G_EINVAL, "null argument");
  if (n_gen == 0) return M3G_OK;
  if (!d->pending) return host_fail(M3G_EINVAL, "generate needs a prefilled prompt (no step has run)");
  if (d->pos + n_gen - 1 > d->cfg.max_pos) return host_fail(M3G_EINVAL, "generation overflows the KV cache");
  DevGuard g(d->device);
  const int first = d->pos;
  if (int rc = run_steps(d, n_gen - 1)) return rc;
  DEC_CUDA(cudaMemcpyAsync(out_tokens, d->tokens + first, 4 * n_gen, cudaMemcpyDeviceToHost, d->st));
  return check_status(d);
}

M3G_API int m3g_decoder_run_async(m3g_decoder* d, uint64_t n_steps) {
  if (!d) return host_fail(M3G_EINVAL, "null decoder");
  if (n_steps && !d->pending) return host_fail(M3G_EINVAL, "run_async needs a prefilled prompt");
  DevGuard g(d->device);
  return run_steps(d, n_steps);
}

M3G_API int m3g_decoder_sync(m3g_decoder* d) {
  if (!d) return host_fail(M3G_EINVAL, "null decoder");
  DevGuard g(d->device);
  return check_status(d);
}

M3G_API int m3g_decoder_tokens(const m3g_decoder* d, uint64_t first, uint64_t n, uint32_t* out) {
  if (!d || (!out && n)) return host_fail(M3G_EINVAL, "null argument");
  if (first + n > d->cfg.max_pos + 1) return host_fail(M3G_EINVAL, "token range outside the stream");
  DevGuard g(d->device);
  DEC_CUDA(cudaStreamSynchronize(d->st));
  if (n) DEC_CUDA(cudaMemcpy(out, d->tokens + first, 4 * n, cudaMemcpyDeviceToHost));
  return M3G_OK;
}

M3G_API uint64_t m3g_decoder_pos(const m3g_decoder* d) { return d ? static_cast<uint64_t>(d->pos) : 0; }

M3G_API int m3g_decoder_truncate(m3g_decoder* d, uint64_t n) {
  if (!d) return host_fail(M3G_EINVAL, "null decoder");
  if (n > static_cast<uint64_t>(d->pos)) return host_fail(M3G_EINVAL, "cannot truncate forward");
  DevGuard g(d->device);
  DEC_CUDA(cudaStreamSynchronize(d->st));
  const int p = static_cast<int>(n);
  DEC_CUDA(cudaMemcpy(d->dpos, &p, 4, cudaMemcpyHostToDevice));
  // Every step's pick leaves its key slot zero.  With peer merges a rank that
  // truncated first may already have merged its next step's key here, so the
  // slots are left alone then.
  if (!d->p2p) DEC_CUDA(cudaMemset(d->key, 0, 16));
  d->pos = p;
  d->pending = false;
  return M3G_OK;
}

M3G_API const float* m3g_decoder_logits_dev(const m3g_decoder* d) { return d ? d->logits : nullptr; }

M3G_API int m3g_decoder_exchange(const m3g_decoder* d) {
  if (!d) return -1;
  return d->world == 1 ? 0 : (!d->shard_ffn ? (d->p2p ? 4 : 3) : (d->p2p ? 2 : 1));
}

M3G_API void* m3g_decoder_stream(const m3g_decoder* d) { return d ? static_cast<void*>(d->st) : nullptr; }

M3G_API int m3g_decoder_set_graph(m3g_decoder* d, int use_graph) {
  if (!d) return host_fail(M3G_EINVAL, "null decoder");
  DevGuard g(d->device);
  DEC_CUDA(cudaStreamSynchronize(d->st));
  drop_graph(d);
  d->use_graph = use_graph != 0;
  return M3G_OK;
}

M3G_API void m3g_decoder_destroy(m3g_decoder* d) {
  if (!d) return;
  DevGuard g(d->device);
  if (d->st) cudaStreamSynchronize(d->st);
  drop_graph(d);  // the graph holds NCCL work: released before the communicator
  if (d->comm && d->p2p) {
    // no rank may still store into another's region when it is unmapped / freed
    int* one = nullptr;
    if (cudaMalloc(&one, 16) == cudaSuccess) {
      m3g::nccl_settle(d->comm, ncclAllReduce(one, one, 1, ncclInt, ncclSum, d->comm, d->st), "ncclAllReduce(exit)",
                       d->timeout_s);
      cudaStreamSynchronize(d->st);
      cudaFree(one);
    }
    for (int p = 0; p < d->world; ++p)
      if (p != d->rank && d->peer_base[p]) cudaIpcCloseMemHandle(d->peer_base[p]);
  }
  if (d->comm) m3g::nccl_comm_close(d->comm, d->timeout_s);
  d->comm = nullptr;
  for (Tensor& t : d->t)
    if (t.d) cudaFree(t.d);
  for (uint8_t* f : d->fused) cudaFree(f);
  for (void* p : {static_cast<void*>(d->xregion), static_cast<void*>(d->qkvb), static_cast<void*>(d->att),
                  static_cast<void*>(d->logits), static_cast<void*>(d->rope),
                  static_cast<void*>(d->kc), static_cast<void*>(d->vc), static_cast<void*>(d->dpos),
                  static_cast<void*>(d->tokens)})
    if (p) cudaFree(p);
  if (d->h_io) cudaFreeHost(d->h_io);
  if (d->st) cudaStreamDestroy(d->st);
  delete d;
}

// Fused GEMV with the decode step's input transforms and residual epilogue.
M3G_API int m3g_matvec_fused_dev(const float* x, const float* x2, const float* gamma, const float* res, int xmode,
                                 int swiglu, const uint8_t* raw, uint64_t raw_len, uint32_t dtype, uint64_t in_dim,
                                 uint64_t out_dim, float* y, void* stream) {
  if (!x || !raw || !y) return host_fail(M3G_EINVAL, "null argument");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return host_fail(M3G_ECUDA, "no CUDA device");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  return m3g::gemv_fused(dev, dtype, raw, raw_len, x, x2, gamma, res, xmode, y, static_cast<long long>(in_dim),
                         static_cast<long long>(out_dim), st, false, nullptr, swiglu != 0);
}


// The fused GEMV of m3g_matvec_fused_dev whose input is gated on a device
// counter: the kernel's weight stream starts at once, and its x preparation
// waits (bounded) until *ready_cnt >= ready_target before reading x.
M3G_API int m3g_matvec_fused_wait_dev(const float* x, const float* x2, const float* gamma, const float* res,
                                      int xmode, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                                      uint64_t in_dim, uint64_t out_dim, float* y, const uint32_t* ready_cnt,
                                      uint32_t ready_target, void* stream) {
  if (!x || !raw || !y || !ready_cnt) return host_fail(M3G_EINVAL, "null argument");
  if (reinterpret_cast<uintptr_t>(ready_cnt) % 4) return host_fail(M3G_EINVAL, "ready counter not 4-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return host_fail(M3G_ECUDA, "no CUDA device");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
  m3g::PeerIO io;
  io.wait_cnt = reinterpret_cast<const unsigned int*>(ready_cnt);
  io.wait_mul = ready_target;
  return m3g::gemv_fused(dev, dtype, raw, raw_len, x, x2, gamma, res, xmode, y, static_cast<long long>(in_dim),
                         static_cast<long long>(out_dim), st, false, nullptr, false, 0, &io);
}

}  // extern "C"
