// m3g_internal.h -- host/device interface between the C ABI and the kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace m3g {

// Status bits the kernels set in the per-device error word.
enum : uint32_t {
  kStatusCopyTimeout = 1u,  // a staged-copy wait gave up
  kStatusBadPos = 2u,       // a decode step found its position outside the KV cache
  kStatusBadToken = 4u,     // a decode step read a token id outside the vocabulary
  kStatusPeerTimeout = 8u,  // a wait for other GPUs' rows gave up
};

constexpr int kMaxPeers = 8;  // ranks one decoder exchanges rows with (itself included)

// Arguments of the staged streaming GEMV (k_gemv_stream).
// Block = one producer warp + TS*RPI consumer threads.  Shared memory:
//   [0, NS*stage_stride)          weight stages (TMA bulk destinations)
//   [off_x, off_x + 4*in_dim)     x staged by the consumers (when stage_x)
//   [off_red, ...)                per-stage row partials [NS][R][TS/32]
//   [off_bar, ...)                full[NS], empty[NS] mbarriers, abort flag
struct StreamArgs {
  const uint8_t* w;   // weight bytes of rows [0, rows), row-major, RB bytes per row, 16-byte aligned
  const float* x;     // x[in_dim]
  float* y;           // y[rows]
  uint32_t* status;   // per-device error word
  int in_dim;         // K
  int rows;           // output rows handled by this launch
  int RB;             // bytes per row (multiple of 16)
  int U;              // units per row = in_dim / unit elements
  int TS;             // consumer threads per row slot (multiple of 32, >= ceil(U / UPT))
  int RPI;            // row slots per CTA
  int R;              // rows per stage (multiple of RPI)
  int NS;             // pipeline stages
  int stage_stride;   // bytes between stage buffers (>= R*RB + 16, multiple of 128)
  int rows_per_cta;   // contiguous rows per CTA
  int stage_x;        // 1: consumers stage x in shared memory with coalesced loads
  int off_x, off_red, off_bar;
};

// Arguments of the tensor-core GEMV (k_gemv_mma).  Block = one producer warp
// + WK*TPS consumer warps.  Stage s holds k-chunk (s % NKC) of the row group
// (s / NKC) of 16*TPS rows: each row's segment of up to KC super-blocks,
// copied CG rows at a time into groups GS bytes apart.
struct MmaArgs {
  const uint8_t* w;   // weight bytes, RB per row, 16-byte aligned
  const float* x;     // x[in_dim], 16-byte aligned
  float* y;           // y[rows]
  uint32_t* status;   // per-device error word
  int rows;
  int RB;             // bytes per row
  int NSB;            // super-blocks per row (in_dim / 256)
  int KC;             // super-blocks per k-chunk
  int NKC;            // k-chunks per tile
  int CG;             // rows per bulk copy: 4 (whole rows, NKC == 1) or 1 (row segments)
  int GS;             // shared-memory stride between copy groups (32 mod 128 bytes for Q4_K, 16 otherwise)
  int SEG;            // bytes of one row's segment within a group
  int NS;             // stages
  int PRE;            // stages issued before the grid dependency resolves
  int tail_first;     // 1: a CTA's partial last row group is visited first
  int rows_per_cta;
  // Non-null (plain GEMV of a host-buffer call): every CTA adds 1 to fin_cnt[0]
  // when it is done, and the last one stores *status to status_host[0] (mapped
  // host memory), clears the count and stores the call's sequence number
  // fin_cnt[1] + 1 (kept in fin_cnt[1]) to status_host[1].
  uint32_t* status_host;
  unsigned int* fin_cnt;
  int off_xsl, off_sum32, off_sum16, off_scale, off_red, off_bar;
  // Fused input transform and epilogue (all zero for a plain GEMV):
  //   xmode 0: the GEMV input is x
  //   xmode 1: rms_norm(x) * gamma, the norm taken over all in_dim elements
  //   xmode 2: silu(x) * x2 (the SwiGLU gate times the up projection)
  //   res != nullptr: y[r] = res[r] + (W x')[r] (res may alias y)
  const float* x2;
  const float* gamma;  // nullptr: ones
  const float* res;
  int xmode;
  // Non-null: atomicMax of argmax_key(y[r], r) over the rows (the greedy
  // pick, decoded as 0xFFFFFFFF - low word; the caller zeroes it first).
  unsigned long long* argmax_key;
  // 1: stages past the first PRE are issued only after the consumers have
  // loaded x (their loads then do not wait behind the weight stream).
  int xfirst;
  // 1: the rows are gate/up pairs in blocks of 8 gate rows then their 8 up
  // rows; y[i] = silu(gate_i) * up_i (rows/2 outputs).  rows_per_cta is a
  // multiple of 16.
  int swiglu;
  // Row number the argmax key reports for local row 0 (a row shard's offset).
  long long key_row0;
  // Row exchange between the GPUs of a sharded decode (FUSED only).  The
  // epilogue also stores every output to the non-null peer_y[p] (this rank's
  // slot in rank p's buffer).  Every CTA then adds 1 to the local done_cnt;
  // the CTA that completes this step's count ((*step + 1) * gridDim.x) merges
  // the local greedy key into the non-null peer_key[p] and adds 1 to every
  // peer_cnt[p] (p < npeer, this rank included).  Before reading x, the
  // consumers wait until *wait_cnt >= (*step + 1) * wait_mul (>= wait_mul
  // when step is null), for at most peer_wait_ns; a wait that runs out sets
  // kStatusPeerTimeout and the kernel goes on with x as it is.
  float* peer_y[kMaxPeers];
  unsigned long long* peer_key[kMaxPeers];
  unsigned int* peer_cnt[kMaxPeers];
  int npeer;
  unsigned int* done_cnt;
  const int* step;
  const unsigned int* wait_cnt;
  unsigned int wait_mul;
  unsigned long long peer_wait_ns;
  // Non-null: every peer store goes ystride floats further on when *ystep is
  // odd (double-buffered exchange; *ystep is read after the grid dependency).
  const int* ystep;
  long long ystride;
  // 1: the greedy key of step *step is argmax_key[*step & 1] (and the same
  // slot of every peer_key), so that a rank one step ahead merges into the
  // other slot while this rank still reads the last one.
  int key_by_step;
};

// Peer-exchange form of a decode GEMV (all pointers device-side; see MmaArgs).
struct PeerIO {
  float* peer_y[kMaxPeers] = {};
  unsigned long long* peer_key[kMaxPeers] = {};
  unsigned int* peer_cnt[kMaxPeers] = {};
  int npeer = 0;
  unsigned int* done_cnt = nullptr;
  const int* step = nullptr;
  const unsigned int* wait_cnt = nullptr;
  unsigned int wait_mul = 0;
  int key_by_step = 0;
  const int* ystep = nullptr;
  long long ystride = 0;
};

enum XMode : int { kXPlain = 0, kXRmsNorm = 1, kXSiluMul = 2 };

// Fused GEMV on the tensor-core path only: M3G_OK, or an error code when the
// shape has no tensor-core plan (the caller treats that as unsupported).
// `decode` plans for a chain of small GEMVs: CTAs sized for half an SM (when
// the rows allow) so the next kernel's CTAs, launched early by PDL, start
// streaming their weights beside the running one.
int gemv_fused(int device, uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, const float* x2,
               const float* gamma, const float* res, int xmode, float* y, long long in_dim, long long out_dim,
               cudaStream_t st, bool decode, unsigned long long* argmax_key = nullptr, bool swiglu = false,
               long long key_row0 = 0, const PeerIO* peers = nullptr, int* grid_out = nullptr);

// GEMV with the greedy-pick epilogue, planned from the given device
// attributes, reporting into the given status word (allocates nothing).
int gemv_greedy_on(uint32_t dtype, const uint8_t* w, uint64_t raw_len, const float* x, float* y, long long in_dim,
                   long long out_dim, cudaStream_t st, int sms, int smem_per_sm, int smem_optin, uint32_t* status,
                   unsigned long long* key);

// Limit of a kernel's wait for a counter that other GPUs (or another
// producer) bump: the tuning key peer_wait_us, 2 s by default.
unsigned long long peer_wait_ns();

// Whether a shard context may exchange rows by peer stores (tuning knob).
bool shard_p2p_enabled(int world);
// Whether the tensor-core GEMV has a plan for `rows` rows of `in_dim` inputs
// of `dtype` on `device` (16-byte aligned weights and input assumed).
bool fused_plannable(int device, uint32_t dtype, long long in_dim, long long rows);

// Whether a sharded decoder may exchange rows by peer stores (tuning knob).
bool decode_p2p_enabled();
// Whether a sharded decoder splits the FFN rows too (tuning knob; else only the head).
bool decode_shard_ffn_enabled();

// The per-device status word the kernels set kStatus* bits in.
int status_word(int device, uint32_t** out);

// Batched Q4_K GEMV, up to 8 columns of X per launch (m3g_mma.cu).
constexpr int kGemm8Cols = 8;
constexpr int kGemm8RecBytes = 6432;  // prepared-x bytes per 256-element super-block
struct Gemm8Args {
  const uint8_t* w;
  const uint8_t* xq;
  float* y;
  uint32_t* status;
  int rows, RB, NSB, KC, NKC, NS, GS, rows_per_cta, cols, ldy;
  int off_stage, off_red, off_acc, off_bar;
};
cudaError_t launch_xprep8(const float* x, int cols, int in_dim, uint8_t* out, cudaStream_t st);
cudaError_t launch_gemm8_q4k(const Gemm8Args& a, int grid, size_t smem, cudaStream_t st);

// Batched Q4_K on tcgen05 (m3g_umma.cu): up to 64 columns per pass, NB = 8,
// 16, 32 or 64 accumulator columns, 128-row tiles split evenly over the CTAs.
struct UmmaArgs {
  const uint8_t* w;   // Q4_K rows, RB bytes apart
  const uint8_t* xt;  // prepared X tiles, umma_xtile(NB) bytes per super-block
  const float* sig;   // [NSB][NB] power-of-two column scales of X per super-block
  unsigned* cnt;      // per-tile super-block counters (zeroed by the X prep)
  float* part;        // [grid][2][NB][128] partial tiles
  float* y;           // y[col * ldy + row]
  uint32_t* status;
  long long RB, rows, T;  // T = tiles * NSB iterations
  int NSB, cols, ldy, tiles, NSW, NSX;
  int off_x, off_am, off_bar;
};
// pdl: the GEMM kernel may start while the X prep runs (programmatic
// dependent launch); it waits for the prep before reading X, scales, counters.
cudaError_t launch_umma_q4k(const UmmaArgs& a, const float* x, long long in_dim, int nb, int chains, int grid,
                            size_t smem, cudaStream_t st, bool pdl);
int umma_xtile(int nb);

// Batch-1 Q4_K GEMV on tcgen05, kind::i8 (m3g_tc8.cu).  One CTA per SM owns
// rows [blockIdx * rows_per_cta, ...), cut into tiles of tile_rows (<= 128)
// rows; the weight tensor maps are built at launch from w.
struct Tc8Args {
  const float* x;      // x[in_dim], 16-byte aligned
  float* y;            // y[rows]
  uint32_t* status;    // error word of the call
  uint32_t* status_host;  // non-null: the last CTA stores [*status, sequence] here (mapped host memory)
  unsigned int* fin_cnt;  // [CTAs done (cleared by the last CTA), sequence of the last call]
  long long rows;
  int NSB, tile_rows, rows_per_cta, NSW, PRE;
  int off_hdr, off_b, off_xsl, off_sum32, off_sum16, off_scale, off_bar;
};
struct Tc8Plan {
  Tc8Args a{};
  int grid = 0;
  long long RB = 0;
  size_t smem = 0;
};
bool plan_tc8(long long in_dim, long long rows, const uint8_t* w, const float* x, int sms, int smem_optin,
              Tc8Plan& p);
cudaError_t launch_tc8(const Tc8Plan& p, const uint8_t* w, cudaStream_t st, bool pdl);

int mma_sb_bytes(int fmt);
cudaError_t launch_gemv_mma(int fmt, const MmaArgs& a, int tps, int wk, int grid, size_t smem, cudaStream_t st,
                            bool pdl);

cudaError_t launch_gemv_stream(int fmt, const StreamArgs& a, int threads, int grid, size_t smem, int upt,
                               cudaStream_t st, bool pdl);
cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, long long in_dim,
                                long long nblocks, int grid, cudaStream_t st);
cudaError_t launch_dequant(int fmt, const uint8_t* w, float* out, long long n_elems, int grid, cudaStream_t st);

// x of a host-buffer GEMV from mapped pinned host memory (device alias; n % 4
// == 0, 16-byte aligned) into device memory.
cudaError_t launch_host_x_in(const float* hx_dev, float* dx, long long n, cudaStream_t st);

}  // namespace m3g
