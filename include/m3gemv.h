/*
 * m3gemv.h -- C ABI of the B200 (sm_100a) fused dequantise-and-matvec library.
 *
 * This is the drop-in boundary for the fused quantised GEMV path of m3_avm:
 * the GGUF block decoders of src/quant.rs and the fused kernels of
 * src/matvec_quant.rs, plus the per-tensor offload shape of
 * src/inference_gpu.rs.  Paths in the citations are relative to the m3_avm
 * source tree.
 *
 * Conventions shared by every entry point:
 *   - dtype uses ggml numbering: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 12 Q4_K,
 *     13 (Q5_K slot, decoded as Q4_K exactly as the reference does), 14 Q6_K.
 *   - Weights are GGUF bytes, K = in_dim fastest: y[j] = sum_i x[i] * W[i + j*in_dim].
 *     A block may straddle two output rows when in_dim is not a multiple of
 *     the block size; every entry point accepts that layout.
 *   - Return value: M3G_OK (0) on success, a negative M3G_E* code otherwise.
 *     M3G_ENONE is the reference's `None` / `false`: an unsupported dtype or a
 *     shape/length that the reference also rejects.  m3g_last_error() gives
 *     a message for the calling thread.
 *   - "_dev" entry points take device pointers and a cudaStream_t passed as
 *     void* (NULL = the legacy default stream); they enqueue work and return
 *     without synchronising.  The other entry points take host pointers and
 *     return when the result is in host memory.
 *   - Nothing here panics or aborts: failures never propagate beyond the
 *     return code (the policy of src/inference_gpu.rs:9-10).
 */
#ifndef M3GEMV_H
#define M3GEMV_H

#include <stddef.h>
#include <stdint.h>

#if defined(M3G_BUILD_LIB) && defined(__GNUC__)
#define M3G_API __attribute__((visibility("default")))
#else
#define M3G_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define M3G_OK 0
#define M3G_ENONE (-1)      /* reference returns None / false                 */
#define M3G_EINVAL (-2)     /* bad argument (null pointer, misaligned, ...)   */
#define M3G_ECUDA (-3)      /* CUDA runtime error                             */
#define M3G_ENOMEM (-4)     /* device or pinned allocation failed             */
#define M3G_ENCCL (-5)      /* NCCL error                                     */
#define M3G_ETIMEOUT (-6)   /* a bounded device-side wait gave up             */
#define M3G_ENOTFOUND (-7)  /* tensor index not uploaded                      */
#define M3G_EPANIC (-8)     /* the reference would panic (assert! on sizes)   */

#define M3G_DTYPE_F32 0u
#define M3G_DTYPE_F16 1u
#define M3G_DTYPE_Q4_0 2u
#define M3G_DTYPE_Q8_0 8u
#define M3G_DTYPE_Q4_K 12u
#define M3G_DTYPE_Q5_K_AS_Q4_K 13u
#define M3G_DTYPE_Q6_K 14u

/* Library ABI version (bumped on any signature change). */
M3G_API int m3g_abi_version(void);

/* Message for the last failing call on this thread ("" if none). */
M3G_API const char* m3g_last_error(void);

/* ---------------------------------------------------------------- host-side rules */

/* Bytes needed for n elements of a fused-kernel dtype.
 * Replaces quant_raw_len (src/matvec_quant.rs:51-83): M3G_ENONE where it
 * returns None (dtype without a fused kernel, n not a multiple of the block). */
M3G_API int m3g_quant_raw_len(uint32_t dtype, uint64_t n, uint64_t* out_len);

/* f32 -> bf16 bits, round-to-nearest-even with a quiet-NaN guard.
 * Replaces f32_to_bf16_bits (src/quant.rs:186-194). */
M3G_API uint16_t m3g_f32_to_bf16_bits(float x);

/* bf16 bits -> f32, exact.  Replaces bf16_bits_to_f32 (src/quant.rs:197-199). */
M3G_API float m3g_bf16_bits_to_f32(uint16_t b);

/* One Q4_0 / Q8_0 block from 32 floats (src_len must be 32).  M3G_ENONE where
 * the reference returns false (wrong length, non-finite input, short dst).
 * Replace quantize_q4_0 (src/quant.rs:206-234), quantize_q8_0 (:239-264). */
M3G_API int m3g_quantize_q4_0(const float* src, uint64_t src_len, uint8_t* dst, uint64_t dst_len);
M3G_API int m3g_quantize_q8_0(const float* src, uint64_t src_len, uint8_t* dst, uint64_t dst_len);

/* ---------------------------------------------------------------- decoders (GPU) */

/* Decode n elements of `dtype` to f32, bit-exact with the reference decoders.
 * Replaces dequantize (src/quant.rs:120-173) and, with a fixed dtype,
 * dequant_q4_0 (:9), dequant_q4_k (:41), dequant_q6_k (:76).
 * M3G_ENONE where dequantize returns false; M3G_EPANIC where the reference's
 * dequant_q4_0/dequant_q4_k would hit assert! (source shorter than n needs). */
M3G_API int m3g_dequantize(const uint8_t* src, uint64_t src_len, uint32_t dtype, float* dst, uint64_t n);
M3G_API int m3g_dequantize_dev(const uint8_t* src, uint64_t src_len, uint32_t dtype, float* dst, uint64_t n,
                       void* stream);

/* ---------------------------------------------------------------- fused GEMV (GPU) */

/* y[out_dim] = W x for GGUF weight bytes `raw`, host buffers.
 * Replaces matvec_quant (src/matvec_quant.rs:87-109) including its None rules
 * (x_len != in_dim, zero dims, dtype without a fused kernel, raw too short),
 * and with a fixed dtype matvec_q4k (:221), matvec_q6k (:361),
 * matvec_q4_0 (:368), matvec_q8_0 (:375).  The weights are copied to the
 * device on every call; use the offload context below to keep them resident. */
M3G_API int m3g_matvec_quant(const float* x, uint64_t x_len, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                     uint64_t in_dim, uint64_t out_dim, float* y);

/* Device-pointer form: Y[batch][out_dim] = X[batch][in_dim] W^T with
 * row-major X and Y.  `raw` must be 16-byte aligned. */
M3G_API int m3g_matvec_quant_dev(const float* x, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                         uint64_t in_dim, uint64_t out_dim, uint64_t batch, float* y, void* stream);

/* ---------------------------------------------------------------- resident offload */

/* Per-tensor resident weights, the GpuOffload shape of src/inference_gpu.rs:40-238:
 * weights are uploaded once in their native block layout; each matvec moves only
 * x and y.  A context belongs to one device and owns one stream; calls on one
 * context must not overlap (the reference calls it from one thread). */
typedef struct m3g_offload m3g_offload;

/* GpuOffload::try_new (src/inference_gpu.rs:58): M3G_ECUDA when no device. */
M3G_API int m3g_offload_create(int device, uint64_t max_in, uint64_t max_out, m3g_offload** out);

/* GpuOffload::upload (src/inference_gpu.rs:131-177): M3G_ENONE for a dtype
 * without a fused kernel, zero dims, or raw_len != quant_raw_len(dtype, in*out).
 * Re-uploading a tidx replaces it. */
M3G_API int m3g_offload_upload(m3g_offload* ctx, uint64_t tidx, uint32_t dtype, const uint8_t* raw, uint64_t raw_len,
                       uint64_t in_dim, uint64_t out_dim);

/* GpuOffload::matvec (src/inference_gpu.rs:188-237), host x and y:
 * M3G_ENOTFOUND if tidx is not resident, M3G_ENONE if dims differ from the
 * upload or exceed max_in/max_out. */
M3G_API int m3g_offload_matvec(m3g_offload* ctx, uint64_t tidx, const float* x, uint64_t in_dim, uint64_t out_dim,
                       float* y);

/* Batched form of the above: X[batch][in_dim] -> Y[batch][out_dim], host buffers. */
M3G_API int m3g_offload_matvec_batch(m3g_offload* ctx, uint64_t tidx, const float* x, uint64_t batch, uint64_t in_dim,
                             uint64_t out_dim, float* y);

/* Device-resident form for callers that keep activations on the GPU:
 * x and y are device pointers, enqueued on `stream` (NULL = the legacy
 * default stream, like every other _dev entry point). */
M3G_API int m3g_offload_matvec_dev(m3g_offload* ctx, uint64_t tidx, const float* x, uint64_t batch, float* y,
                           void* stream);

/* GpuOffload::offloaded (:179) -> 1/0, tensor_count (:183), the `calls`
 * counter (:50) and the device pointer of a resident tensor's bytes. */
M3G_API int m3g_offload_offloaded(const m3g_offload* ctx, uint64_t tidx);
M3G_API uint64_t m3g_offload_tensor_count(const m3g_offload* ctx);
M3G_API uint64_t m3g_offload_calls(const m3g_offload* ctx);
M3G_API const uint8_t* m3g_offload_tensor_ptr(const m3g_offload* ctx, uint64_t tidx);

M3G_API void m3g_offload_destroy(m3g_offload* ctx);

/* ---------------------------------------------------------------- multi-GPU row sharding */

/* One process per GPU.  Rank r keeps output rows [r*RPR, min(out, (r+1)*RPR))
 * of each tensor, RPR = ceil(out_dim / world); a matvec computes the local
 * rows and every rank receives the whole fp32 output: by one in-place NCCL
 * all-gather of the fp32 slices, or -- when the tuning key "shard_p2p" at
 * creation selects it (1; the default -1 selects it from 8 ranks up, where it
 * measured faster, 0 never), batch 1, a tensor-core plan for the shape, and
 * every rank able to map every other rank's region -- by peer stores from the
 * GEMV's epilogue into every rank's exchange region over NVLink.  No counterpart in the
 * reference (it is single-host, single-CPU); this is the sharded form of the
 * GpuOffload shape above. */
typedef struct m3g_shard m3g_shard;

/* Row partition of a tensor (pure host arithmetic): M3G_ENONE when rows do
 * not hold whole blocks (in_dim % block != 0) or the dtype has no kernel. */
M3G_API int m3g_shard_plan(uint32_t dtype, uint64_t in_dim, uint64_t out_dim, int world, int rank,
                           uint64_t* row_begin, uint64_t* rows_local, uint64_t* rows_per_rank,
                           uint64_t* byte_begin, uint64_t* byte_len);

/* 128-byte NCCL unique id, made on one rank and shared with the others. */
M3G_API int m3g_shard_unique_id(uint8_t* out128);

/* Join the communicator; M3G_ETIMEOUT (communicator aborted) when it is not
 * complete within timeout_s seconds, e.g. because a rank never joined.  With
 * world > 1 it also maps the ranks' exchange regions (collective: every rank
 * calls it with the same max_out). */
M3G_API int m3g_shard_create(int device, int rank, int world, const uint8_t* id128, uint64_t max_in,
                             uint64_t max_out, double timeout_s, m3g_shard** out);

/* Keep this rank's rows of a full GGUF tensor (raw_len == quant_raw_len). */
M3G_API int m3g_shard_upload(m3g_shard* ctx, uint64_t tidx, uint32_t dtype, const uint8_t* raw, uint64_t raw_len,
                             uint64_t in_dim, uint64_t out_dim);

/* Device x [batch][in_dim]; y holds batch*RPR*world floats.  batch == 1:
 * y[0 .. out_dim) is the full output; batch > 1: y is [rank][b][RPR]. */
M3G_API int m3g_shard_matvec_dev(m3g_shard* ctx, uint64_t tidx, const float* x, uint64_t batch, float* y,
                                 void* stream);

/* Host x [batch][in_dim] -> host y [batch][out_dim] on every rank. */
M3G_API int m3g_shard_matvec(m3g_shard* ctx, uint64_t tidx, const float* x, uint64_t batch, uint64_t in_dim,
                             uint64_t out_dim, float* y);

M3G_API int m3g_shard_info(const m3g_shard* ctx, uint64_t tidx, uint64_t* row_begin, uint64_t* rows_local,
                           uint64_t* rows_per_rank);
M3G_API uint64_t m3g_shard_calls(const m3g_shard* ctx);
/* How rows are exchanged: 0 one rank, 1 NCCL all-gather, 2 peer stores. */
M3G_API int m3g_shard_exchange(const m3g_shard* ctx);
M3G_API void m3g_shard_destroy(m3g_shard* ctx);

/* ---------------------------------------------------------------- fused GEMV forms of the decode step */

/* y = W x' (+ res) on the tensor-core GEMV, with the input transform of the
 * step that feeds it (device pointers, 16-byte aligned):
 *   xmode 0: x' = x
 *   xmode 1: x' = rms_norm_into(x, gamma) -- x / sqrt(mean(x^2) + 1e-5) * gamma,
 *            src/inference.rs:1575-1585 (gamma NULL = ones)
 *   xmode 2: x' = x * sigmoid(x) * x2 -- the SwiGLU product of
 *            src/inference.rs:1092-1097 (x = gate, x2 = up)
 *   res != NULL: y[j] = res[j] + (W x')[j], the residual adds of
 *            src/inference.rs:1083 and :1103 (res may equal y).
 *   swiglu != 0: W holds gate and up rows interleaved in blocks of 8 (8 gate
 *            rows, then the same 8 up rows; out_dim % 16 == 0) and y gets
 *            out_dim/2 values silu(gate_i) * up_i (src/inference.rs:1092-1097);
 *            not combined with res or xmode 2.
 * Needs in_dim % 256 == 0 and 16-byte rows (the tensor-core plan);
 * M3G_EINVAL otherwise.  Enqueues on `stream` (NULL = legacy default stream). */
M3G_API int m3g_matvec_fused_dev(const float* x, const float* x2, const float* gamma, const float* res, int xmode,
                                 int swiglu, const uint8_t* raw, uint64_t raw_len, uint32_t dtype, uint64_t in_dim,
                                 uint64_t out_dim, float* y, void* stream);

/* The same GEMV with its input gated on a device counter, for an x that
 * another stream, process or GPU produces and then signals by incrementing
 * *ready_cnt (device memory, 4-byte aligned).  The weight stream starts at
 * once; the x preparation waits until *ready_cnt >= ready_target (wrap-safe
 * comparison) before reading x -- the wait a sharded decode step makes for the
 * rows other GPUs store into it (src/inference.rs:1083-1103 are the steps it
 * gates).  The wait is bounded by the tuning key "peer_wait_us" (default
 * 2 s): when it runs out the kernel sets bit 8 (kStatusPeerTimeout) of the
 * device status word (m3g_device_status), computes with x as it is and
 * returns; the context stays usable.  No swiglu form.  M3G_EINVAL where
 * m3g_matvec_fused_dev gives it. */
M3G_API int m3g_matvec_fused_wait_dev(const float* x, const float* x2, const float* gamma, const float* res,
                                      int xmode, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                                      uint64_t in_dim, uint64_t out_dim, float* y, const uint32_t* ready_cnt,
                                      uint32_t ready_target, void* stream);

/* ---------------------------------------------------------------- device-resident greedy decode
 *
 * RealInference::forward_one (src/inference.rs:953-1152) for a Llama-style
 * model, every MATVEC on the fused kernels and no host round trip between
 * tokens.  The engine owns one CUDA stream, the weights (uploaded once, GGUF
 * bytes), a compact KV cache of max_pos positions and the token stream.
 *
 * Tensor slots: 0 token_embd (vocab x hidden; F32, F16 or a block dtype),
 * 1 output_norm (f32[hidden]), 2 output (vocab x hidden), then nine per
 * layer l at 3 + 9*l: attn_norm (f32), attn_q (hidden x hidden), attn_k and
 * attn_v (n_kv_heads*head_dim x hidden), attn_output (hidden x hidden),
 * ffn_norm (f32), ffn_gate and ffn_up (ffn x hidden), ffn_down (hidden x ffn).
 * Matrices are out x in with in fastest (the GGUF orientation); head_dim =
 * hidden / n_heads must be 64 or 128; hidden and ffn multiples of 256.
 *
 * Greedy sampling is sample_with_params (src/inference.rs:1315-1369) with
 * top_k = 1: the lowest index holding the largest logit. */
typedef struct m3g_decoder m3g_decoder;

typedef struct {
    uint64_t n_layers, hidden, ffn, n_heads, n_kv_heads, vocab, max_pos;
    float rope_theta;
} m3g_decoder_config;

M3G_API int m3g_decoder_create(int device, const m3g_decoder_config* cfg, m3g_decoder** out);
/* The same engine sharded over `world` ranks (one process per GPU) sharing
 * one NCCL unique id (m3g_shard_unique_id): each rank keeps the attention
 * weights whole and rows [r*ffn/world, ...) of ffn_gate and ffn_up, rows
 * [r*hidden/world, ...) of ffn_down and rows [r*ceil(vocab/world), ...) of
 * output; uploads still pass the full tensors.  Each step adds two in-place
 * all-gathers per layer and one 64-bit MAX all-reduce of the greedy key.
 * Needs ffn % (8*world) == 0, hidden % world == 0, gate and up of one dtype.
 * Creation gives up with M3G_ETIMEOUT when a rank does not join within
 * timeout_s.  Every rank must issue the same calls in the same order. */
M3G_API int m3g_decoder_create_sharded(int device, const m3g_decoder_config* cfg, int rank, int world,
                                       const uint8_t* nccl_id128, double timeout_s, m3g_decoder** out);
/* Copies one tensor to HBM (replacing an earlier upload of the slot). */
M3G_API int m3g_decoder_upload(m3g_decoder* dec, uint32_t slot, uint32_t dtype, const void* raw, uint64_t raw_len);
/* forward_one(token): one step at the current position; vocab logits to the
 * host when `logits` is not NULL.  Replaces RealInference::forward_one. */
M3G_API int m3g_decoder_forward(m3g_decoder* dec, uint32_t token, float* logits);
/* prefill_logits (src/inference.rs:1388-1399): n steps over the prompt; the
 * last step's logits to the host when `logits` is not NULL.  Afterwards the
 * greedy pick of those logits is pending as the next token. */
M3G_API int m3g_decoder_prefill(m3g_decoder* dec, const uint32_t* tokens, uint64_t n, float* logits);
/* Greedy generation after a prefill or forward: out_tokens[0] is the pending
 * pick, each of the next n_gen - 1 steps feeds the previous pick and picks
 * the next.  All on the device; returns when the tokens are on the host. */
M3G_API int m3g_decoder_generate(m3g_decoder* dec, uint64_t n_gen, uint32_t* out_tokens);
/* Enqueues n_steps greedy steps without waiting (for timing); m3g_decoder_sync
 * waits and reports kernel status. */
M3G_API int m3g_decoder_run_async(m3g_decoder* dec, uint64_t n_steps);
M3G_API int m3g_decoder_sync(m3g_decoder* dec);
/* Token stream entries [first, first + n) (prompt tokens and greedy picks). */
M3G_API int m3g_decoder_tokens(const m3g_decoder* dec, uint64_t first, uint64_t n, uint32_t* out);
/* Positions held in the KV cache. */
M3G_API uint64_t m3g_decoder_pos(const m3g_decoder* dec);
/* truncate_kv_cache: keep the first n positions (0 clears the cache). */
M3G_API int m3g_decoder_truncate(m3g_decoder* dec, uint64_t n);
/* How a sharded decoder exchanges rows: 0 single GPU, 1 NCCL all-gathers,
 * 2 peer stores from the GEMV epilogues over NVLink (chosen at creation when
 * every rank can map every other rank's buffers), 3 only the vocab head is
 * split (every rank keeps the layers; one NCCL all-reduce of the greedy key
 * per step; tuning key decode_shard_ffn = 0 at creation), 4 only the head is
 * split and the greedy keys merge by peer atomics over NVLink (no collective
 * per step; chosen like 2). */
M3G_API int m3g_decoder_exchange(const m3g_decoder* dec);
/* Device logits of the last step and the engine's stream (a cudaStream_t). */
M3G_API const float* m3g_decoder_logits_dev(const m3g_decoder* dec);
M3G_API void* m3g_decoder_stream(const m3g_decoder* dec);
/* 1 (default): replay each step from a captured CUDA graph; 0: launch eagerly. */
M3G_API int m3g_decoder_set_graph(m3g_decoder* dec, int use_graph);
M3G_API void m3g_decoder_destroy(m3g_decoder* dec);

/* ---------------------------------------------------------------- VM opcodes MATVEC and FFN
 *
 * The MATVEC opcode (exec_matvec, src/vm.rs:2643-2685): y[M][N] from x[M][K]
 * (f32) and W of K*N elements (F32, F16 or a block dtype).  M = 1 keeps the
 * reference's matvec::matvec orientation y[j] = sum_i x[i] W[i + j*K] (the
 * fused GEMV for block dtypes); M > 1 keeps its ndarray reading of W as a
 * row-major [K, N] array, y[m][j] = sum_k x[m][k] W[k*N + j].  Device
 * pointers, enqueued on `stream`.  Differences: W is decoded by its ggml
 * dtype (read_f32_tensor, src/memory.rs:1331-1338, decodes a memory::DType
 * Q8_0 tensor with the Q4_K decoder); the row-major sums use another order. */
M3G_API int m3g_vm_matvec_dev(const float* x, uint64_t M, uint64_t K, const uint8_t* w, uint64_t w_len,
                              uint32_t dtype, uint64_t N, float* y, void* stream);
/* The FFN opcode (exec_ffn, src/vm.rs:2471-2576): hidden = x W1 + b1,
 * gated = hidden * sigmoid(hidden), y = gated W2 + b2, x [M][D], W1 row-major
 * [D, H], W2 row-major [H, D_out]; a bias of length H (D_out) is broadcast
 * over the rows, of length M*H (M*D_out) taken per row, any other length (or
 * NULL) is zero.  The hidden buffer is stream-ordered (cudaMallocAsync). */
M3G_API int m3g_vm_ffn_dev(const float* x, uint64_t M, uint64_t D, const uint8_t* w1, uint64_t w1_len,
                           uint32_t dtype1, uint64_t H, const uint8_t* w2, uint64_t w2_len, uint32_t dtype2,
                           uint64_t D_out, const float* b1, uint64_t b1_len, const float* b2, uint64_t b2_len,
                           float* y, void* stream);

/* ---------------------------------------------------------------- greedy head without allocation
 *
 * No counterpart in the reference.  *token (device memory) = the greedy pick
 * of y = W x -- the lowest row index holding the largest value, the pick of
 * sample_with_params with top_k = 1 -- computed by the tensor-core GEMV with
 * its argmax epilogue.  Allocates no device memory: the logits and the
 * reduction key live in a static device array of this library, so out_dim is
 * at most 262144 (M3G_EINVAL beyond).  It runs only on the tensor-core plan:
 * in_dim % 256 == 0, rows of a whole number of 16 bytes (Q4_K, Q8_0, Q4_0
 * rows always are; Q6_K needs in_dim % 2048 == 0), raw and x 16-byte
 * aligned; M3G_EINVAL ("no tensor-core plan") otherwise.  The first call on a
 * device (with that device current) sets up that array's address; make it
 * before any stream capture begins.  A call that finds another context
 * current than at set-up (after cudaDeviceReset) repeats the set-up, so make
 * the first call after a reset outside a capture too.  One call at a time per
 * device: overlapping calls
 * on different streams share the array and race.  *token = 0xFFFFFFFF when a
 * bounded wait inside the GEMV gave up.  Enqueues on `stream` (NULL = the
 * legacy default stream) and returns without waiting. */
M3G_API int m3g_matvec_greedy_noalloc(const float* x, const uint8_t* raw, uint64_t raw_len, uint32_t dtype,
                                      uint64_t in_dim, uint64_t out_dim, uint32_t* token, void* stream);

/* ---------------------------------------------------------------- diagnostics */

/* Error word the kernels of `device` set when a bounded wait gives up
 * (bit 0: a staged-copy wait timed out; bit 3, value 8: a wait for a counter
 * bumped by another GPU or producer ran out, see "peer_wait_us").  clear != 0
 * resets it.  Synchronises the device. */
M3G_API int m3g_device_status(int device, uint32_t* out, int clear);

/* Number of kernel launches this library has enqueued in this process. */
M3G_API uint64_t m3g_launch_count(void);

/* Launch-shape knobs of the streaming GEMV ("stage_bytes", "ctas_per_sm",
 * "max_stages"), "force_generic" (route every GEMV through the
 * row-straddling generic kernel) and "peer_wait_us" (limit, in microseconds,
 * of a kernel's wait for a counter bumped by another GPU or producer; default
 * 2000000; read when a GEMV is enqueued or a decode step captured), "tc8"
 * (1: batch-1 Q4_K GEMVs with in_dim <= 4096 on the tcgen05 kind::i8 kernel;
 * default 0, the mma.sync kernel being faster), "shard_p2p" (see
 * m3g_shard_create) and "offload_mapped" (1, default: host-buffer offload
 * calls through mapped pinned memory; 0: explicit copies).
 * Process-wide; M3G_ENONE for an unknown key or out-of-range value.  No
 * counterpart in the reference. */
M3G_API int m3g_set_tuning(const char* key, int64_t value);

#ifdef __cplusplus
}
#endif
#endif /* M3GEMV_H */
