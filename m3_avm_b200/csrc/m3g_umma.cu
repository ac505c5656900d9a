// m3g_umma.cu -- batched Q4_K GEMV on the fifth-generation tensor cores.
//
// Y[b][j] = sum_i X[b][i] * W[i + j*in] for up to 64 columns of X per pass:
// the per-column product of matvec_q4k (src/matvec_quant.rs:94-170) for a
// batch of activations, the batched-decode shape of the decode loop.
//
// The factorisation is exact.  A Q4_K super-block of row j contributes
//   d * sum_k (sc_g(k) * q_k) * x_k  -  dmin * sum_g m_g * sum_{k in g} x_k
// (dequantize_q4_k, src/quant.rs: d*sc*q - dmin*m per element), where sc, m
// are 6-bit and q 4-bit integers.  sc*q <= 945 and m <= 63 are integers that
// fp16 holds exactly, so the decoded tensor-core operand is exact.  Each
// column of X is scaled per super-block by a power of two (its largest
// magnitude there lands in [2^14, 2^15)) and split into fp16 hi + lo (22
// significant bits); the group sums enter as sum/32 against 32*m (<= 2016,
// still exact) so they stay in fp16 range too.  The tensor core sums the
// exact products in fp32.  Every super-block gets its own fp32 accumulators
// in tensor memory, and the readout threads apply d and dmin in fp32, undo
// the super-block's column scale (exact) and add the super-blocks in order.
//
// k_umma_q4k<NB, C> (NB = 8, 16, 32 or 64; one CTA per SM, 512 TMEM columns;
// D = 16 decoder warps for NB <= 16, 8 otherwise; R = 4 readout warps, 8 for
// NB = 64):
//   decoders    warp w owns TMEM lanes 32*(w%4).. (one weight row per
//               thread) and part w/4 of the super-block's quants; they decode
//               the 4-bit quants straight into tensor memory (tcgen05.st, the
//               A operand), the m values into shared memory and (d, dmin) into
//               a shared ring;
//   readout     warp D+r reads lanes 32*(r%4).. of the super-block's
//               accumulators back (tcgen05.ld; two warps per quarter split the
//               columns), applies d, dmin and the column scale, keeps the
//               per-row fp32 sums and writes finished tiles;
//   producer    warp D+R: per super-block, one 2-D tensor copy of the 128-row
//               weight tile (a box of 36 words x 128 rows of the row-major
//               Q4_K matrix; rows past the end read as zero) and one bulk
//               copy of the prepared X tile;
//   issuers     C warps (the first also allocates TMEM): lane 0 of issuer c
//               issues the K-steps t = c, c + C, ... of each super-block
//               (M = 128, N = 2*NB, K = 16): sc*q (TMEM) x [X hi | X lo]
//               (shared) into main accumulator c; the last issuer also issues
//               m (shared) x [group sums hi | lo] into the min accumulator;
//               each commits once per super-block.  An MMA costs an issuing
//               warp about as much at N = 32 as at N = 128 and several issuing
//               warps proceed in parallel, so the hi and lo halves of X share
//               one instruction and C warps issue.
// The (tile, super-block) iteration space is split evenly over the CTAs; a
// tile cut between CTAs is finished by the CTA whose piece completes it, which
// adds the pieces in CTA order (the result does not depend on timing).
//
// TMEM columns: A [2 stages][128] | DB buffers of (C main + 1 min) x 2*NB.
// Every wait is bounded; a timeout raises the copy-timeout status bit and the
// CTA runs to its end without waiting again, freeing its tensor memory.
#include <cstdint>
#include <mutex>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "m3g_device.cuh"
#include "m3g_internal.h"

namespace m3g {
namespace {

constexpr int kTileRows = 128;
constexpr int kSBBytes = 144;                       // Q4_K super-block
constexpr int kStageW = kTileRows * kSBBytes;       // one weight stage: 128 rows x 1 super-block
// Decoder warps for NB accumulator columns (16: four per TMEM lane quarter).
__host__ __device__ constexpr int umma_decoders(int nb) { return nb <= 16 ? 16 : 8; }
// Readout warps: one or two per TMEM lane quarter (two split the columns).
__host__ __device__ constexpr int umma_readouts(int nb) { return nb <= 32 ? 4 : 8; }
// Warps: decoders | readout | producer | C MMA issuers.
__host__ __device__ constexpr int umma_threads(int nb, int issuers) {
  return 32 * (umma_decoders(nb) + umma_readouts(nb) + 1 + issuers);
}
constexpr int kAmBytes = 4096;                      // one m-operand stage: 128 rows x 16 fp16
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kUmmaTimeoutNs = 2000000000ull;  // 2 s

// ------------------------------------------------------------ tcgen05 PTX
__device__ __forceinline__ void tc_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrive once on `bar` when every earlier MMA of this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// D (TMEM) (+)= A (TMEM) x B (shared memory descriptor); kind::f16, fp32 D.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D (TMEM) (+)= A (shared) x B (shared).
__device__ __forceinline__ void tc_mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Two loads of 8 columns (main and min accumulators) and the wait for them,
// in one statement so no use of the results can be scheduled before the wait.
__device__ __forceinline__ void tc_ld2x8(uint32_t ta, uint32_t tb, uint32_t (&x)[8], uint32_t (&y)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%17];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]), "=r"(y[0]),
        "=r"(y[1]), "=r"(y[2]), "=r"(y[3]), "=r"(y[4]), "=r"(y[5]), "=r"(y[6]), "=r"(y[7])
      : "r"(ta), "r"(tb)
      : "memory");
}
// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices, `lbo` bytes between the two core matrices along K, `sbo` bytes
// between 8-row groups; descriptor version 1, base offset 0.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: fp16 A and B, both K-major, fp32 D, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16_m128(int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// The bytes that selector nibbles 0 and 2 pick from the 8 bytes {hi:lo}, as
// an fp16 pair of small integers: (1024 + v) - 1024, exact.
__device__ __forceinline__ uint32_t byte_pair_f16(uint32_t lo, uint32_t hi, uint32_t sel) {
  return hfma2(0x64006400u | (__byte_perm(lo, hi, sel) & 0x00FF00FFu), 0x3C003C00u, 0xE400E400u);
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 2-D tiled tensor copy global -> this CTA's shared memory (no multicast):
// box origin (x words, y rows) of the tensor map, completing its bytes on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// K position k' (0..255) of a super-block's decoded operand -> element index.
// Column c = k'/2 of TMEM holds the fp16 pair the decoder builds from byte
// lane p = c%4 of word u = (c/4)%4 of 16-byte vector v = c/16 of the quants.
__host__ __device__ constexpr int umma_elem(int kp) {
  const int c = kp >> 1, h = kp & 1, v = c >> 4, u = (c >> 2) & 3, p = c & 3;
  return 64 * (v >> 1) + 16 * (v & 1) + 4 * u + 32 * (p & 1) + (p >> 1) + 2 * h;
}

__device__ __forceinline__ void raise_timeout(volatile int* abort_flag, uint32_t* status) {
  *abort_flag = 1;
  atomicOr(status, kStatusCopyTimeout);
}

}  // namespace

// X tile bytes per super-block for NB columns: 16 K-steps of the main operand
// then one K-step of group sums, each K-step 2*NB rows (rows n < NB the hi
// halves of column n, rows NB + n the lo halves) x 16 fp16, K-major.
__host__ __device__ constexpr int umma_xtile_bytes(int nb) { return 1088 * nb; }

// 2^e as a float, exactly (|e| <= 126).
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// One super-block s of X per CTA: each column scaled by a power of two (its
// largest magnitude in the super-block lands in [2^14, 2^15); the inverse goes
// to sig[s][n] for the epilogue), permuted to the decoder's K order, split into
// fp16 hi/lo and laid out as the MMA's K-major B tiles.  Also zeroes the tile
// counters of the launch that follows.
template <int NB>
__global__ void __launch_bounds__(256) k_umma_xprep(const float* __restrict__ x, int cols, long long in_dim,
                                                    float* __restrict__ sig, uint8_t* __restrict__ xt,
                                                    unsigned* __restrict__ cnt, int tiles) {
  extern __shared__ float xsm[];  // [NB][257] scaled values, then [NB][8] group sums, then [NB] scales
  float* gsum = xsm + NB * 257;
  float* sinv = gsum + NB * 8;
  const int s = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The GEMM kernel that follows may start now: it streams and decodes the
  // weights, and waits for this grid before it touches X, the scales or the
  // counters.
  grid_dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tiles; i += gridDim.x * blockDim.x) cnt[i] = 0u;
  for (int i = threadIdx.x; i < NB * 256; i += blockDim.x) {
    const int n = i >> 8, e = i & 255;
    xsm[n * 257 + e] = n < cols ? x[static_cast<long long>(n) * in_dim + static_cast<long long>(s) * 256 + e] : 0.f;
  }
  __syncthreads();
  for (int n = warp; n < NB; n += 8) {
    float m = 0.f;
#pragma unroll
    for (int e = lane; e < 256; e += 32) m = fmaxf(m, fabsf(xsm[n * 257 + e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    int e = 0;
    if (m > 0.f && m <= 3.4e38f) e = min(110, max(-110, ilogbf(m) - 14));
    if (lane == 0) {
      sinv[n] = pow2f(-e);
      sig[static_cast<size_t>(s) * NB + n] = pow2f(e);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB * 256; i += blockDim.x) {
    const int n = i >> 8, e = i & 255;
    xsm[n * 257 + e] *= sinv[n];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB * 8; i += blockDim.x) {
    const int n = i >> 3, g = i & 7;
    float sum = 0.f;
    for (int e = 0; e < 32; ++e) sum += xsm[n * 257 + 32 * g + e];
    gsum[i] = sum * 0.03125f;  // sum / 32 stays below 2^15 in fp16; the m operand carries 32 * m
  }
  uint8_t* out = xt + static_cast<size_t>(s) * umma_xtile_bytes(NB);
  // main tiles: one 16-byte chunk = 8 consecutive K positions of one column
  for (int ch = threadIdx.x; ch < 32 * NB; ch += blockDim.x) {
    const int kc = ch & 1, n = (ch >> 1) % NB, t = (ch >> 1) / NB;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v0 = xsm[n * 257 + umma_elem(16 * t + 8 * kc + 2 * j)];
      const float v1 = xsm[n * 257 + umma_elem(16 * t + 8 * kc + 2 * j + 1)];
      const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      hi[j] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
      lo[j] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
    }
    const int off = t * 64 * NB + kc * 128;
    const int nl = n + NB;
    *reinterpret_cast<uint4*>(out + off + (n >> 3) * 256 + (n & 7) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(out + off + (nl >> 3) * 256 + (nl & 7) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  __syncthreads();
  // group-sum tiles: K positions 0..7 = groups, 8..15 zero
  for (int ch = threadIdx.x; ch < 2 * NB; ch += blockDim.x) {
    const int kc = ch & 1, n = ch >> 1;
    uint32_t hi[4] = {0u, 0u, 0u, 0u}, lo[4] = {0u, 0u, 0u, 0u};
    if (kc == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v0 = gsum[n * 8 + 2 * j], v1 = gsum[n * 8 + 2 * j + 1];
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
        hi[j] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
        lo[j] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
      }
    }
    const int off = 1024 * NB + kc * 128;
    const int nl = n + NB;
    *reinterpret_cast<uint4*>(out + off + (n >> 3) * 256 + (n & 7) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(out + off + (nl >> 3) * 256 + (nl & 7) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

template <int NB, int C>
__global__ void __launch_bounds__(umma_threads(NB, C), 1)
    k_umma_q4k(const UmmaArgs a, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kThreads = umma_threads(NB, C);
  constexpr int kDec = umma_decoders(NB);         // decoder warps
  constexpr int kParts = kDec / 4;                // decoder warps per TMEM lane quarter
  constexpr int kVecs = 8 / kParts;               // 16-byte quant vectors per decoder thread
  constexpr int kRd = umma_readouts(NB);           // readout warps
  constexpr int RC = NB / (kRd / 4);               // accumulator columns per readout thread
  constexpr int kProducer = kDec + kRd;            // producer warp
  constexpr int kIssuer0 = kProducer + 1;          // first MMA issuer (allocates TMEM)
  constexpr int DW = 2 * NB;                                            // accumulator width
  constexpr int DB = 256 + 2 * (C + 1) * DW <= static_cast<int>(kTmemCols) ? 2 : 1;  // accumulator buffers
  static_assert(256 + DB * (C + 1) * DW <= static_cast<int>(kTmemCols), "TMEM columns");
  constexpr uint32_t XS = umma_xtile_bytes(NB);
  constexpr int CH = 8;  // accumulator columns per tcgen05.ld
  static_assert(RC % CH == 0, "readout columns");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long G = gridDim.x;
  const long long it0 = static_cast<long long>(blockIdx.x) * a.T / G;
  const long long it1 = static_cast<long long>(blockIdx.x + 1) * a.T / G;
  const int K = static_cast<int>(it1 - it0);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* wempty = wfull + a.NSW;
  uint64_t* xfull = wempty + a.NSW;
  uint64_t* afull = xfull + a.NSX;  // [2] decoded operand stage ready (decoder warps)
  uint64_t* dfree = afull + 2;      // [2] accumulator buffer read back (readout warps)
  uint64_t* ddfull = dfree + 2;     // [4] d, dmin of super-block k written (decoder warps of part 0)
  uint64_t* sbdone = ddfull + 4;    // [4] MMAs of super-block k complete (one commit per issuer)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sbdone + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  volatile int* fin_flag = reinterpret_cast<volatile int*>(tslot + 2);
  uint8_t* am = smem + a.off_am;                                           // [2][4 KB] m operand
  float2* dd = reinterpret_cast<float2*>(smem + a.off_am + 2 * kAmBytes);  // [4][128] (d, dmin)
  // Super-block k's MMAs complete <=> phase k/4 of sbdone[k % 4].  Every waiter
  // is at most one phase behind: the barrier's next phase needs work that
  // comes after the wait in the waiter's own order.
  auto wait_sb = [&](int k) {
    return mbar_wait_bounded(&sbdone[k & 3], (k >> 2) & 1, kUmmaTimeoutNs, abort_flag);
  };

  if (tid == 0) {
    for (int s = 0; s < a.NSW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kDec);
    }
    for (int s = 0; s < a.NSX; ++s) mbar_init(&xfull[s], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull[s], kDec);
      mbar_init(&dfree[s], kRd);
    }
    for (int s = 0; s < 4; ++s) {
      mbar_init(&ddfull[s], 4);
      mbar_init(&sbdone[s], C);
    }
    *abort_flag = 0;
    *fin_flag = 0;
    fence_mbar_init();
  }
  // K positions 8..15 of the m operand stay zero
  for (int i = tid; i < 2 * kAmBytes / 16; i += kThreads) reinterpret_cast<uint4*>(am)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == kIssuer0) {
    tc_alloc(tslot, kTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp < kDec) {
    // ------------------------------------------------------------ decoders
    const int q = warp & 3, part = warp >> 2;
    const int r = 32 * q + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * q) << 16);
    const int g0 = part * kVecs;  // first group of this thread's vectors (a vector pair spans two groups)
    int ws = 0, wph = 0;
    for (int k = 0; k < K; ++k) {
      const int buf = k & 1;
      if (!mbar_wait_bounded(&wfull[ws], wph, kUmmaTimeoutNs, abort_flag) || (k >= 2 && !wait_sb(k - 2)))
        raise_timeout(abort_flag, a.status);
      const uint8_t* rowp = smem + static_cast<size_t>(ws) * kStageW + r * kSBBytes;
      const uint4 hd = *reinterpret_cast<const uint4*>(rowp);
      uint4 qv[kVecs];
#pragma unroll
      for (int v = 0; v < kVecs; ++v) qv[v] = *reinterpret_cast<const uint4*>(rowp + 16 + 16 * (part * kVecs + v));
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[ws]);
      if (++ws == a.NSW) ws = 0, wph ^= 1;
      tc_fence_after();
      // 6-bit scales and mins of all eight groups (get_scale_min_k4)
      const uint32_t sc_lo = hd.y & 0x3F3F3F3Fu, m_lo = hd.z & 0x3F3F3F3Fu;
      const uint32_t sc_hi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
      const uint32_t m_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
      // byte_perm selector of group g into result bytes 0 and 2
      auto sel2 = [](int ga, int gb) { return static_cast<uint32_t>(ga) | (static_cast<uint32_t>(gb) << 8); };
      // low nibbles enter as 1024 + q, high nibbles in place as 1024 + 16 q:
      // q*sc = (1024 + q)*sc - 1024*sc = (1024 + 16q)*(sc/16) - 64*sc, exact
      constexpr int NG = kVecs / 2 > 0 ? kVecs / 2 : 1;  // vector pairs = group pairs
      uint32_t SL[NG], NL[NG], SH[NG], NH[NG];
#pragma unroll
      for (int j = 0; j < NG; ++j) {
        const int ga = g0 + 2 * j, gb = ga + 1;
        SL[j] = byte_pair_f16(sc_lo, sc_hi, sel2(ga, ga));
        NL[j] = hfma2(SL[j], 0xE400E400u, 0x80008000u);  // -1024 * sc
        const uint32_t S = byte_pair_f16(sc_lo, sc_hi, sel2(gb, gb));
        SH[j] = hfma2(S, 0x2C002C00u, 0x80008000u);      // sc / 16
        NH[j] = hfma2(S, 0xD400D400u, 0x80008000u);      // -64 * sc
      }
#pragma unroll
      for (int v = 0; v < kVecs; ++v) {
        const uint32_t wv[4] = {qv[v].x, qv[v].y, qv[v].z, qv[v].w};
        const int j = v >> 1;
        uint32_t o[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t w = wv[u], w8 = w >> 8;
          o[4 * u + 0] = hfma2((w & 0x000F000Fu) | 0x64006400u, SL[j], NL[j]);
          o[4 * u + 1] = hfma2((w & 0x00F000F0u) | 0x64006400u, SH[j], NH[j]);
          o[4 * u + 2] = hfma2((w8 & 0x000F000Fu) | 0x64006400u, SL[j], NL[j]);
          o[4 * u + 3] = hfma2((w8 & 0x00F000F0u) | 0x64006400u, SH[j], NH[j]);
        }
        tc_st16(tl + static_cast<uint32_t>(buf * 128 + 16 * (part * kVecs + v)), o);
      }
      {
        // 32 * m (<= 2016, exact in fp16) against the group sums / 32
        uint8_t* dst = am + buf * kAmBytes + (r >> 3) * 256 + (r & 7) * 16 + 2 * g0;
        if constexpr (kVecs == 4) {
          const uint32_t m01 = hfma2(byte_pair_f16(m_lo, m_hi, sel2(g0, g0 + 1)), 0x50005000u, 0x80008000u);
          const uint32_t m23 = hfma2(byte_pair_f16(m_lo, m_hi, sel2(g0 + 2, g0 + 3)), 0x50005000u, 0x80008000u);
          *reinterpret_cast<uint2*>(dst) = make_uint2(m01, m23);
        } else {
          *reinterpret_cast<uint32_t*>(dst) =
              hfma2(byte_pair_f16(m_lo, m_hi, sel2(g0, g0 + 1)), 0x50005000u, 0x80008000u);
        }
      }
      if (part == 0) {
        dd[(k & 3) * kTileRows + r] =
            make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(hd.x & 0xFFFFu))),
                        __half2float(__ushort_as_half(static_cast<unsigned short>(hd.x >> 16))));
      }
      tc_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[buf]);
        if (part == 0) mbar_arrive(&ddfull[k & 3]);
      }
    }
  } else if (warp < kProducer) {
    // ------------------------------------------------------------ readout / epilogue
    grid_dep_wait();  // the column scales and the tile counters come from the X prep
    const int q = warp & 3, cb = kRd == 4 ? 0 : ((warp - kDec) >> 2) * RC;  // lane quarter, first column
    const int r = 32 * q + lane;
    const int rt = tid - kDec * 32;  // index within the readout warps
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * q) << 16);
    const long long tile0 = it0 / a.NSB;
    long long rtile = tile0;  // tile and super-block being read back
    int rs = static_cast<int>(it0 - tile0 * a.NSB);
    float acc[RC];
#pragma unroll
    for (int c = 0; c < RC; ++c) acc[c] = 0.f;

    auto flush = [&](long long tile, int sbeg, int send) {
      const long long row = tile * kTileRows + r;
      if (sbeg == 0 && send == a.NSB) {
        if (row < a.rows) {
#pragma unroll
          for (int c = 0; c < RC; ++c)
            if (cb + c < a.cols) a.y[static_cast<long long>(cb + c) * a.ldy + row] = acc[c];
        }
      } else {
        const int slot = tile == tile0 ? 0 : 1;
        float* p = a.part + (static_cast<size_t>(blockIdx.x) * 2 + slot) * NB * kTileRows;
#pragma unroll
        for (int c = 0; c < RC; ++c) p[(cb + c) * kTileRows + r] = acc[c];
        __threadfence();
        named_bar_sync(1, 32 * kRd);
        if (rt == 0) {
          const unsigned len = static_cast<unsigned>(send - sbeg);
          *fin_flag = atomicAdd(&a.cnt[tile], len) + len == static_cast<unsigned>(a.NSB) ? 1 : 0;
        }
        named_bar_sync(1, 32 * kRd);
        if (*fin_flag) {
          __threadfence();
          const long long i_first = tile * a.NSB, i_last = i_first + a.NSB - 1;
          const long long c0 = ((i_first + 1) * G - 1) / a.T, c1 = ((i_last + 1) * G - 1) / a.T;
          // the pieces in CTA order (this CTA's own included, from the buffer)
#pragma unroll
          for (int c = 0; c < RC; ++c) acc[c] = 0.f;
          for (long long cta = c0; cta <= c1; ++cta) {
            const int sl = (cta * a.T / G) / a.NSB == tile ? 0 : 1;
            const float* pp = a.part + (static_cast<size_t>(cta) * 2 + sl) * NB * kTileRows;
#pragma unroll
            for (int c = 0; c < RC; ++c) acc[c] += __ldcg(pp + (cb + c) * kTileRows + r);
          }
          if (row < a.rows) {
#pragma unroll
            for (int c = 0; c < RC; ++c)
              if (cb + c < a.cols) a.y[static_cast<long long>(cb + c) * a.ldy + row] = acc[c];
          }
        }
        named_bar_sync(1, 32 * kRd);  // fin_flag is rewritten by the next piece
      }
#pragma unroll
      for (int c = 0; c < RC; ++c) acc[c] = 0.f;
    };

    for (int kk = 0; kk < K; ++kk) {
      const int db = DB == 2 ? (kk & 1) : 0;
      float sg[RC];  // column scales of this super-block, fetched before the waits
#pragma unroll
      for (int c = 0; c < RC; ++c) sg[c] = __ldg(a.sig + static_cast<size_t>(rs) * NB + cb + c);
      if (!mbar_wait_bounded(&ddfull[kk & 3], (kk >> 2) & 1, kUmmaTimeoutNs, abort_flag) || !wait_sb(kk))
        raise_timeout(abort_flag, a.status);
      const float2 dm = dd[(kk & 3) * kTileRows + r];
      __syncwarp();
      tc_fence_after();
      const uint32_t dbase = tl + 256u + static_cast<uint32_t>(db * (C + 1) * DW + cb);
#pragma unroll
      for (int c0 = 0; c0 < RC; c0 += CH) {
        float sm[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) sm[c] = 0.f;
#pragma unroll
        for (int ch = 0; ch <= C; ++ch) {  // C main accumulators, then the min accumulator
          uint32_t u[CH], v[CH];
          const uint32_t ta = dbase + static_cast<uint32_t>(ch * DW + c0);
          tc_ld2x8(ta, ta + NB, u, v);  // hi and lo halves of columns c0..c0+7
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const float hl = __uint_as_float(u[c]) + __uint_as_float(v[c]);
            if (ch < C) sm[c] += hl;
            else acc[c0 + c] = fmaf(sg[c0 + c], fmaf(dm.x, sm[c], -dm.y * hl), acc[c0 + c]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfree[db]);
      if (rs == a.NSB - 1 || kk == K - 1)
        flush(rtile, rtile == tile0 ? static_cast<int>(it0 - tile0 * a.NSB) : 0, rs + 1);
      if (++rs == a.NSB) rs = 0, ++rtile;
    }
  } else if (warp == kProducer) {
    // ------------------------------------------------------------ producer
    const uint64_t wpol = l2_evict_first_policy(), xpol = l2_evict_last_policy();
    int wiss = 0, xiss = 0;  // weight and X stages issued
    if (lane == 0) {
      long long tile = it0 / a.NSB;
      int s = static_cast<int>(it0 - tile * a.NSB), ws = 0, wph = 0, xs = 0, xph = 0;
      // The X prep never writes the weights: the first weight stages (all
      // free at the start) stream while it finishes; the X tiles wait for it.
      const int npre = min(K, a.NSW);
      {
        long long t2 = tile;
        int s2 = s;
        for (; wiss < npre; ++wiss) {
          mbar_arrive_expect_tx(&wfull[wiss], static_cast<uint32_t>(kStageW));
          tma_load_2d(smem + static_cast<size_t>(wiss) * kStageW, &wmap, s2 * (kSBBytes / 4),
                      static_cast<int>(t2 * kTileRows), &wfull[wiss], wpol);
          if (++s2 == a.NSB) s2 = 0, ++t2;
        }
      }
      grid_dep_wait();
      for (int k = 0; k < K; ++k) {
        if (*abort_flag) break;
        if (k >= npre) {  // weight stage free (decoders)
          if (!mbar_wait_bounded(&wempty[ws], wph ^ 1, kUmmaTimeoutNs, abort_flag)) {
            raise_timeout(abort_flag, a.status);
            break;
          }
          mbar_arrive_expect_tx(&wfull[ws], static_cast<uint32_t>(kStageW));
          tma_load_2d(smem + static_cast<size_t>(ws) * kStageW, &wmap, s * (kSBBytes / 4),
                      static_cast<int>(tile * kTileRows), &wfull[ws], wpol);
          wiss = k + 1;
        }
        // X stage free (the MMAs of super-block k - NSX)
        if (k >= a.NSX && !wait_sb(k - a.NSX)) {
          raise_timeout(abort_flag, a.status);
          break;
        }
        mbar_arrive_expect_tx(&xfull[xs], XS);
        bulk_g2s(smem + a.off_x + static_cast<size_t>(xs) * XS, a.xt + static_cast<size_t>(s) * XS, XS, &xfull[xs],
                 xpol);
        xiss = k + 1;
        if (++ws == a.NSW) ws = 0, wph ^= 1;
        if (++xs == a.NSX) xs = 0, xph ^= 1;
        if (++s == a.NSB) s = 0, ++tile;
      }
    }
    wiss = __shfl_sync(0xFFFFFFFFu, wiss, 0);
    xiss = __shfl_sync(0xFFFFFFFFu, xiss, 0);
    // every copy this warp issued lands before the CTA can exit
    for (int k = max(0, wiss - a.NSW); k < wiss; ++k)
      mbar_wait_bounded(&wfull[k % a.NSW], (k / a.NSW) & 1, kUmmaTimeoutNs, nullptr);
    for (int k = max(0, xiss - a.NSX); k < xiss; ++k)
      mbar_wait_bounded(&xfull[k % a.NSX], (k / a.NSX) & 1, kUmmaTimeoutNs, nullptr);
  } else {
    // ------------------------------------------------------------ MMA issuers
    const int ci = warp - kIssuer0;  // issuer / main accumulator index
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_m128(DW);
      const uint32_t xbase = smem_addr(smem + a.off_x), ambase = smem_addr(am);
      int last = -1, xs = 0, xph = 0;
      for (int k = 0; k < K; ++k) {
        if (*abort_flag) break;
        const int buf = k & 1, db = DB == 2 ? (k & 1) : 0, use = DB == 2 ? (k >> 1) : k;
        if (!mbar_wait_bounded(&xfull[xs], xph, kUmmaTimeoutNs, abort_flag) ||
            !mbar_wait_bounded(&afull[buf], (k >> 1) & 1, kUmmaTimeoutNs, abort_flag) ||
            !mbar_wait_bounded(&dfree[db], (use & 1) ^ 1, kUmmaTimeoutNs, abort_flag)) {
          raise_timeout(abort_flag, a.status);
          break;
        }
        tc_fence_after();
        const uint32_t dbase = tbase + 256u + static_cast<uint32_t>(db * (C + 1) * DW);
        const uint32_t aop = tbase + static_cast<uint32_t>(buf * 128);
        const uint32_t xb = xbase + static_cast<uint32_t>(xs) * XS;
#pragma unroll
        for (int t = ci; t < 16; t += C)
          tc_mma_ts(dbase + static_cast<uint32_t>(ci * DW), aop + 8u * t, smem_desc(xb + t * 64u * NB, 128u, 256u),
                    idesc, t >= C ? 1u : 0u);
        if (ci == C - 1)
          tc_mma_ss(dbase + static_cast<uint32_t>(C * DW),
                    smem_desc(ambase + static_cast<uint32_t>(buf) * kAmBytes, 128u, 256u),
                    smem_desc(xb + 1024u * NB, 128u, 256u), idesc, 0u);
        tc_commit(&sbdone[k & 3]);
        last = k;
        if (++xs == a.NSX) xs = 0, xph ^= 1;
      }
      // the tensor core is idle before the allocation is released
      if (last >= 0) mbar_wait_bounded(&sbdone[last & 3], (last >> 2) & 1, kUmmaTimeoutNs, nullptr);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kIssuer0) {
    tc_fence_after();
    tc_dealloc(tbase, kTmemCols);
  }
}

namespace {
template <auto Kern>
cudaError_t set_smem(size_t bytes) {
  return cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}
}  // namespace

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

template <int NB, int C>
cudaError_t launch_q4k(const UmmaArgs& a, int grid, size_t smem, const CUtensorMap& wmap, cudaStream_t st,
                      bool pdl) {
  cudaError_t e = set_smem<k_umma_q4k<NB, C>>(smem);
  if (e != cudaSuccess) return e;
  // Programmatic dependent launch: the kernel may start while the X prep
  // before it runs (see k_umma_xprep / the producer and readout waits).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(umma_threads(NB, C)));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_umma_q4k<NB, C>, a, wmap);
}

// Largest chain count that fits TMEM for NB columns, capped by the request.
template <int NB>
cudaError_t launch_nb(const UmmaArgs& a, const float* x, long long in_dim, int chains, int grid, size_t smem,
                      int xprep_smem, const CUtensorMap& wmap, cudaStream_t st, bool pdl) {
  cudaError_t e = set_smem<k_umma_xprep<NB>>(xprep_smem);
  if (e != cudaSuccess) return e;
  k_umma_xprep<NB><<<a.NSB, 256, xprep_smem, st>>>(x, a.cols, in_dim, const_cast<float*>(a.sig),
                                                    const_cast<uint8_t*>(a.xt), a.cnt, a.tiles);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if constexpr (NB == 8) {
    if (chains >= 3) return launch_q4k<8, 3>(a, grid, smem, wmap, st, pdl);
    if (chains >= 2) return launch_q4k<8, 2>(a, grid, smem, wmap, st, pdl);
    return launch_q4k<8, 1>(a, grid, smem, wmap, st, pdl);
  } else if constexpr (NB == 16) {
    if (chains >= 3) return launch_q4k<16, 3>(a, grid, smem, wmap, st, pdl);
    if (chains >= 2) return launch_q4k<16, 2>(a, grid, smem, wmap, st, pdl);
    return launch_q4k<16, 1>(a, grid, smem, wmap, st, pdl);
  } else if constexpr (NB == 32) {
    if (chains >= 3) return launch_q4k<32, 3>(a, grid, smem, wmap, st, pdl);
    if (chains >= 2) return launch_q4k<32, 2>(a, grid, smem, wmap, st, pdl);
    return launch_q4k<32, 1>(a, grid, smem, wmap, st, pdl);
  } else {
    return launch_q4k<64, 1>(a, grid, smem, wmap, st, pdl);
  }
}

cudaError_t launch_umma_q4k(const UmmaArgs& a, const float* x, long long in_dim, int nb, int chains, int grid,
                            size_t smem, cudaStream_t st, bool pdl) {
  // The weight matrix as rows x (RB / 4) words; one box = one super-block of 128 rows.
  auto encode = tensor_map_encoder();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap wmap;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.RB / 4), static_cast<cuuint64_t>(a.rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.RB)};
  const cuuint32_t box[2] = {kSBBytes / 4, kTileRows};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(a.w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const int xprep_smem = (nb * 257 + nb * 8 + nb) * 4;
  cudaError_t e = cudaSuccess;
  switch (nb) {
    case 8: e = launch_nb<8>(a, x, in_dim, chains, grid, smem, xprep_smem, wmap, st, pdl); break;
    case 16: e = launch_nb<16>(a, x, in_dim, chains, grid, smem, xprep_smem, wmap, st, pdl); break;
    case 32: e = launch_nb<32>(a, x, in_dim, chains, grid, smem, xprep_smem, wmap, st, pdl); break;
    case 64: e = launch_nb<64>(a, x, in_dim, chains, grid, smem, xprep_smem, wmap, st, pdl); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int umma_xtile(int nb) { return umma_xtile_bytes(nb); }

}  // namespace m3g
