// m3g_tc8.cu -- the batch-1 Q4_K GEMV on the fifth-generation tensor cores.
//
// y[j] = sum_i x[i] * W[i + j*in] for Q4_K weights: matvec_q4k
// (src/matvec_quant.rs:221-356) on one vector.  The quant bytes are the MMA
// operand as they lie in HBM.  A byte of a 144-byte block holds two 4-bit
// quants, lo (element 64c + l of the super-block) and hi (element
// 64c + 32 + l); read as an unsigned 8-bit integer it is lo + 16 hi, and
// masked with 0xF0 it is 16 hi.  With x split per super-block into three
// int8 slices (x ~= s * (x0 + x1/254 + x2/254^2), as the mma.sync GEMV does),
// one 32-byte chunk c of the quants gives, in one accumulator of 16 columns,
//   D[n < 3]  = sum_l (lo + 16 hi) * x_lo,n  -  sum_l 16 hi * x_lo,n  = sum_l lo * x_lo,n
//   D[3 + n]  = sum_l 16 hi * x_hi,n
// from two kind::i8 MMAs (K = 32 each): the raw bytes against [x_lo | 0] and
// the masked bytes against [-x_lo | x_hi].  Integer and exact.  The 6-bit
// sub-block scales multiply these per row in the readout, where d, dmin,
// the min terms (dmin * sum m * sum x) and the slice weights are applied in
// fp32 -- the same factorisation as the mma.sync kernel, with the products
// done by the tensor core and the accumulators in tensor memory.
//
// Per CTA (one per SM): a contiguous range of rows, cut into tiles of at most
// 128 rows (the MMA's M; a tile's TMA box is exactly its rows), every
// super-block of each.  No tile is shared between CTAs, so no fix-up pass.
// Units (tile, super-block) flow through kNST shared-memory stages and kNA
// tensor-memory A buffers:
//   producer  warp 0: one 2-D tensor copy of the unit's quants (128-byte
//             rows, 128-byte swizzle) and one of its 16-byte block headers;
//   maskers   warps 1-8, one row per thread: warps 1-4 copy the row's 128
//             quant bytes into tensor memory as they are (the raw A operand),
//             warps 5-8 masked with 0xF0 (the 16 hi operand);
//   readout   warps 9-12, one row per thread: the eight accumulators back
//             from tensor memory, scales, d, dmin, the sum over super-blocks,
//             y;
//   issuers   warps 13-20: one MMA each per unit (chunk c = i / 2, raw or
//             masked = i % 2; A in tensor memory, B in shared memory; M = 128,
//             N = 16, K = 32) into its own accumulator, and one commit.  A
//             kind::i8 MMA holds its issuing thread for ~230 SM clocks
//             whatever N is, while eight issuing warps overlap almost fully
//             (~35 clocks per MMA, measured on B200), so the eight MMAs of a
//             unit go out from eight warps at once.
// Before their first unit, the readout and issuer warps turn x into int8
// slices written straight into the x operand tiles of every super-block
// (K <= 4096); the maskers and the producer run ahead meanwhile.  With PRE <
// kNST the producer streams only PRE stages until x is in registers, so the
// loads of x do not queue behind the whole ring.  An x tile holds only the
// eight rows of N that can be nonzero; the descriptor's row-group stride
// points the other eight at a shared block of zeros.  Every wait is bounded;
// a timeout raises the copy-timeout status bit and every role leaves its
// loop, so the CTA frees its tensor memory and exits.
//
// Off by default (tuning key tc8): on the headline shape (14336 x 4096, 97
// rows and 16 units per SM) it takes 12.5 us against 9.3 us for the mma.sync
// kernel.  A phase trace of one CTA shows the tensor-core side keeping up
// (masker ~150 ns, issue ~250 ns, readout ~250 ns a unit, overlapped); what
// binds is the weight stream: the row-strided boxes (one 128- and one
// 16-byte piece per row and unit) land at ~30 GB/s per SM inside the kernel,
// and x arrives ~2.5 us after the CTA starts.  A 3-D box of two super-blocks
// per copy (144-byte rows) landed at ~20 GB/s per SM, with L2-resident
// weights as well.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "m3g_device.cuh"
#include "m3g_internal.h"

namespace m3g {
namespace {

constexpr int kRawStage = 128 * 128;  // quants of one unit: up to 128 rows x 128 bytes
constexpr int kHdrStage = 128 * 16;   // block headers of one unit: up to 128 rows x 16 bytes
constexpr int kStage = kRawStage + kHdrStage;
constexpr int kBTile = 2048;          // x operand of one super-block: [chunk 4][K-step 2][K half 2][row 8][16 bytes]
constexpr int kZeroBytes = 256;       // the zero row group every x tile's rows 8-15 point at
constexpr int kNST = 8;               // shared-memory stages
constexpr int kNA = 4;                // tensor-memory A buffers
constexpr int kMaxNSB = 16;           // super-blocks whose x tiles fit shared memory (K <= 4096)
constexpr int kMaskWarps = 8, kReadWarps = 4, kIssuers = 8;
constexpr int kProducerW = 0, kMask0 = 1, kRead0 = kMask0 + kMaskWarps, kIssue0 = kRead0 + kReadWarps;
constexpr int kPrepWarps = kReadWarps + kIssuers;    // readout and issuers prepare x
constexpr int kThreads = 32 * (kIssue0 + kIssuers);  // 672
// TMEM columns: A operands [kNA][raw 32 | 16 hi 32] (4 int8 per column),
// then accumulators [2][8 MMAs][16].
constexpr uint32_t kTmemA = 0, kTmemD = 64 * kNA, kTmemCols = 512;
static_assert(kTmemD + 2 * 16 * kIssuers <= kTmemCols, "TMEM columns");
constexpr uint64_t kWaitNs = 2000000000ull;          // 2 s

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
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// Columns 0..7 of the four chunk accumulators of this thread's lane, and the wait.
__device__ __forceinline__ void tc_ld4x8(uint32_t t0, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%33];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%34];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24, %25, %26, %27, %28, %29, %30, %31}, [%35];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(t0), "r"(t0 + 16u), "r"(t0 + 32u), "r"(t0 + 48u)
      : "memory");
}
// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (TMEM, s32) (+)= A (TMEM, u8) x B (shared, s8).
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Shared-memory matrix descriptor (version 1, base offset 0), K-major without
// swizzle: 8-row x 16-byte core matrices, `lbo` bytes apart along K, `sbo`
// bytes apart along M/N.
__device__ __forceinline__ uint64_t desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// kind::i8 instruction descriptor: s32 D, u8 A, s8 B, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_i8_m128(int n) {
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}
// 2-D tiled tensor copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

// As host_status_count of the mma.sync GEMV: y visible system-wide before
// the count; the last CTA returns the status word, then the call's sequence
// number.
__device__ __forceinline__ void tc8_status_count(const Tc8Args& a) {
  __threadfence_system();
  if (atomicAdd(a.fin_cnt, 1u) == gridDim.x - 1) {
    *a.fin_cnt = 0u;
    volatile uint32_t* hs = a.status_host;
    hs[0] = *reinterpret_cast<volatile uint32_t*>(a.status);
    const uint32_t seq = a.fin_cnt[1] + 1u;
    a.fin_cnt[1] = seq;
    __threadfence_system();
    hs[1] = seq;
  }
}

// x -> three int8 slices of super-block sb written into its x operand tile;
// lane holds elements 8*lane .. 8*lane+7 in v (sub-block j = lane / 4, bytes
// 8*(lane%4) .. of its 32).  Chunk c = j / 2 of the quants pairs lo quants
// with sub-block 2c and hi quants with 2c + 1:
//   K-step 0 (raw quants):    rows 0-2 = slices of 2c, rows 3-7 zero;
//   K-step 1 (16 hi quants):  rows 0-2 = -slices of 2c, rows 3-5 = slices
//                             of 2c + 1, rows 6-7 zero.
// Also the sub-block sums of x (sum32) and the super-block scale (sxs).
__device__ __forceinline__ void quantize_sb_tile(const float (&v)[8], int sb, int lane, uint8_t* bop, float* sum32,
                                                 float* sxs) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float inv = amax > 0.f ? 127.0f / amax : 0.f;
  uint32_t sl[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    part += v[i];
    const float q = v[i] * inv;
    const float q0 = rintf(q);
    const float u1 = (q - q0) * 254.0f;
    const float q1 = rintf(u1);
    const float q2 = rintf((u1 - q1) * 254.0f);
    const int sh = 8 * (i & 3);
    sl[0][i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q0)) & 0xFFu) << sh;
    sl[1][i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q1)) & 0xFFu) << sh;
    sl[2][i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q2)) & 0xFFu) << sh;
  }
  const int j = lane >> 2, c = j >> 1, h = (lane >> 1) & 1;
  uint8_t* t0 = bop + static_cast<size_t>(sb) * kBTile + c * 512 + h * 128 + 8 * (lane & 1);  // K-step 0, row 0
  uint8_t* t1 = t0 + 256;                                                                      // K-step 1, row 0
  const uint2 z = make_uint2(0u, 0u);
  if ((j & 1) == 0) {
#pragma unroll
    for (int n = 0; n < 3; ++n) {
      *reinterpret_cast<uint2*>(t0 + 16 * n) = make_uint2(sl[n][0], sl[n][1]);
      *reinterpret_cast<uint2*>(t1 + 16 * n) = make_uint2(__vsub4(0u, sl[n][0]), __vsub4(0u, sl[n][1]));
    }
#pragma unroll
    for (int n = 3; n < 8; ++n) *reinterpret_cast<uint2*>(t0 + 16 * n) = z;
  } else {
#pragma unroll
    for (int n = 0; n < 3; ++n) *reinterpret_cast<uint2*>(t1 + 16 * (3 + n)) = make_uint2(sl[n][0], sl[n][1]);
    *reinterpret_cast<uint2*>(t1 + 16 * 6) = z;
    *reinterpret_cast<uint2*>(t1 + 16 * 7) = z;
  }
  float p32 = part + __shfl_xor_sync(0xFFFFFFFFu, part, 1);
  p32 += __shfl_xor_sync(0xFFFFFFFFu, p32, 2);
  if ((lane & 3) == 0) sum32[sb * 8 + j] = p32;
  if (lane == 0) sxs[sb] = amax > 0.f ? amax / 127.0f : 0.f;
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    k_tc8_q4k(const Tc8Args a, const __grid_constant__ CUtensorMap wq, const __grid_constant__ CUtensorMap wh) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the swizzled stages need 1024-byte alignment: the launch asks for 1 KB more
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long row0 = static_cast<long long>(blockIdx.x) * a.rows_per_cta;
  const long long row_end = min(row0 + static_cast<long long>(a.rows_per_cta), a.rows);
  if (row0 >= row_end) {  // uniform across the CTA
    if (a.status_host && tid == 0) tc8_status_count(a);
    return;
  }
  const int NSB = a.NSB, TR = a.tile_rows;
  const int ntiles = static_cast<int>((row_end - row0 + TR - 1) / TR);
  const int K = ntiles * NSB;      // units: (tile, super-block), tile-major

  uint8_t* stg = smem;                       // [kNST][quants kRawStage | headers kHdrStage], 1024-aligned
  uint8_t* bop = smem + a.off_b;             // [NSB][kBTile], then kZeroBytes of zeros
  float* sum32 = reinterpret_cast<float*>(smem + a.off_sum32);
  float* sxs = reinterpret_cast<float*>(smem + a.off_scale);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* wempty = wfull + kNST;
  uint64_t* afull = wempty + kNST;  // [kNA] A operands of unit k in buffer k % kNA (maskers)
  uint64_t* dfree = afull + kNA;    // [2] accumulator buffer read back (readout)
  uint64_t* sbdone = dfree + 2;     // [4] MMAs of unit k complete (one commit per issuer)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sbdone + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  if (tid == 0) {
    for (int s = 0; s < kNST; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kReadWarps);
    }
    for (int s = 0; s < kNA; ++s) mbar_init(&afull[s], kMaskWarps);
    for (int s = 0; s < 2; ++s) mbar_init(&dfree[s], kReadWarps);
    for (int s = 0; s < 4; ++s) mbar_init(&sbdone[s], kIssuers);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kIssue0) {
    tc_alloc(tslot, kTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  auto fail = [&]() {
    *abort_flag = 1;
    atomicOr(a.status, kStatusCopyTimeout);
  };

  if (warp == kProducerW) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    const uint32_t tx = static_cast<uint32_t>(TR) * (128u + 16u);  // whole boxes, rows past the end included
    auto issue = [&](int k) {
      const int t = k / NSB, sb = k - t * NSB, ws = k % kNST;
      const int y = static_cast<int>(row0 + static_cast<long long>(t) * TR);
      uint8_t* dst = stg + static_cast<size_t>(ws) * kStage;
      mbar_arrive_expect_tx(&wfull[ws], tx);
      tma_2d(dst, &wq, sb * 144 + 16, y, &wfull[ws], pol);
      tma_2d(dst + kRawStage, &wh, sb * 144, y, &wfull[ws], pol);
    };
    // Weights are never written by an earlier kernel: the first PRE stages
    // stream before the grid dependency resolves, the rest once x is loaded.
    const int pre = min(min(a.PRE, kNST), K);
    if (lane == 0)
      for (int g = 0; g < pre; ++g) issue(g);
    grid_dep_wait();
    grid_dep_launch();
    if (a.PRE < kNST) named_bar_sync(2, 32 * (kPrepWarps + 1));
    if (lane == 0) {
      int issued = pre;
      for (int g = pre; g < K; ++g) {
        const int ws = g % kNST;
        if (g >= kNST && !mbar_wait_bounded(&wempty[ws], ((g / kNST) & 1) ^ 1, kWaitNs, abort_flag)) {
          fail();
          break;
        }
        issue(g);
        issued = g + 1;
      }
      // every copy issued lands before the CTA can exit
      for (int g = max(0, issued - kNST); g < issued; ++g)
        (void)mbar_wait_bounded(&wfull[g % kNST], (g / kNST) & 1, kWaitNs / 8, nullptr);
    }
    __syncwarp();
  } else if (warp < kRead0) {
    // ------------------------------------------------------------ maskers
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = 32 * q + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * q) << 16);
    const bool masked = warp - kMask0 >= 4;  // warps 5-8: the 16 hi operand
    for (int k = 0; k < K && !*abort_flag; ++k) {
      const int g = k, ws = g % kNST, ab = k % kNA;
      // the stage's quants have landed; the A buffer's previous unit
      // (k - kNA) has finished its MMAs
      bool ok = mbar_wait_bounded(&wfull[ws], (g / kNST) & 1, kWaitNs, abort_flag);
      if (ok && k >= kNA) ok = mbar_wait_bounded(&sbdone[k & 3], ((k >> 2) & 1) ^ 1, kWaitNs, abort_flag);
      if (!__all_sync(0xFFFFFFFFu, ok)) {
        if (lane == 0) fail();
        break;
      }
      // row r's 128 quant bytes in natural order: 16-byte chunk j of a
      // 128-byte-swizzled row lies at chunk j ^ (r % 8)
      const uint8_t* rowp = stg + static_cast<size_t>(ws) * kStage + r * 128;
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 c4 = *reinterpret_cast<const uint4*>(rowp + ((j ^ (r & 7)) << 4));
        w[4 * j] = c4.x; w[4 * j + 1] = c4.y; w[4 * j + 2] = c4.z; w[4 * j + 3] = c4.w;
      }
      if (masked) {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] &= 0xF0F0F0F0u;
      }
      tc_fence_after();
      tc_st32(tl + kTmemA + static_cast<uint32_t>(ab * 64 + (masked ? 32 : 0)), w);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ab]);
    }
  } else {
    // ------------------------------------------------------------ x tiles (readout and issuer warps)
    grid_dep_wait();
    {
      const int pw = warp - kRead0;
      float v[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {  // NSB <= 16 < 2 * kPrepWarps: every load in flight at once
        const int sb = pw + kPrepWarps * u;
        if (sb < NSB) {
          const float4* xp = reinterpret_cast<const float4*>(a.x + 256 * sb + 8 * lane);
          const float4 v0 = __ldg(xp), v1 = __ldg(xp + 1);
          v[u][0] = v0.x; v[u][1] = v0.y; v[u][2] = v0.z; v[u][3] = v0.w;
          v[u][4] = v1.x; v[u][5] = v1.y; v[u][6] = v1.z; v[u][7] = v1.w;
        }
      }
      if (a.PRE < kNST) {  // x is in registers: the producer may fill the ring
        float t = 0.f;
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (pw + kPrepWarps * u < NSB) t += v[u][0];
        asm volatile("" ::"f"(t));
        named_bar_arrive(2, 32 * (kPrepWarps + 1));
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int sb = pw + kPrepWarps * u;
        if (sb < NSB) quantize_sb_tile(v[u], sb, lane, bop, sum32, sxs);
      }
      if (pw == 0)
        *reinterpret_cast<uint2*>(bop + static_cast<size_t>(NSB) * kBTile + 8 * lane) = make_uint2(0u, 0u);
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 32 * kPrepWarps);
    if (warp < kIssue0) {
      // ---------------------------------------------------------- readout
      const int q = warp & 3;
      const int r = 32 * q + lane;
      const uint32_t tl = tbase + (static_cast<uint32_t>(32 * q) << 16);
      float acc = 0.f;
      for (int k = 0; k < K && !*abort_flag; ++k) {
        const int ws = k % kNST, db = k & 1;
        const int t = k / NSB, s = k - t * NSB;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&sbdone[k & 3], (k >> 2) & 1, kWaitNs, abort_flag))) {
          if (lane == 0) fail();
          break;
        }
        tc_fence_after();
        const uint4 h = *reinterpret_cast<const uint4*>(stg + static_cast<size_t>(ws) * kStage + kRawStage + r * 16);
        uint32_t v[64];  // accumulator m = 2c + (0 raw, 1 masked), columns 0-7
        const uint32_t d0 = tl + kTmemD + static_cast<uint32_t>(db * 16 * kIssuers);
        tc_ld4x8(d0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tc_ld4x8(d0 + 64u, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&dfree[db]);
          mbar_arrive(&wempty[ws]);
        }
        // get_scale_min_k4 of all eight sub-blocks (bytes: sc, m of sub-block j)
        const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
        int alo[3] = {0, 0, 0}, ahi[3] = {0, 0, 0};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t sw = c < 2 ? sc_lo : sc_hi;
          const int sa = static_cast<int>((sw >> (16 * (c & 1))) & 0xFFu);       // sub-block 2c
          const int sb = static_cast<int>((sw >> (16 * (c & 1) + 8)) & 0xFFu);   // sub-block 2c + 1
#pragma unroll
          for (int n = 0; n < 3; ++n) {
            alo[n] += sa * (static_cast<int>(v[16 * c + n]) + static_cast<int>(v[16 * c + 8 + n]));
            ahi[n] += sb * static_cast<int>(v[16 * c + 8 + 3 + n]);
          }
        }
        const float main = static_cast<float>(16 * alo[0] + ahi[0]) +
                           static_cast<float>(16 * alo[1] + ahi[1]) * (1.0f / 254.0f) +
                           static_cast<float>(16 * alo[2] + ahi[2]) * (1.0f / 64516.0f);
        float mg = 0.f;
        const float* ss = sum32 + s * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t mw = j < 4 ? m_lo : m_hi;
          mg = fmaf(static_cast<float>((mw >> (8 * (j & 3))) & 0xFFu), ss[j], mg);
        }
        const float d = f16_to_f32(h.x), dmin = f16_to_f32(h.x >> 16);
        acc += fmaf(d * (sxs[s] * (1.0f / 16.0f)), main, -dmin * mg);
        if (s == NSB - 1) {
          const long long row = row0 + static_cast<long long>(t) * TR + r;
          if (r < TR && row < row_end) a.y[row] = acc;
          acc = 0.f;
        }
      }
    } else if (lane == 0) {
      // ---------------------------------------------------------- MMA issuers
      const int i = warp - kIssue0, c = i >> 1, part = i & 1;  // part 0: raw quants, 1: 16 hi
      constexpr uint32_t idesc = idesc_i8_m128(16);
      const uint32_t b_a = smem_addr(bop);
      const uint32_t z_a = b_a + static_cast<uint32_t>(NSB * kBTile);
      int last = -1;
      for (int k = 0; k < K; ++k) {
        if (*abort_flag) break;
        const int ab = k % kNA, db = k & 1, s = k % NSB;
        if (!mbar_wait_bounded(&afull[ab], (k / kNA) & 1, kWaitNs, abort_flag) ||
            !mbar_wait_bounded(&dfree[db], ((k >> 1) & 1) ^ 1, kWaitNs, abort_flag)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t d = tbase + kTmemD + static_cast<uint32_t>(db * 16 * kIssuers + 16 * i);
        const uint32_t at = tbase + kTmemA + static_cast<uint32_t>(ab * 64 + 32 * part + 8 * c);
        const uint32_t bt = b_a + static_cast<uint32_t>(s * kBTile + c * 512 + part * 256);
        tc_mma_i8_ts(d, at, desc_plain(bt, 128u, z_a - bt), idesc, 0u);
        tc_commit(&sbdone[k & 3]);
        last = k;
      }
      // the tensor core is idle before the allocation is released
      if (last >= 0) (void)mbar_wait_bounded(&sbdone[last & 3], (last >> 2) & 1, kWaitNs, nullptr);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kIssue0) {
    tc_fence_after();
    tc_dealloc(tbase, kTmemCols);
  }
  if (a.status_host && tid == 0) tc8_status_count(a);
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tc8_encoder() {
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

bool plan_tc8(long long in_dim, long long rows, const uint8_t* w, const float* x, int sms, int smem_optin,
              Tc8Plan& p) {
  if (in_dim % 256 || in_dim / 256 > kMaxNSB || rows < 1 || rows > (1ll << 31) - 1 || sms < 1) return false;
  if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16) return false;
  const long long NSB = in_dim / 256;
  const long long rpc = (rows + sms - 1) / sms;
  const long long ntiles = (rpc + 127) / 128;
  const long long tr = (rpc + ntiles - 1) / ntiles;
  // shared memory: weight stages (1024-aligned for the 128-byte swizzle) |
  // x tiles and the zero block | x sums and scales | barriers
  long long off = static_cast<long long>(kNST) * kStage;
  p.a.off_hdr = 0;
  p.a.off_b = static_cast<int>(off);
  off += NSB * kBTile + kZeroBytes;
  p.a.off_xsl = 0;
  p.a.off_sum16 = 0;
  p.a.off_sum32 = static_cast<int>(off);
  off += NSB * 32;
  p.a.off_scale = static_cast<int>(off);
  off += (NSB * 4 + 15) / 16 * 16;
  p.a.off_bar = static_cast<int>(off);
  off += (2 * kNST + kNA + 6) * 8 + 16;
  p.smem = static_cast<size_t>(off + 1024);  // room to align the base to 1024 bytes
  if (static_cast<long long>(p.smem) > smem_optin) return false;
  p.a.rows = rows;
  p.a.NSB = static_cast<int>(NSB);
  p.a.tile_rows = static_cast<int>(tr);
  p.a.rows_per_cta = static_cast<int>(rpc);
  p.a.NSW = kNST;
  p.a.PRE = kNST;  // the caller may lower it (x first)
  p.grid = static_cast<int>((rows + rpc - 1) / rpc);
  p.RB = NSB * 144;
  return true;
}

cudaError_t launch_tc8(const Tc8Plan& p, const uint8_t* w, cudaStream_t st, bool pdl) {
  auto encode = tc8_encoder();
  if (!encode) return cudaErrorNotSupported;
  // quants: box 128 bytes x rows, 128-byte swizzle; headers: box 16 bytes x rows
  CUtensorMap wq, wh;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.RB), static_cast<cuuint64_t>(p.a.rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.RB)};
  const cuuint32_t boxq[2] = {128u, static_cast<cuuint32_t>(p.a.tile_rows)};
  const cuuint32_t boxh[2] = {16u, static_cast<cuuint32_t>(p.a.tile_rows)};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, boxq, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  if (encode(&wh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, boxh, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  {  // the shared-memory limit of the kernel, raised once per device
    constexpr int kMaxDev = 64;
    static int limit[kMaxDev] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
    if (static_cast<int>(p.smem) > limit[dev]) {
      e = cudaFuncSetAttribute(k_tc8_q4k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p.smem));
      if (e != cudaSuccess) return e;
      limit[dev] = static_cast<int>(p.smem);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid));
  cfg.blockDim = dim3(static_cast<unsigned>(kThreads));
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_tc8_q4k, p.a, wq, wh);
}

}  // namespace m3g
