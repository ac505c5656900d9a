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
// Units (tile, super-block) flow through NSW stages:
//   producer  warp 0: one 2-D tensor copy of the unit's quants (128-byte
//             rows, 128-byte swizzle) and one of its 16-byte block headers;
//   maskers   warps 1-8, one row per thread: warps 1-4 copy the row's 128
//             quant bytes into tensor memory as they are (the raw A operand),
//             warps 5-8 masked with 0xF0 (the 16 hi operand), into the A
//             buffer of the unit's stage;
//   issuers   warps 13-14: two chunks each, two MMAs per chunk (A in tensor
//             memory, B in shared memory; M = 128, N = 16, K = 32), one
//             commit per unit;
//   readout   warps 9-12, one row per thread: the four chunk accumulators
//             back from tensor memory, scales, d, dmin, the sum over
//             super-blocks, y.
// Before the units, warps 1-12 turn x into int8 slices and lay out the x
// operand tiles of every super-block once (shared memory, K <= 4096).
// Each stage has its own A buffer, so the maskers wait only for the stage's
// copy: the stage is refilled after the readout of the unit that last used
// it, which follows that unit's MMAs.  Every wait is bounded; a timeout
// raises the copy-timeout status bit and every role leaves its loop, so the
// CTA frees its tensor memory and exits.
//
// Off by default (tuning key tc8): measured on B200, one kind::i8 MMA with
// M = 128, K = 32 occupies the tensor core for ~200 SM clocks whatever N is
// (16 to 256) and wherever A lies (tensor or shared memory), and a unit needs
// eight of them, so the issuers bound a unit at ~560 ns.  The headline shape
// (14336 x 4096, 97 rows and 16 units per SM) then takes 15.4 us against
// 9.3 us for the mma.sync kernel: for one vector the tensor core's A intake
// (4 KB per MMA, two passes over the quants) is below the HBM rate.  The
// kernel stays as the tested tcgen05 formulation of the batch-1 product.
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
constexpr int kBTile = 4096;          // x operand of one super-block: 4 chunks x 2 K-steps x (16 rows x 32 bytes)
constexpr int kNSW = 6;               // stages (one tensor-memory A buffer each)
constexpr int kMaxNSB = 16;           // super-blocks whose x tiles fit shared memory (K <= 4096)
constexpr int kMaskWarps = 8, kReadWarps = 4, kIssuers = 2;
constexpr int kProducerW = 0, kMask0 = 1, kRead0 = kMask0 + kMaskWarps, kIssue0 = kRead0 + kReadWarps;
constexpr int kThreads = 32 * (kIssue0 + kIssuers);  // 480
// TMEM columns: A operands [kNSW][raw 32 | 16 hi 32] (4 int8 per column),
// then accumulators [2][4 chunks][16].
constexpr uint32_t kTmemA = 0, kTmemD = 64 * kNSW, kTmemCols = 512;
static_assert(kTmemD + 128 <= kTmemCols, "TMEM columns");
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

__device__ __forceinline__ void tc8_status_count(const Tc8Args& a) {
  __threadfence();
  if (atomicAdd(a.fin_cnt, 1u) == gridDim.x - 1) {
    *a.fin_cnt = 0u;
    *reinterpret_cast<volatile uint32_t*>(a.status_host) = *reinterpret_cast<volatile uint32_t*>(a.status);
  }
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
  constexpr int NSW = kNSW;
  const int ntiles = static_cast<int>((row_end - row0 + TR - 1) / TR);
  const int K = ntiles * NSB;  // units: (tile, super-block), tile-major

  uint8_t* raw = smem;                       // [NSW][kRawStage], 1024-aligned
  uint8_t* hdr = smem + a.off_hdr;           // [NSW][kHdrStage]
  uint8_t* bop = smem + a.off_b;             // [NSB][kBTile]
  uint8_t* xsl = smem + a.off_xsl;           // [NSB][8][3][32] int8
  float* sum32 = reinterpret_cast<float*>(smem + a.off_sum32);
  float* sum16 = reinterpret_cast<float*>(smem + a.off_sum16);
  float* sxs = reinterpret_cast<float*>(smem + a.off_scale);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* wempty = wfull + NSW;
  uint64_t* afull = wempty + NSW;   // [NSW] A operands of the stage's unit in tensor memory (maskers)
  uint64_t* dfree = afull + NSW;    // [2] accumulator buffer read back (readout)
  uint64_t* sbdone = dfree + 2;     // [4] MMAs of unit k complete (one commit per issuer)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sbdone + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  if (tid == 0) {
    for (int s = 0; s < NSW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kReadWarps);
      mbar_init(&afull[s], kMaskWarps);
    }
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
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      const uint32_t tx = static_cast<uint32_t>(TR) * (128u + 16u);
      auto issue = [&](int k) {
        const int t = k / NSB, s = k - t * NSB, ws = k % NSW;
        const int y = static_cast<int>(row0 + static_cast<long long>(t) * TR);
        mbar_arrive_expect_tx(&wfull[ws], tx);
        tma_2d(raw + static_cast<size_t>(ws) * kRawStage, &wq, s * 144 + 16, y, &wfull[ws], pol);
        tma_2d(hdr + static_cast<size_t>(ws) * kHdrStage, &wh, s * 144, y, &wfull[ws], pol);
      };
      // Weights are never written by an earlier kernel: the first stages
      // stream before the grid dependency resolves.
      const int pre = min(NSW, K);
      for (int k = 0; k < pre; ++k) issue(k);
      grid_dep_wait();
      grid_dep_launch();
      int issued = pre;
      for (int k = NSW; k < K; ++k) {
        const int ws = k % NSW;
        if (!mbar_wait_bounded(&wempty[ws], ((k / NSW) & 1) ^ 1, kWaitNs, abort_flag)) {
          fail();
          break;
        }
        issue(k);
        issued = k + 1;
      }
      // every copy issued lands before the CTA can exit
      for (int k = max(0, issued - NSW); k < issued; ++k)
        (void)mbar_wait_bounded(&wfull[k % NSW], (k / NSW) & 1, kWaitNs / 8, nullptr);
    }
    __syncwarp();
  } else if (warp < kIssue0) {
    // ------------------------------------------------------------ x slices and x tiles (warps 1-12)
    grid_dep_wait();
    {
      constexpr int kPrep = kMaskWarps + kReadWarps;
      const int pw = warp - kMask0;
      float v[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {  // NSB <= 16 < 2 * kPrep: every load in flight at once
        const int sb = pw + kPrep * u;
        if (sb < NSB) {
          const float4* xp = reinterpret_cast<const float4*>(a.x + 256 * sb + 8 * lane);
          const float4 v0 = __ldg(xp), v1 = __ldg(xp + 1);
          v[u][0] = v0.x; v[u][1] = v0.y; v[u][2] = v0.z; v[u][3] = v0.w;
          v[u][4] = v1.x; v[u][5] = v1.y; v[u][6] = v1.z; v[u][7] = v1.w;
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int sb = pw + kPrep * u;
        if (sb < NSB) quantize_sb(v[u], sb, lane, xsl, sum32, sum16, sxs);
      }
    }
    named_bar_sync(1, 32 * (kMaskWarps + kReadWarps));
    // x tiles of every super-block, 16-byte pieces of K-major core matrices
    // (8 rows x 16 bytes; the two K halves 128 bytes apart, row groups 256):
    // chunk c, K-step 0 rows 0-2 = x_lo slices (against the raw quants),
    // K-step 1 rows 0-2 = -x_lo and rows 3-5 = x_hi slices (against 16 hi);
    // every other row zero.
    for (int pc = tid - 32 * kMask0; pc < NSB * (kBTile / 16); pc += 32 * (kMaskWarps + kReadWarps)) {
      const int sb = pc / (kBTile / 16), off = (pc % (kBTile / 16)) * 16;
      const int c = off / 1024, ks = (off % 1024) / 512, rg = (off % 512) / 256, h = (off % 256) / 128;
      const int n = rg * 8 + (off % 128) / 16;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      const bool lo = n < 3, hi = ks == 1 && n >= 3 && n < 6;
      if (lo || hi) {
        const int j = hi ? 2 * c + 1 : 2 * c, sl = hi ? n - 3 : n;
        v = *reinterpret_cast<const uint4*>(xsl + (static_cast<size_t>(sb) * 8 + j) * 96 + sl * 32 + 16 * h);
        if (ks == 1 && lo) v = make_uint4(__vsub4(0u, v.x), __vsub4(0u, v.y), __vsub4(0u, v.z), __vsub4(0u, v.w));
      }
      *reinterpret_cast<uint4*>(bop + static_cast<size_t>(pc) * 16) = v;
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 32 * (kMaskWarps + kReadWarps));
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = 32 * q + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * q) << 16);
    if (warp < kRead0) {
      // ---------------------------------------------------------- maskers
      const bool masked = warp - kMask0 >= 4;  // warps 5-8: the 16 hi operand
      for (int k = 0; k < K && !*abort_flag; ++k) {
        const int ws = k % NSW;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&wfull[ws], (k / NSW) & 1, kWaitNs, abort_flag));
        if (!ok) {
          if (lane == 0) fail();
          break;
        }
        // row r's 128 quant bytes in natural order: 16-byte chunk j of a
        // 128-byte-swizzled row lies at chunk j ^ (r % 8)
        const uint8_t* rowp = raw + static_cast<size_t>(ws) * kRawStage + r * 128;
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
        tc_st32(tl + kTmemA + static_cast<uint32_t>(ws * 64 + (masked ? 32 : 0)), w);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ws]);
      }
    } else {
      // ---------------------------------------------------------- readout
      float acc = 0.f;
      for (int k = 0; k < K && !*abort_flag; ++k) {
        const int ws = k % NSW, db = k & 1;
        const int t = k / NSB, s = k - t * NSB;
        if (!mbar_wait_bounded(&sbdone[k & 3], (k >> 2) & 1, kWaitNs, abort_flag)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint4 h = *reinterpret_cast<const uint4*>(hdr + static_cast<size_t>(ws) * kHdrStage + r * 16);
        uint32_t v[32];
        tc_ld4x8(tl + kTmemD + static_cast<uint32_t>(db * 64), v);
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
            alo[n] += sa * static_cast<int>(v[8 * c + n]);
            ahi[n] += sb * static_cast<int>(v[8 * c + 3 + n]);
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
    }
  } else {
    // ------------------------------------------------------------ MMA issuers
    const int ci = warp - kIssue0;
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8_m128(16);
      const uint32_t b_a = smem_addr(bop);
      int last = -1;
      for (int k = 0; k < K; ++k) {
        if (*abort_flag) break;
        const int ws = k % NSW, db = k & 1, s = k % NSB;
        if (!mbar_wait_bounded(&afull[ws], (k / NSW) & 1, kWaitNs, abort_flag) ||
            !mbar_wait_bounded(&dfree[db], ((k >> 1) & 1) ^ 1, kWaitNs, abort_flag)) {
          fail();
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * ci + cc;
          const uint32_t d = tbase + kTmemD + static_cast<uint32_t>(db * 64 + c * 16);
          const uint32_t at = tbase + kTmemA + static_cast<uint32_t>(ws * 64 + 8 * c);
          const uint32_t bt = b_a + static_cast<uint32_t>(s * kBTile + c * 1024);
          tc_mma_i8_ts(d, at, desc_plain(bt, 128u, 256u), idesc, 0u);
          tc_mma_i8_ts(d, at + 32u, desc_plain(bt + 512u, 128u, 256u), idesc, 1u);
        }
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
  // shared memory: quant stages (1024-aligned for the 128-byte swizzle) |
  // header stages | x tiles | x slices and sums | barriers
  long long off = static_cast<long long>(kNSW) * kRawStage;
  p.a.off_hdr = static_cast<int>(off);
  off += static_cast<long long>(kNSW) * kHdrStage;
  p.a.off_b = static_cast<int>(off);
  off += NSB * kBTile;
  p.a.off_xsl = static_cast<int>(off);
  off += (NSB * 768 + 127) / 128 * 128;
  p.a.off_sum32 = static_cast<int>(off);
  off += NSB * 32;
  p.a.off_sum16 = static_cast<int>(off);
  off += NSB * 64;
  p.a.off_scale = static_cast<int>(off);
  off += (NSB * 4 + 15) / 16 * 16;
  p.a.off_bar = static_cast<int>(off);
  off += (3 * kNSW + 6) * 8 + 16;
  p.smem = static_cast<size_t>(off + 1024);  // room to align the base to 1024 bytes
  if (static_cast<long long>(p.smem) > smem_optin) return false;
  p.a.rows = rows;
  p.a.NSB = static_cast<int>(NSB);
  p.a.tile_rows = static_cast<int>(tr);
  p.a.rows_per_cta = static_cast<int>(rpc);
  p.a.NSW = kNSW;
  p.a.PRE = kNSW;
  p.grid = static_cast<int>((rows + rpc - 1) / rpc);
  p.RB = NSB * 144;
  return true;
}

cudaError_t launch_tc8(const Tc8Plan& p, const uint8_t* w, cudaStream_t st, bool pdl) {
  auto encode = tc8_encoder();
  if (!encode) return cudaErrorNotSupported;
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
