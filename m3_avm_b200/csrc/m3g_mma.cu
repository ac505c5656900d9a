// m3g_mma.cu -- the HBM-rate GEMV: GGUF quants as exact int8 tensor-core operands.
//
// Why: decoding a 4-bit weight to fp32 and FMA-ing it costs ~4 instructions
// per weight, which caps a CUDA-core GEMV far below the HBM roofline.  Here
// the quants stay integers and the dot products run on the tensor cores:
//
//   x is split once per CTA into three int8 slices per 256-element super-block
//   sb, x ~= s_sb * (x0 + x1/254 + x2/254^2), s_sb = max|x_sb| / 127, which
//   represents x to within 6.1e-8 * max|x_sb| (the third slice's rounding).
//   Each MMA (mma.sync m16n8k32 / m16n8k16, 8-bit integer -> s32) multiplies
//   16 rows of quants by the 3 slices (columns 0..2 of the n8 tile) exactly;
//   the 6-bit / int8 block scales of Q4_K / Q6_K are applied in integer, and
//   d, dmin, s_sb, the Q8_0/Q4_0 block scales and every min/bias term in fp32.
//
// Data flow per CTA (one per SM): a producer warp streams 16-row tiles of
// weight bytes into a ring of shared-memory stages with 1-D TMA bulk copies
// (one per row, into rows padded so the fragment loads are conflict-free),
// completing on mbarriers; eight consumer warps split each tile's
// super-blocks, build the A fragments from the staged bytes with a few LOPs
// per word, and keep per-row fp32 partials; the producer adds the warps'
// partials into y.
#include <cstdint>
#include <cuda_runtime.h>

#include "m3g_device.cuh"
#include "m3g_internal.h"

namespace m3g {

constexpr uint64_t kMmaTimeoutNs = 2000000000ull;
constexpr int kConsumerWarps = 8;

__device__ __forceinline__ void mma_k32_u8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_k32_s8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_k16_u8s8(uint32_t a0, uint32_t a1, uint32_t b0, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// A 32-bit word at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  return __funnelshift_r(b[0], b[1], static_cast<uint32_t>(a & 2u) * 8u);
}
// Two consecutive words at a 2-byte aligned address.
__device__ __forceinline__ uint2 lds64_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>(a & 2u) * 8u;
  const uint32_t w0 = b[0], w1 = b[1], w2 = b[2];
  return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

// Per-CTA prepared activation (shared memory).
struct XPrep {
  const uint8_t* sl;   // [K/32 sub-blocks][3 slices][32] int8, natural element order
  const float* sum32;  // [K/32] fp32 sum of x over each 32-element sub-block
  const float* sum16;  // [K/16] fp32 sum over each 16-element group
  const float* scale;  // [K/256] s_sb
};

// ---------------------------------------------------------------- Q4_K
// Super-block = one 144-byte block [d][dmin][scales 12][qs 128].  For chunk c
// of qs, quad thread t takes qs[32c + 8t .. +8] of its two rows; with the K
// order (4t..4t+3 -> bytes 8t..8t+3, 16+4t.. -> bytes 8t+4..8t+7) the low
// nibbles are the A fragment of sub-block 2c and the high nibbles (kept as
// 16*q in u8) that of sub-block 2c+1.  acc = 16 * sum_s sc_s sum_l q_l x_l.
struct MmaQ4K {
  static constexpr int kSBBytes = 144;

  __device__ static __forceinline__ void sc_words(const uint4& h, uint32_t& sc_lo, uint32_t& sc_hi, uint32_t& m_lo,
                                                  uint32_t& m_hi) {
    sc_lo = h.y & 0x3F3F3F3Fu;                                            // j < 4: q[j] & 63
    m_lo = h.z & 0x3F3F3F3Fu;                                             // j < 4: q[j+4] & 63
    sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);             // j >= 4
    m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  }

  __device__ static __forceinline__ void tile(const uint8_t* rg, const uint8_t* rg8, int sbg, const XPrep& xp, int g,
                                              int t, float w0, float w1, float& pg, float& pg8) {
    const uint4 hg = *reinterpret_cast<const uint4*>(rg);
    const uint4 hg8 = *reinterpret_cast<const uint4*>(rg8);
    uint32_t scl, sch, ml, mh, scl8, sch8, ml8, mh8;
    sc_words(hg, scl, sch, ml, mh);
    sc_words(hg8, scl8, sch8, ml8, mh8);
    int acc[4] = {0, 0, 0, 0};
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 8 * t;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint2 q = lds64(rg + 16 + 32 * c + 8 * t);
      const uint2 q8 = lds64(rg8 + 16 + 32 * c + 8 * t);
      uint2 blo = make_uint2(0u, 0u), bhi = make_uint2(0u, 0u);
      if (g < 3) {
        blo = lds64(xsl + (2 * c) * 96);
        bhi = lds64(xsl + (2 * c + 1) * 96);
      }
      int dlo[4], dhi[4];
      mma_k32_u8s8(q.x & 0x0F0F0F0Fu, q8.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q8.y & 0x0F0F0F0Fu, blo.x, blo.y, dlo);
      mma_k32_u8s8(q.x & 0xF0F0F0F0u, q8.x & 0xF0F0F0F0u, q.y & 0xF0F0F0F0u, q8.y & 0xF0F0F0F0u, bhi.x, bhi.y, dhi);
      const uint32_t w = c < 2 ? scl : sch, w8 = c < 2 ? scl8 : sch8;
      const int sh = (c & 1) * 16;
      const int sa = static_cast<int>((w >> sh) & 0xFFu) * 16, sb = static_cast<int>((w >> (sh + 8)) & 0xFFu);
      const int sa8 = static_cast<int>((w8 >> sh) & 0xFFu) * 16, sb8 = static_cast<int>((w8 >> (sh + 8)) & 0xFFu);
      acc[0] += sa * dlo[0] + sb * dhi[0];
      acc[1] += sa * dlo[1] + sb * dhi[1];
      acc[2] += sa8 * dlo[2] + sb8 * dhi[2];
      acc[3] += sa8 * dlo[3] + sb8 * dhi[3];
    }
    const float sx = xp.scale[sbg] * (1.0f / 16.0f);
    const float d = f16_to_f32(hg.x), dmin = f16_to_f32(hg.x >> 16);
    const float d8 = f16_to_f32(hg8.x), dmin8 = f16_to_f32(hg8.x >> 16);
    // min term over this thread's sub-blocks j = 2t, 2t+1: dmin * sum_j m_j * sum(x_j)
    const uint32_t mw = t < 2 ? ml : mh, mw8 = t < 2 ? ml8 : mh8;
    const int shm = (t & 1) * 16;
    const float xa = xp.sum32[sbg * 8 + 2 * t], xb = xp.sum32[sbg * 8 + 2 * t + 1];
    const float mg = static_cast<float>((mw >> shm) & 0xFFu) * xa + static_cast<float>((mw >> (shm + 8)) & 0xFFu) * xb;
    const float mg8 =
        static_cast<float>((mw8 >> shm) & 0xFFu) * xa + static_cast<float>((mw8 >> (shm + 8)) & 0xFFu) * xb;
    const float main = static_cast<float>(acc[0]) * w0 + static_cast<float>(acc[1]) * w1;
    const float main8 = static_cast<float>(acc[2]) * w0 + static_cast<float>(acc[3]) * w1;
    pg += fmaf(d * sx, main, -dmin * mg);
    pg8 += fmaf(d8 * sx, main8, -dmin8 * mg8);
  }
};

// ---------------------------------------------------------------- Q6_K
// Super-block = one 210-byte block [ql 128][qh 64][scales 16 x i8][d].  The
// 16-element group (n, k, h) (elements 128n + 32k + 16h + i) is one m16n8k16
// MMA; thread t holds its elements 4t..4t+3 built from
// ql[64n + 32(k&1) + 16h + 4t] (low nibble for k < 2, high for k >= 2) and
// qh[32n + 16h + 4t] bits 2k..2k+1, as unsigned 0..63.  The -32 offset is
// applied in fp32 through the group sums of x:
//   sum_l d s (q_l - 32) x_l = d * [ s * sum_l q_l x_l - 32 s * sum_l x_l ].
struct MmaQ6K {
  static constexpr int kSBBytes = 210;

  __device__ static __forceinline__ void tile(const uint8_t* rg, const uint8_t* rg8, int sbg, const XPrep& xp, int g,
                                              int t, float w0, float w1, float& pg, float& pg8) {
    int acc[4] = {0, 0, 0, 0};
    float bias = 0.f, bias8 = 0.f;
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 4 * t;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      // int8 scales s[8n .. 8n+8) of both rows
      const uint2 s = lds64_a2(rg + 192 + 8 * n);
      const uint2 s8 = lds64_a2(rg8 + 192 + 8 * n);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t A = lds32_a2(rg + 64 * n + 16 * h + 4 * t);
        const uint32_t B = lds32_a2(rg + 64 * n + 32 + 16 * h + 4 * t);
        const uint32_t C = lds32_a2(rg + 128 + 32 * n + 16 * h + 4 * t);
        const uint32_t A8 = lds32_a2(rg8 + 64 * n + 16 * h + 4 * t);
        const uint32_t B8 = lds32_a2(rg8 + 64 * n + 32 + 16 * h + 4 * t);
        const uint32_t C8 = lds32_a2(rg8 + 128 + 32 * n + 16 * h + 4 * t);
        uint32_t q[4], q8[4];
        q[0] = (A & 0x0F0F0F0Fu) | ((C << 4) & 0x30303030u);
        q[1] = (B & 0x0F0F0F0Fu) | ((C << 2) & 0x30303030u);
        q[2] = ((A >> 4) & 0x0F0F0F0Fu) | (C & 0x30303030u);
        q[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((C >> 2) & 0x30303030u);
        q8[0] = (A8 & 0x0F0F0F0Fu) | ((C8 << 4) & 0x30303030u);
        q8[1] = (B8 & 0x0F0F0F0Fu) | ((C8 << 2) & 0x30303030u);
        q8[2] = ((A8 >> 4) & 0x0F0F0F0Fu) | (C8 & 0x30303030u);
        q8[3] = ((B8 >> 4) & 0x0F0F0F0Fu) | ((C8 >> 2) & 0x30303030u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // group elements 128n + 32k + 16h .. : sub-block 4n + k, half h
          const uint32_t b = g < 3 ? lds32(xsl + (4 * n + k) * 96 + 16 * h) : 0u;
          int dd[4];
          mma_k16_u8s8(q[k], q8[k], b, dd);
          // scale index 8n + h + 2k: byte (h + 2k) of the pair of words s
          const int si = h + 2 * k;
          const uint32_t sw = si < 4 ? s.x : s.y, sw8 = si < 4 ? s8.x : s8.y;
          const int sc = static_cast<int>(static_cast<int8_t>((sw >> (8 * (si & 3))) & 0xFFu));
          const int sc8 = static_cast<int>(static_cast<int8_t>((sw8 >> (8 * (si & 3))) & 0xFFu));
          acc[0] += sc * dd[0];
          acc[1] += sc * dd[1];
          acc[2] += sc8 * dd[2];
          acc[3] += sc8 * dd[3];
          // this thread carries the bias of one group in four: (k == t)
          if (k == t) {
            const float xg = xp.sum16[sbg * 16 + 8 * n + 2 * k + h];
            bias = fmaf(static_cast<float>(sc), xg, bias);
            bias8 = fmaf(static_cast<float>(sc8), xg, bias8);
          }
        }
      }
    }
    const float sx = xp.scale[sbg];
    const float d = f16_to_f32(lds16(rg + 208)), d8 = f16_to_f32(lds16(rg8 + 208));
    const float main = static_cast<float>(acc[0]) * w0 + static_cast<float>(acc[1]) * w1;
    const float main8 = static_cast<float>(acc[2]) * w0 + static_cast<float>(acc[3]) * w1;
    pg += d * fmaf(sx, main, -32.0f * bias);
    pg8 += d8 * fmaf(sx, main8, -32.0f * bias8);
  }
};

// ---------------------------------------------------------------- Q8_0
// Super-block = 8 blocks of [d][32 x i8] (272 bytes).  Per block one k32 MMA
// with the K order of Q4_K (thread t: bytes 8t..8t+7 of the quants).
struct MmaQ80 {
  static constexpr int kSBBytes = 272;

  __device__ static __forceinline__ void tile(const uint8_t* rg, const uint8_t* rg8, int sbg, const XPrep& xp, int g,
                                              int t, float w0, float w1, float& pg, float& pg8) {
    float f = 0.f, f8 = 0.f;
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 8 * t;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint8_t* p = rg + 34 * b;
      const uint8_t* p8 = rg8 + 34 * b;
      const uint2 q = lds64_a2(p + 2 + 8 * t);
      const uint2 q8 = lds64_a2(p8 + 2 + 8 * t);
      const uint2 bx = g < 3 ? lds64(xsl + b * 96) : make_uint2(0u, 0u);
      int dd[4];
      mma_k32_s8s8(q.x, q8.x, q.y, q8.y, bx.x, bx.y, dd);
      const float d = f16_to_f32(lds16(p)), d8 = f16_to_f32(lds16(p8));
      f = fmaf(d, static_cast<float>(dd[0]) * w0 + static_cast<float>(dd[1]) * w1, f);
      f8 = fmaf(d8, static_cast<float>(dd[2]) * w0 + static_cast<float>(dd[3]) * w1, f8);
    }
    const float sx = xp.scale[sbg];
    pg = fmaf(sx, f, pg);
    pg8 = fmaf(sx, f8, pg8);
  }
};

// ---------------------------------------------------------------- Q4_0
// Super-block = 8 blocks of [d][16 bytes] (144 bytes).  Element i < 16 is the
// low nibble of qs[i], element 16 + i the high nibble, so with the natural K
// order thread t's A words are (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F) of
// qs[4t..4t+3].  The -8 offset is applied in fp32 through the block sums of x.
struct MmaQ40 {
  static constexpr int kSBBytes = 144;

  __device__ static __forceinline__ void tile(const uint8_t* rg, const uint8_t* rg8, int sbg, const XPrep& xp, int g,
                                              int t, float w0, float w1, float& pg, float& pg8) {
    float f = 0.f, f8 = 0.f, bias = 0.f, bias8 = 0.f;
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 4 * t;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint8_t* p = rg + 18 * b;
      const uint8_t* p8 = rg8 + 18 * b;
      const uint32_t q = lds32_a2(p + 2 + 4 * t);
      const uint32_t q8 = lds32_a2(p8 + 2 + 4 * t);
      uint32_t b0 = 0u, b1 = 0u;
      if (g < 3) {
        b0 = lds32(xsl + b * 96);
        b1 = lds32(xsl + b * 96 + 16);
      }
      int dd[4];
      mma_k32_u8s8(q & 0x0F0F0F0Fu, q8 & 0x0F0F0F0Fu, (q >> 4) & 0x0F0F0F0Fu, (q8 >> 4) & 0x0F0F0F0Fu, b0, b1, dd);
      const float d = f16_to_f32(lds16(p)), d8 = f16_to_f32(lds16(p8));
      f = fmaf(d, static_cast<float>(dd[0]) * w0 + static_cast<float>(dd[1]) * w1, f);
      f8 = fmaf(d8, static_cast<float>(dd[2]) * w0 + static_cast<float>(dd[3]) * w1, f8);
      if ((b & 3) == t) {  // this thread carries the bias of blocks t and t + 4
        const float xs = xp.sum32[sbg * 8 + b];
        bias = fmaf(d, xs, bias);
        bias8 = fmaf(d8, xs, bias8);
      }
    }
    const float sx = xp.scale[sbg];
    pg += fmaf(sx, f, -8.0f * bias);
    pg8 += fmaf(sx, f8, -8.0f * bias8);
  }
};

// ---------------------------------------------------------------- the kernel
template <class F>
__global__ void __launch_bounds__(32 * (kConsumerWarps + 1), 1) k_gemv_mma(const MmaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  const long long row0 = static_cast<long long>(blockIdx.x) * a.rows_per_cta;
  long long row_end = row0 + a.rows_per_cta;
  if (row_end > a.rows) row_end = a.rows;
  if (row0 >= row_end) return;  // uniform across the CTA
  const int nrows = static_cast<int>(row_end - row0);
  const int ntiles = (nrows + 15) >> 4;
  const int nst = ntiles * a.NKC;

  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [NS][16][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + a.NS);

  if (tid == 0) {
    for (int s = 0; s < a.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------ producer warp
    uint64_t policy = 0;
    if (lane == 0) policy = l2_evict_first_policy();
    policy = __shfl_sync(0xFFFFFFFFu, policy, 0);
    // Stage s = k-chunk (s % NKC) of 16-row tile (s / NKC); one bulk copy per row.
    auto issue = [&](int s) {
      const int tile = s / a.NKC, kc = s - tile * a.NKC;
      const int rows_t = min(16, nrows - 16 * tile);
      const int sb0 = kc * a.KC;
      const int seg = min(a.KC, a.NSB - sb0) * F::kSBBytes;
      const int b = s % a.NS;
      if (lane == 0) mbar_arrive_expect_tx(&full[b], static_cast<uint32_t>(rows_t * seg));
      __syncwarp();
      if (lane < rows_t) {
        const long long row = row0 + 16 * tile + lane;
        bulk_g2s(smem + static_cast<size_t>(b) * 16 * a.RS + static_cast<size_t>(lane) * a.RS,
                 a.w + row * a.RB + static_cast<long long>(sb0) * F::kSBBytes, static_cast<uint32_t>(seg), &full[b],
                 policy);
      }
    };
    // Weights are never written by an earlier kernel: their stream starts
    // before the grid dependency resolves.
    const int pre = min(a.NS, nst);
    for (int s = 0; s < pre; ++s) issue(s);
    grid_dep_wait();
    grid_dep_launch();
    int buf = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int s = 0; s < nst; ++s) {
      ok = mbar_wait_bounded(&empty[buf], ph, kMmaTimeoutNs, abort_flag);
      if (!ok) break;
      const int tile = s / a.NKC;
      if (s - tile * a.NKC == a.NKC - 1) {
        const int rows_t = min(16, nrows - 16 * tile);
        const float* rb = red + static_cast<size_t>(buf) * 16 * kConsumerWarps;
        if (lane < rows_t) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) acc += rb[lane * kConsumerWarps + w];
          a.y[row0 + 16 * tile + lane] = acc;
        }
      }
      __syncwarp();
      if (s + a.NS < nst) {
        if (lane == 0) fence_proxy_async_smem();
        issue(s + a.NS);
      }
      if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusCopyTimeout);
      // Let copies still in flight land (bounded) before the CTA exits.
      for (int s = 0; s < a.NS; ++s) (void)mbar_wait_bounded(&full[s], 0u, kMmaTimeoutNs / 8);
    }
    return;
  }

  // -------------------------------------------------- consumer warps
  const int cw = warp - 1;
  const int ctid = tid - 32;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* xsl = smem + a.off_xsl;
  float* sum32 = reinterpret_cast<float*>(smem + a.off_sum32);
  float* sum16 = reinterpret_cast<float*>(smem + a.off_sum16);
  float* sxs = reinterpret_cast<float*>(smem + a.off_scale);
  grid_dep_wait();
  // x -> per-super-block int8 slices and group sums (lane: 8 elements).
  for (int sb = cw; sb < a.NSB; sb += kConsumerWarps) {
    const float4* xp4 = reinterpret_cast<const float4*>(a.x + 256 * sb + 8 * lane);
    const float4 v0 = __ldg(xp4), v1 = __ldg(xp4 + 1);
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    uint32_t s0[2] = {0u, 0u}, s1[2] = {0u, 0u}, s2[2] = {0u, 0u};
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      part += v[i];
      const float u = v[i] * inv;
      const float q0 = rintf(u);
      const float u1 = (u - q0) * 254.0f;
      const float q1 = rintf(u1);
      const float q2 = rintf((u1 - q1) * 254.0f);
      const int sh = 8 * (i & 3);
      s0[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q0)) & 0xFFu) << sh;
      s1[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q1)) & 0xFFu) << sh;
      s2[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q2)) & 0xFFu) << sh;
    }
    // lane covers elements 8*lane .. +8: sub-block j = lane / 4, offset 8 * (lane % 4)
    uint8_t* dst = xsl + (static_cast<size_t>(sb) * 8 + (lane >> 2)) * 96 + 8 * (lane & 3);
    *reinterpret_cast<uint2*>(dst) = make_uint2(s0[0], s0[1]);
    *reinterpret_cast<uint2*>(dst + 32) = make_uint2(s1[0], s1[1]);
    *reinterpret_cast<uint2*>(dst + 64) = make_uint2(s2[0], s2[1]);
    float p16 = part + __shfl_xor_sync(0xFFFFFFFFu, part, 1);
    if ((lane & 1) == 0) sum16[sb * 16 + (lane >> 1)] = p16;
    const float p32 = p16 + __shfl_xor_sync(0xFFFFFFFFu, p16, 2);
    if ((lane & 3) == 0) sum32[sb * 8 + (lane >> 2)] = p32;
    if (lane == 0) sxs[sb] = amax > 0.f ? amax / 127.0f : 0.f;
  }
  named_bar_sync(1, 32 * kConsumerWarps);
  (void)ctid;

  const XPrep xp{xsl, sum32, sum16, sxs};
  // Column weights of this thread's two accumulator columns (2t, 2t+1):
  // column c carries slice c, weighted 254^-c; columns 3..7 are empty.
  const float w0 = t == 0 ? 1.0f : (t == 1 ? 1.0f / 64516.0f : 0.f);
  const float w1 = t == 0 ? 1.0f / 254.0f : 0.f;
  float pg = 0.f, pg8 = 0.f;
  int buf = 0, kc = 0, tile = 0;
  uint32_t ph = 0;
  for (int s = 0; s < nst; ++s) {
    const bool ok = mbar_wait_bounded(&full[buf], ph, kMmaTimeoutNs, abort_flag);
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        atomicOr(a.status, kStatusCopyTimeout);
      }
      return;
    }
    const uint8_t* st = smem + static_cast<size_t>(buf) * 16 * a.RS;
    const int sb0 = kc * a.KC;
    const int nsb = min(a.KC, a.NSB - sb0);
    const int j0 = cw * nsb / kConsumerWarps, j1 = (cw + 1) * nsb / kConsumerWarps;
    const uint8_t* rg = st + static_cast<size_t>(g) * a.RS;
    const uint8_t* rg8 = st + static_cast<size_t>(g + 8) * a.RS;
    for (int j = j0; j < j1; ++j)
      F::tile(rg + j * F::kSBBytes, rg8 + j * F::kSBBytes, sb0 + j, xp, g, t, w0, w1, pg, pg8);
    if (kc == a.NKC - 1) {
      pg += __shfl_xor_sync(0xFFFFFFFFu, pg, 1);
      pg += __shfl_xor_sync(0xFFFFFFFFu, pg, 2);
      pg8 += __shfl_xor_sync(0xFFFFFFFFu, pg8, 1);
      pg8 += __shfl_xor_sync(0xFFFFFFFFu, pg8, 2);
      if (t == 0) {
        float* rb = red + static_cast<size_t>(buf) * 16 * kConsumerWarps;
        rb[g * kConsumerWarps + cw] = pg;
        rb[(g + 8) * kConsumerWarps + cw] = pg8;
      }
      pg = pg8 = 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
    if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    if (++kc == a.NKC) { kc = 0; ++tile; }
  }
}

// ---------------------------------------------------------------- launcher
template <auto Kern>
static cudaError_t set_smem_once(size_t smem) {
  constexpr int kMaxDev = 64;
  static int limit[kMaxDev] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  if (static_cast<int>(smem) <= limit[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) limit[dev] = static_cast<int>(smem);
  return e;
}

template <auto Kern>
static cudaError_t launch_mma_kernel(const MmaArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl) {
  cudaError_t e = set_smem_once<Kern>(smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(32 * (kConsumerWarps + 1));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, Kern, a);
}

int mma_sb_bytes(int fmt) {
  switch (fmt) {
    case 12: return MmaQ4K::kSBBytes;
    case 14: return MmaQ6K::kSBBytes;
    case 8: return MmaQ80::kSBBytes;
    case 2: return MmaQ40::kSBBytes;
    default: return 0;
  }
}

cudaError_t launch_gemv_mma(int fmt, const MmaArgs& a, int grid, size_t smem, cudaStream_t st, bool pdl) {
  switch (fmt) {
    case 12: return launch_mma_kernel<k_gemv_mma<MmaQ4K>>(a, grid, smem, st, pdl);
    case 14: return launch_mma_kernel<k_gemv_mma<MmaQ6K>>(a, grid, smem, st, pdl);
    case 8: return launch_mma_kernel<k_gemv_mma<MmaQ80>>(a, grid, smem, st, pdl);
    case 2: return launch_mma_kernel<k_gemv_mma<MmaQ40>>(a, grid, smem, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m3g
