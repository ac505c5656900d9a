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

// Shared-memory loads addressed as (dynamic shared base, 32-bit byte offset):
// keeping offsets 32-bit lets the compiler fold them into shared addressing.
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* sm, uint32_t o) { return *reinterpret_cast<const uint2*>(sm + o); }
__device__ __forceinline__ uint4 lds128(const uint8_t* sm, uint32_t o) { return *reinterpret_cast<const uint4*>(sm + o); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* sm, uint32_t o) {
  return *reinterpret_cast<const uint16_t*>(sm + o);
}
// A 32-bit word at a 2-byte aligned offset (the base is 128-byte aligned).
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t* sm, uint32_t o) {
  const uint32_t* b = reinterpret_cast<const uint32_t*>(sm + (o & ~3u));
  return __funnelshift_r(b[0], b[1], (o & 2u) * 8u);
}
// Two consecutive words at a 2-byte aligned offset.
__device__ __forceinline__ uint2 lds64_a2(const uint8_t* sm, uint32_t o) {
  const uint32_t* b = reinterpret_cast<const uint32_t*>(sm + (o & ~3u));
  const uint32_t sh = (o & 2u) * 8u;
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

// Zero-extended / sign-extended byte K of w (one PRMT each).  The sign form
// uses prmt.b32 directly: __byte_perm ignores the selector's sign bit.
template <int K>
__device__ __forceinline__ int ubyte(uint32_t w) {
  return static_cast<int>(__byte_perm(w, 0u, 0x4440u + K));
}
template <int K>
__device__ __forceinline__ int sbyte(uint32_t w) {
  int r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "n"((8 + K) * 0x1110 + K));
  return r;
}

// ---------------------------------------------------------------- Q4_K
// Super-block = one 144-byte block [d][dmin][scales 12][qs 128].  For chunk c
// of qs, quad thread t takes qs[32c + 8t .. +8] of its two rows; with the K
// order (4t..4t+3 -> bytes 8t..8t+3, 16+4t.. -> bytes 8t+4..8t+7) the low
// nibbles are the A fragment of sub-block 2c and the high nibbles (kept as
// 16*q in u8) that of sub-block 2c+1.  acc = 16 * sum_s sc_s sum_l q_l x_l.
struct MmaQ4K {
  static constexpr int kSBBytes = 144;

  // x operands of one super-block for this thread: B fragments of its 8
  // sub-blocks, the sums of x over sub-blocks 2t and 2t+1, and s_sb / 16.
  struct XB {
    uint2 b[8];
    float xa, xb, sx;
  };

  __device__ static __forceinline__ void load_x(const XPrep& xp, int sbg, int g, int t, XB& o) {
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 8 * t;
#pragma unroll
    for (int s = 0; s < 8; ++s) o.b[s] = g < 3 ? lds64(xsl + s * 96) : make_uint2(0u, 0u);
    o.xa = xp.sum32[sbg * 8 + 2 * t];
    o.xb = xp.sum32[sbg * 8 + 2 * t + 1];
    o.sx = xp.scale[sbg] * (1.0f / 16.0f);
  }

  __device__ static __forceinline__ void sc_words(const uint4& h, uint32_t& sc_lo, uint32_t& sc_hi, uint32_t& m_lo,
                                                  uint32_t& m_hi) {
    sc_lo = h.y & 0x3F3F3F3Fu;                                            // j < 4: q[j] & 63
    m_lo = h.z & 0x3F3F3F3Fu;                                             // j < 4: q[j+4] & 63
    sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);             // j >= 4
    m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  }

  __device__ static __forceinline__ void tile(const uint8_t* sm, uint32_t rg, uint32_t rg8, const XB& xb, int t,
                                              float w0, float w1, float& pg, float& pg8) {
    const uint4 hg = lds128(sm, rg);
    const uint4 hg8 = lds128(sm, rg8);
    const uint32_t qo = rg + 16 + 8 * t, qo8 = rg8 + 16 + 8 * t;
    uint32_t scl, sch, ml, mh, scl8, sch8, ml8, mh8;
    sc_words(hg, scl, sch, ml, mh);
    sc_words(hg8, scl8, sch8, ml8, mh8);
    int alo[4] = {0, 0, 0, 0}, ahi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint2 q = lds64(sm, qo + 32 * c);
      const uint2 q8 = lds64(sm, qo8 + 32 * c);
      int dlo[4], dhi[4];
      mma_k32_u8s8(q.x & 0x0F0F0F0Fu, q8.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q8.y & 0x0F0F0F0Fu, xb.b[2 * c].x,
                   xb.b[2 * c].y, dlo);
      mma_k32_u8s8(q.x & 0xF0F0F0F0u, q8.x & 0xF0F0F0F0u, q.y & 0xF0F0F0F0u, q8.y & 0xF0F0F0F0u,
                   xb.b[2 * c + 1].x, xb.b[2 * c + 1].y, dhi);
      const uint32_t w = c < 2 ? scl : sch, w8 = c < 2 ? scl8 : sch8;
      int sa, sb, sa8, sb8;
      if (c & 1) {
        sa = ubyte<2>(w); sb = ubyte<3>(w); sa8 = ubyte<2>(w8); sb8 = ubyte<3>(w8);
      } else {
        sa = ubyte<0>(w); sb = ubyte<1>(w); sa8 = ubyte<0>(w8); sb8 = ubyte<1>(w8);
      }
      alo[0] += sa * dlo[0];
      alo[1] += sa * dlo[1];
      alo[2] += sa8 * dlo[2];
      alo[3] += sa8 * dlo[3];
      ahi[0] += sb * dhi[0];
      ahi[1] += sb * dhi[1];
      ahi[2] += sb8 * dhi[2];
      ahi[3] += sb8 * dhi[3];
    }
    const float d = f16_to_f32(hg.x), dmin = f16_to_f32(hg.x >> 16);
    const float d8 = f16_to_f32(hg8.x), dmin8 = f16_to_f32(hg8.x >> 16);
    // min term over this thread's sub-blocks j = 2t, 2t+1: dmin * sum_j m_j * sum(x_j)
    const uint32_t mw = t < 2 ? ml : mh, mw8 = t < 2 ? ml8 : mh8;
    const bool odd = t & 1;
    const float ma = static_cast<float>(odd ? ubyte<2>(mw) : ubyte<0>(mw));
    const float mb = static_cast<float>(odd ? ubyte<3>(mw) : ubyte<1>(mw));
    const float ma8 = static_cast<float>(odd ? ubyte<2>(mw8) : ubyte<0>(mw8));
    const float mb8 = static_cast<float>(odd ? ubyte<3>(mw8) : ubyte<1>(mw8));
    const float mg = fmaf(ma, xb.xa, mb * xb.xb);
    const float mg8 = fmaf(ma8, xb.xa, mb8 * xb.xb);
    const float main = static_cast<float>(16 * alo[0] + ahi[0]) * w0 + static_cast<float>(16 * alo[1] + ahi[1]) * w1;
    const float main8 = static_cast<float>(16 * alo[2] + ahi[2]) * w0 + static_cast<float>(16 * alo[3] + ahi[3]) * w1;
    pg += fmaf(d * xb.sx, main, -dmin * mg);
    pg8 += fmaf(d8 * xb.sx, main8, -dmin8 * mg8);
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

  // B fragments of the 16 groups (index 2 * (4n + k) + h) and the x sums of
  // the four groups whose bias this thread carries (k == t): index 2n + h.
  struct XB {
    uint32_t b[16];
    float xg[4];
    float sx;
  };

  __device__ static __forceinline__ void load_x(const XPrep& xp, int sbg, int g, int t, XB& o) {
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 4 * t;
#pragma unroll
    for (int sub = 0; sub < 8; ++sub)
#pragma unroll
      for (int h = 0; h < 2; ++h) o.b[2 * sub + h] = g < 3 ? lds32(xsl + sub * 96 + 16 * h) : 0u;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int h = 0; h < 2; ++h) o.xg[2 * n + h] = xp.sum16[sbg * 16 + 8 * n + 2 * t + h];
    o.sx = xp.scale[sbg];
  }

  template <int K>
  __device__ static __forceinline__ int scale_of(const uint2& s, int h) {
    // int8 scale 8n + h + 2K of a row: byte (h + 2K) of the two words s
    constexpr int lo = (2 * K) & 3;
    const uint32_t w = (2 * K) < 4 ? s.x : s.y;
    return h ? sbyte<lo + 1>(w) : sbyte<lo>(w);
  }

  __device__ static __forceinline__ void tile(const uint8_t* sm, uint32_t rg, uint32_t rg8, const XB& xb, int t,
                                              float w0, float w1, float& pg, float& pg8) {
    int acc[4] = {0, 0, 0, 0};
    float bias = 0.f, bias8 = 0.f;
    const uint32_t qo = rg + 4 * t, qo8 = rg8 + 4 * t;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const uint2 s = lds64_a2(sm, rg + 192 + 8 * n);
      const uint2 s8 = lds64_a2(sm, rg8 + 192 + 8 * n);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t A = lds32_a2(sm, qo + 64 * n + 16 * h);
        const uint32_t B = lds32_a2(sm, qo + 64 * n + 32 + 16 * h);
        const uint32_t C = lds32_a2(sm, qo + 128 + 32 * n + 16 * h);
        const uint32_t A8 = lds32_a2(sm, qo8 + 64 * n + 16 * h);
        const uint32_t B8 = lds32_a2(sm, qo8 + 64 * n + 32 + 16 * h);
        const uint32_t C8 = lds32_a2(sm, qo8 + 128 + 32 * n + 16 * h);
        uint32_t q[4], q8[4];
        q[0] = (A & 0x0F0F0F0Fu) | ((C << 4) & 0x30303030u);
        q[1] = (B & 0x0F0F0F0Fu) | ((C << 2) & 0x30303030u);
        q[2] = ((A >> 4) & 0x0F0F0F0Fu) | (C & 0x30303030u);
        q[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((C >> 2) & 0x30303030u);
        q8[0] = (A8 & 0x0F0F0F0Fu) | ((C8 << 4) & 0x30303030u);
        q8[1] = (B8 & 0x0F0F0F0Fu) | ((C8 << 2) & 0x30303030u);
        q8[2] = ((A8 >> 4) & 0x0F0F0F0Fu) | (C8 & 0x30303030u);
        q8[3] = ((B8 >> 4) & 0x0F0F0F0Fu) | ((C8 >> 2) & 0x30303030u);
        int sc[4], sc8[4];
        sc[0] = scale_of<0>(s, h); sc[1] = scale_of<1>(s, h); sc[2] = scale_of<2>(s, h); sc[3] = scale_of<3>(s, h);
        sc8[0] = scale_of<0>(s8, h); sc8[1] = scale_of<1>(s8, h); sc8[2] = scale_of<2>(s8, h);
        sc8[3] = scale_of<3>(s8, h);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          int dd[4];
          mma_k16_u8s8(q[k], q8[k], xb.b[2 * (4 * n + k) + h], dd);
          acc[0] += sc[k] * dd[0];
          acc[1] += sc[k] * dd[1];
          acc[2] += sc8[k] * dd[2];
          acc[3] += sc8[k] * dd[3];
        }
        // this thread carries the bias of group k == t
        const int st = t == 0 ? sc[0] : (t == 1 ? sc[1] : (t == 2 ? sc[2] : sc[3]));
        const int st8 = t == 0 ? sc8[0] : (t == 1 ? sc8[1] : (t == 2 ? sc8[2] : sc8[3]));
        bias = fmaf(static_cast<float>(st), xb.xg[2 * n + h], bias);
        bias8 = fmaf(static_cast<float>(st8), xb.xg[2 * n + h], bias8);
      }
    }
    const float d = f16_to_f32(lds16(sm, rg + 208)), d8 = f16_to_f32(lds16(sm, rg8 + 208));
    const float main = static_cast<float>(acc[0]) * w0 + static_cast<float>(acc[1]) * w1;
    const float main8 = static_cast<float>(acc[2]) * w0 + static_cast<float>(acc[3]) * w1;
    pg += d * fmaf(xb.sx, main, -32.0f * bias);
    pg8 += d8 * fmaf(xb.sx, main8, -32.0f * bias8);
  }
};

// ---------------------------------------------------------------- Q8_0
// Super-block = 8 blocks of [d][32 x i8] (272 bytes).  Per block one k32 MMA
// with the K order of Q4_K (thread t: bytes 8t..8t+7 of the quants).
struct MmaQ80 {
  static constexpr int kSBBytes = 272;

  struct XB {
    uint2 b[8];
    float sx;
  };

  __device__ static __forceinline__ void load_x(const XPrep& xp, int sbg, int g, int t, XB& o) {
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 8 * t;
#pragma unroll
    for (int b = 0; b < 8; ++b) o.b[b] = g < 3 ? lds64(xsl + b * 96) : make_uint2(0u, 0u);
    o.sx = xp.scale[sbg];
  }

  __device__ static __forceinline__ void tile(const uint8_t* sm, uint32_t rg, uint32_t rg8, const XB& xb, int t,
                                              float w0, float w1, float& pg, float& pg8) {
    float f = 0.f, f8 = 0.f;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t p = rg + 34 * b, p8 = rg8 + 34 * b;
      const uint2 q = lds64_a2(sm, p + 2 + 8 * t);
      const uint2 q8 = lds64_a2(sm, p8 + 2 + 8 * t);
      int dd[4];
      mma_k32_s8s8(q.x, q8.x, q.y, q8.y, xb.b[b].x, xb.b[b].y, dd);
      const float d = f16_to_f32(lds16(sm, p)), d8 = f16_to_f32(lds16(sm, p8));
      f = fmaf(d, static_cast<float>(dd[0]) * w0 + static_cast<float>(dd[1]) * w1, f);
      f8 = fmaf(d8, static_cast<float>(dd[2]) * w0 + static_cast<float>(dd[3]) * w1, f8);
    }
    pg = fmaf(xb.sx, f, pg);
    pg8 = fmaf(xb.sx, f8, pg8);
  }
};

// ---------------------------------------------------------------- Q4_0
// Super-block = 8 blocks of [d][16 bytes] (144 bytes).  Element i < 16 is the
// low nibble of qs[i], element 16 + i the high nibble, so with the natural K
// order thread t's A words are (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F) of
// qs[4t..4t+3].  The -8 offset is applied in fp32 through the block sums of x.
struct MmaQ40 {
  static constexpr int kSBBytes = 144;

  struct XB {
    uint32_t b0[8], b1[8];
    float xs[2];  // sums of x over blocks t and t + 4 (this thread carries their bias)
    float sx;
  };

  __device__ static __forceinline__ void load_x(const XPrep& xp, int sbg, int g, int t, XB& o) {
    const uint8_t* xsl = xp.sl + static_cast<size_t>(sbg) * 8 * 96 + g * 32 + 4 * t;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      o.b0[b] = g < 3 ? lds32(xsl + b * 96) : 0u;
      o.b1[b] = g < 3 ? lds32(xsl + b * 96 + 16) : 0u;
    }
    o.xs[0] = xp.sum32[sbg * 8 + t];
    o.xs[1] = xp.sum32[sbg * 8 + t + 4];
    o.sx = xp.scale[sbg];
  }

  __device__ static __forceinline__ void tile(const uint8_t* sm, uint32_t rg, uint32_t rg8, const XB& xb, int t,
                                              float w0, float w1, float& pg, float& pg8) {
    float f = 0.f, f8 = 0.f, bias = 0.f, bias8 = 0.f;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t p = rg + 18 * b, p8 = rg8 + 18 * b;
      const uint32_t q = lds32_a2(sm, p + 2 + 4 * t);
      const uint32_t q8 = lds32_a2(sm, p8 + 2 + 4 * t);
      int dd[4];
      mma_k32_u8s8(q & 0x0F0F0F0Fu, q8 & 0x0F0F0F0Fu, (q >> 4) & 0x0F0F0F0Fu, (q8 >> 4) & 0x0F0F0F0Fu, xb.b0[b],
                   xb.b1[b], dd);
      const float d = f16_to_f32(lds16(sm, p)), d8 = f16_to_f32(lds16(sm, p8));
      f = fmaf(d, static_cast<float>(dd[0]) * w0 + static_cast<float>(dd[1]) * w1, f);
      f8 = fmaf(d8, static_cast<float>(dd[2]) * w0 + static_cast<float>(dd[3]) * w1, f8);
      if ((b & 3) == t) {  // this thread carries the bias of blocks t and t + 4
        bias = fmaf(d, xb.xs[b >> 2], bias);
        bias8 = fmaf(d8, xb.xs[b >> 2], bias8);
      }
    }
    pg += fmaf(xb.sx, f, -8.0f * bias);
    pg8 += fmaf(xb.sx, f8, -8.0f * bias8);
  }
};

// (value, row) packed so that unsigned order is the greedy order: larger value
// first, then the lower row (the first index of the maximum).  The value maps
// to an order-preserving unsigned word; key 0 is below every finite value.
__device__ __forceinline__ unsigned long long argmax_key(float v, long long row) {
  const uint32_t u = v == 0.f ? 0u : __float_as_uint(v);  // -0 ties with +0
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(row));
}

// One CTA's arrival in a peer exchange (after its stores are fenced): the
// CTA completing this step's count pushes the local greedy key to the peers
// and signals each peer once.
// Slot of the greedy key this step uses (see MmaArgs::key_by_step).
__device__ __forceinline__ int key_slot(const MmaArgs& a) { return a.key_by_step ? (*a.step & 1) : 0; }

__device__ __forceinline__ void peer_arrive(const MmaArgs& a) {
  const unsigned int target = static_cast<unsigned int>(*a.step + 1) * gridDim.x;
  const unsigned int prev = atomicAdd(a.done_cnt, 1u);
  if (prev + 1u != target) return;
  __threadfence_system();
  if (a.argmax_key) {
    const int ks = key_slot(a);
    const unsigned long long k = atomicAdd(a.argmax_key + ks, 0ull);
    for (int p = 0; p < a.npeer; ++p)
      if (a.peer_key[p] && k) atomicMax_system(a.peer_key[p] + ks, k);
    __threadfence_system();
  }
  for (int p = 0; p < a.npeer; ++p) atomicAdd_system(a.peer_cnt[p], 1u);
}

// A CTA of a host-buffer call is done: its rows of y (mapped host memory)
// are made visible system-wide before it counts; the last CTA returns the
// status word and then the call's sequence number (fin_cnt[1] + 1) to the
// host, which waits for that number instead of synchronising the stream.
__device__ __forceinline__ void host_status_count(const MmaArgs& a) {
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

// Named barriers of the kernel (0 is __syncthreads): 1..WK pair the warps of
// two-tile stages (TPS > 1); the next id combines the norm's partial sums and
// the one after releases the producer once x is loaded.  Ids stay low: the
// highest id used sets the barriers a CTA reserves.
template <int TPS, int WK>
struct Bars {
  static constexpr int kRms = TPS > 1 ? WK + 1 : 1;
  static constexpr int kXLoaded = kRms + 1;
};

// ---------------------------------------------------------------- the kernel
// TPS 16-row tiles per stage; WK consumer warps per tile split its k-chunk of
// at most 16 super-blocks, so a warp owns at most 16 / WK of them.
// FUSED adds the decode-step features (input transforms, residual and argmax
// epilogues, x-first issue); the plain GEMV is compiled without them.
template <class F, int TPS, int WK, bool FUSED>
__global__ void __launch_bounds__(32 * (WK * TPS + 1), 1) k_gemv_mma(const MmaArgs a) {
  constexpr int NCW = WK * TPS;  // consumer warps
  constexpr int SR = 16 * TPS;   // rows per stage
  constexpr int MAXJ = 16 / WK;  // super-blocks per warp per stage
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  const long long row0 = static_cast<long long>(blockIdx.x) * a.rows_per_cta;
  long long row_end = row0 + a.rows_per_cta;
  if (row_end > a.rows) row_end = a.rows;
  if (row0 >= row_end) {  // uniform across the CTA; a peer-exchange CTA still counts
    if constexpr (FUSED) {
      if (a.npeer && threadIdx.x == 0) {
        grid_dep_wait();
        peer_arrive(a);
      }
    } else {
      if (a.status_host && threadIdx.x == 0) host_status_count(a);
    }
    return;
  }
  const int nrows = static_cast<int>(row_end - row0);
  const int ngroups = (nrows + SR - 1) / SR;
  const int nst = ngroups * a.NKC;
  // Row group of the s-th group visited.  With tail_first a partial last
  // group is visited first: its tile costs as much arithmetic as a full one
  // but little HBM time, so done early it hides behind the weight stream
  // instead of adding its arithmetic after the last bytes arrive.
  const bool tail_first = a.tail_first && ngroups > 1 && (nrows % SR) != 0;
  auto group_of = [&](int v) -> int { return tail_first ? (v == 0 ? ngroups - 1 : v - 1) : v; };

  float* red = reinterpret_cast<float*>(smem + a.off_red);  // [NS][SR][WK]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + a.NS);

  if (tid == 0) {
    for (int s = 0; s < a.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
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
    // Stage s = k-chunk (s % NKC) of row group (s / NKC): one bulk copy per
    // CG consecutive rows (whole rows when CG > 1, since then NKC == 1).
    const size_t stage_bytes = static_cast<size_t>(SR / a.CG) * a.GS;
    auto issue = [&](int s) {
      const int vis = s / a.NKC, kc = s - vis * a.NKC;
      const int grp = group_of(vis);
      const int rows_g = min(SR, nrows - SR * grp);
      const int sb0 = kc * a.KC;
      const int seg = min(a.KC, a.NSB - sb0) * F::kSBBytes;
      const int b = s % a.NS;
      if (lane == 0) mbar_arrive_expect_tx(&full[b], static_cast<uint32_t>(rows_g * seg));
      __syncwarp();
      const int ncopies = (rows_g + a.CG - 1) / a.CG;
      if (lane < ncopies) {
        const int rows_c = min(a.CG, rows_g - a.CG * lane);
        const long long row = row0 + SR * grp + a.CG * lane;
        bulk_g2s(smem + b * stage_bytes + static_cast<size_t>(lane) * a.GS,
                 a.w + row * a.RB + static_cast<long long>(sb0) * F::kSBBytes,
                 static_cast<uint32_t>(rows_c * seg), &full[b], policy);
      }
    };
    // Weights are never written by an earlier kernel: the first PRE stages
    // stream before the grid dependency resolves.  The rest wait for it, so
    // that the consumers' loads of x do not queue behind the whole ring.
    const int pre = min(min(a.PRE, a.NS), nst);
    for (int s = 0; s < pre; ++s) issue(s);
    grid_dep_wait();
    grid_dep_launch();
    // x first: with XFIRST the rest of the ring waits until the preparing
    // warps hold x in registers, so their L2 reads do not queue behind a
    // burst of weight misses.
    if constexpr (FUSED) {
      if (a.xfirst) named_bar_sync(Bars<TPS, WK>::kXLoaded, 32 * (WK + 1));
    }
    for (int s = pre; s < min(a.NS, nst); ++s) issue(s);
    int buf = 0;
    uint32_t ph = 0;
    bool ok = true;
    unsigned long long best_key = 0ull;  // argmax epilogue: this lane's best (value, row)
    // Peer stores go to the half of the exchange buffers this call's parity
    // selects (read after the grid dependency: an earlier kernel advances it).
    long long ypar = 0;
    if constexpr (FUSED) ypar = a.ystep ? static_cast<long long>(*a.ystep & 1) * a.ystride : 0;
    for (int s = 0; s < nst; ++s) {
      ok = mbar_wait_bounded(&empty[buf], ph, kMmaTimeoutNs, abort_flag);
      if (!ok) break;
      const int vis = s / a.NKC;
      if (s - vis * a.NKC == a.NKC - 1) {
        const int grp = group_of(vis);
        const int rows_g = min(SR, nrows - SR * grp);
        const float* rb = red + static_cast<size_t>(buf) * SR * WK;
        float acc = 0.f;
        if (lane < rows_g) {
#pragma unroll
          for (int w = 0; w < WK; ++w) acc += rb[lane * WK + w];
        }
        const long long r = row0 + SR * grp + lane;
        if constexpr (FUSED) {
          if (a.swiglu) {
            // Rows come in blocks of 8 gate rows then the 8 matching up rows
            // (every tile starts on a block boundary): h = silu(g) * u.
            const float u = __shfl_down_sync(0xFFFFFFFFu, acc, 8);
            if ((lane & 15) < 8 && lane < rows_g) {
              const long long o = (r >> 4) * 8 + (r & 7);
              const float h = __fmul_rn(__fdividef(acc, 1.0f + __expf(-acc)), u);
              a.y[o] = h;
              for (int p = 0; p < a.npeer; ++p)
                if (a.peer_y[p]) a.peer_y[p][o + ypar] = h;
            }
          } else if (lane < rows_g) {
            const float yv = a.res ? a.res[r] + acc : acc;
            a.y[r] = yv;
            for (int p = 0; p < a.npeer; ++p)
              if (a.peer_y[p]) a.peer_y[p][r + ypar] = yv;
            if (a.argmax_key && yv == yv) best_key = max(best_key, argmax_key(yv, r + a.key_row0));
          }
        } else if (lane < rows_g) {
          a.y[r] = acc;
        }
      }
      __syncwarp();
      if (s + a.NS < nst) {
        if (lane == 0) fence_proxy_async_smem();
        issue(s + a.NS);
      }
      if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    }
    if constexpr (FUSED) {
      if (a.argmax_key) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best_key = max(best_key, __shfl_xor_sync(0xFFFFFFFFu, best_key, o));
        if (lane == 0 && best_key) atomicMax(a.argmax_key + key_slot(a), best_key);
      }
      if (a.npeer) {  // this CTA's rows are in every peer's memory: count it
        __threadfence_system();
        __syncwarp();
        if (lane == 0) peer_arrive(a);
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusCopyTimeout);
      // Let copies still in flight land (bounded) before the CTA exits.
      for (int s = 0; s < a.NS; ++s) (void)mbar_wait_bounded(&full[s], 0u, kMmaTimeoutNs / 8);
    }
    if constexpr (!FUSED) {
      if (a.status_host) {
        __syncwarp();
        if (lane == 0) host_status_count(a);
      }
    }
    return;
  }

  // -------------------------------------------------- consumer warps
  const int cw = warp - 1;
  const int ti = cw / WK, wk = cw % WK;  // tile within the stage, k-split index
  const int g = lane >> 2, t = lane & 3;
  // Staged rows this thread's MMA rows g and g + 8 read.  With 4-row copy
  // groups, MMA rows g = 0..3 (one half-warp) come from four different
  // groups, whose 32-mod-128 stride puts their bytes in distinct banks.
  const int rr = a.CG == 4 ? (g & 3) * 4 + (g >> 2) : g;
  const int rr8 = a.CG == 4 ? (g & 3) * 4 + 2 + (g >> 2) : g + 8;
  const uint32_t off_g = static_cast<uint32_t>((rr / a.CG) * a.GS + (rr % a.CG) * a.SEG);
  const uint32_t off_g8 = static_cast<uint32_t>((rr8 / a.CG) * a.GS + (rr8 % a.CG) * a.SEG);
  const uint32_t stage_bytes = static_cast<uint32_t>((SR / a.CG) * a.GS);
  const uint32_t tile_bytes = static_cast<uint32_t>((16 / a.CG) * a.GS);
  uint8_t* xsl = smem + a.off_xsl;
  float* sum32 = reinterpret_cast<float*>(smem + a.off_sum32);
  float* sum16 = reinterpret_cast<float*>(smem + a.off_sum16);
  float* sxs = reinterpret_cast<float*>(smem + a.off_scale);
  // x -> per-super-block int8 slices and group sums (lane: 8 elements).  Each
  // warp prepares exactly the super-blocks it consumes (its share [j0, j1) of
  // every k-chunk), so it never waits for another warp; with two tiles per
  // stage the warp of tile 0 prepares and its tile-1 partner waits for it.
  if constexpr (!FUSED) {
    grid_dep_wait();
    // x -> per-super-block int8 slices and group sums (lane: 8 elements).  Each
    // warp prepares exactly the super-blocks it consumes (its share [j0, j1) of
    // every k-chunk), so it never waits for another warp; with two tiles per
    // stage the warp of tile 0 prepares and its tile-1 partner waits for it.
    // The loads of up to kXBatch super-blocks go out together, so a warp
    // with several (long rows: one per k-chunk) pays one L2 round trip per
    // batch instead of one per super-block.
    if (ti == 0 && a.NKC == 1) {  // one k-chunk: at most 16 / WK super-blocks, loaded one by one
      for (int sb = wk * a.NSB / WK; sb < (wk + 1) * a.NSB / WK; ++sb) {
        const float4* xp4 = reinterpret_cast<const float4*>(a.x + 256 * sb + 8 * lane);
        const float4 v0 = __ldg(xp4), v1 = __ldg(xp4 + 1);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        quantize_sb(v, sb, lane, xsl, sum32, sum16, sxs);
      }
    } else if (ti == 0) {
      constexpr int kXBatch = 4;
      int kcp = 0, sb = -1, sb_end = -1;  // the walk: [sb, sb_end) of k-chunk kcp
      auto advance = [&]() {
        while (sb >= sb_end && kcp < a.NKC) {
          const int sb0p = kcp * a.KC, nsbp = min(a.KC, a.NSB - sb0p);
          sb = sb0p + wk * nsbp / WK;
          sb_end = sb0p + (wk + 1) * nsbp / WK;
          ++kcp;
        }
      };
      advance();
      while (sb < sb_end) {
        float v[kXBatch][8];
        int sbs[kXBatch];
        int n = 0;
#pragma unroll
        for (int i = 0; i < kXBatch; ++i) {
          if (sb < sb_end) {
            const float4* xp4 = reinterpret_cast<const float4*>(a.x + 256 * sb + 8 * lane);
            const float4 v0 = __ldg(xp4), v1 = __ldg(xp4 + 1);
            v[i][0] = v0.x; v[i][1] = v0.y; v[i][2] = v0.z; v[i][3] = v0.w;
            v[i][4] = v1.x; v[i][5] = v1.y; v[i][6] = v1.z; v[i][7] = v1.w;
            sbs[i] = sb;
            n = i + 1;
            ++sb;
            advance();
          }
        }
#pragma unroll
        for (int i = 0; i < kXBatch; ++i)
          if (i < n) quantize_sb(v[i], sbs[i], lane, xsl, sum32, sum16, sxs);
      }
    }
  } else {
    if (ti == 0) {
      // This warp's super-blocks: its share [wk*n/WK, (wk+1)*n/WK) of every
      // k-chunk, visited in order; sb < 0 ends the walk.
      auto first_sb = [&](int kcp) -> int {
        for (; kcp < a.NKC; ++kcp) {
          const int sb0p = kcp * a.KC, nsbp = min(a.KC, a.NSB - sb0p);
          if (wk * nsbp / WK < (wk + 1) * nsbp / WK) return sb0p + wk * nsbp / WK;
        }
        return -1;
      };
      auto next_sb = [&](int sb) -> int {
        const int kcp = sb / a.KC, sb0p = kcp * a.KC, nsbp = min(a.KC, a.NSB - sb0p);
        return sb + 1 < sb0p + (wk + 1) * nsbp / WK ? sb + 1 : first_sb(kcp + 1);
      };
      auto load8 = [&](const float* base, int sb, float (&v)[8]) {
        const float4* p4 = reinterpret_cast<const float4*>(base + 256 * sb + 8 * lane);
        const float4 v0 = __ldg(p4), v1 = __ldg(p4 + 1);
        v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
        v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
      };
      // Transform (fused norm or SwiGLU), quantise into three int8 slices and
      // store the slices and group sums of super-block sb.
      auto prep = [&](int sb, float (&v)[8], const float (&gm)[8], const float (&u)[8], float inv_rms) {
        if (a.xmode == kXRmsNorm) {
          // rms_norm_into, x / rms * gamma, as x * (1 / rms) * gamma: within an
          // ulp of the reference per element
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv_rms), gm[i]);
        } else if (a.xmode == kXSiluMul) {
          // g * sigmoid(g) * up = g * up / (1 + exp(-g)), fast exponential and
          // division (relative error ~|g| * 2^-22); a huge 1 + exp(-g) divides
          // to 0, the limit of the sigmoid.
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fdividef(v[i], 1.0f + __expf(-v[i])), u[i]);
        }
        quantize_sb(v, sb, lane, xsl, sum32, sum16, sxs);
      };
      // The first two super-blocks of this warp stay in registers, so all of
      // their loads are in flight together: the norm weights (constant) before
      // the grid dependency resolves, x (and the up projection) right after.
      const int sbA = first_sb(0);
      const int sbB = sbA >= 0 ? next_sb(sbA) : -1;
      const int sbC = sbB >= 0 ? next_sb(sbB) : -1;  // further ones: one at a time
      float gA[8], gB[8], xA[8], xB[8], uA[8], uB[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) gA[i] = gB[i] = uA[i] = uB[i] = 1.f;
      if (a.xmode == kXRmsNorm && a.gamma) {
        if (sbA >= 0) load8(a.gamma, sbA, gA);
        if (sbB >= 0) load8(a.gamma, sbB, gB);
      }
      grid_dep_wait();
      grid_dep_launch();
      if (a.wait_cnt) {  // x holds other GPUs' rows: wait until every rank's CTAs have stored theirs
        if (lane == 0) {
          const unsigned int target = a.step ? static_cast<unsigned int>(*a.step + 1) * a.wait_mul : a.wait_mul;
          if (!wait_count_bounded(a.wait_cnt, target, a.peer_wait_ns)) atomicOr(a.status, kStatusPeerTimeout);
        }
        __syncwarp();
      }
      if (sbA >= 0) load8(a.x, sbA, xA);
      if (sbB >= 0) load8(a.x, sbB, xB);
      if (a.xmode == kXSiluMul) {
        if (sbA >= 0) load8(a.x2, sbA, uA);
        if (sbB >= 0) load8(a.x2, sbB, uB);
      }
      float inv_rms = 1.f;
      if (a.xmode == kXRmsNorm) {
        // Sum of squares: each warp over its own super-blocks, then the WK
        // preparing warps combine their partials in a fixed order through
        // shared memory, so every CTA derives the same rms.
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (sbA >= 0) ss = fmaf(xA[i], xA[i], ss);
          if (sbB >= 0) ss = fmaf(xB[i], xB[i], ss);
        }
        for (int sb = sbC; sb >= 0; sb = next_sb(sb)) {
          float v[8];
          load8(a.x, sb, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
        }
        ss = warp_sum(ss);
        float* part = reinterpret_cast<float*>(smem + a.off_red);  // free until the first tile ends
        if (lane == 0) part[wk] = ss;
        named_bar_sync(Bars<TPS, WK>::kRms, 32 * WK);
        float tot = 0.f;
        for (int w = 0; w < WK; ++w) tot += part[w];
        named_bar_sync(Bars<TPS, WK>::kRms, 32 * WK);
        inv_rms = __frcp_rn(__fsqrt_rn(__fdiv_rn(tot, static_cast<float>(256 * a.NSB)) + 1e-5f));
      }
      if (sbA >= 0) prep(sbA, xA, gA, uA, inv_rms);
      if (sbB >= 0) prep(sbB, xB, gB, uB, inv_rms);
      if (a.xfirst) named_bar_arrive(Bars<TPS, WK>::kXLoaded, 32 * (WK + 1));  // x, x2 of sbA, sbB are consumed
      for (int sb = sbC; sb >= 0; sb = next_sb(sb)) {
        float v[8], gm[8], u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) gm[i] = u[i] = 1.f;
        load8(a.x, sb, v);
        if (a.xmode == kXRmsNorm && a.gamma) load8(a.gamma, sb, gm);
        if (a.xmode == kXSiluMul) load8(a.x2, sb, u);
        prep(sb, v, gm, u, inv_rms);
      }
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  }
  if (TPS > 1) named_bar_sync(1 + wk, 64);  // warps wk (tile 0) and WK + wk (tile 1)
  __syncwarp();

  const XPrep xp{xsl, sum32, sum16, sxs};
  // Column weights of this thread's two accumulator columns (2t, 2t+1):
  // column c carries slice c, weighted 254^-c; columns 3..7 are empty.
  const float w0 = t == 0 ? 1.0f : (t == 1 ? 1.0f / 64516.0f : 0.f);
  const float w1 = t == 0 ? 1.0f / 254.0f : 0.f;
  float pg = 0.f, pg8 = 0.f;
  int buf = 0, kc = 0, loaded_kc = -1;
  uint32_t ph = 0;
  // x operands of this warp's (at most two) super-blocks of the current
  // k-chunk; with one k-chunk per row they are loaded once for the kernel.
  typename F::XB xb0, xb1;
  for (int s = 0; s < nst; ++s) {
    const bool ok = mbar_wait_bounded(&full[buf], ph, kMmaTimeoutNs, abort_flag);
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        atomicOr(a.status, kStatusCopyTimeout);
      }
      return;
    }
    const uint32_t st = static_cast<uint32_t>(buf) * stage_bytes + static_cast<uint32_t>(ti) * tile_bytes;
    const int sb0 = kc * a.KC;
    const int nsb = min(a.KC, a.NSB - sb0);
    const int j0 = wk * nsb / WK, j1 = (wk + 1) * nsb / WK;  // at most MAXJ (KC <= 16)
    if (kc != loaded_kc) {
      if (j0 < j1) F::load_x(xp, sb0 + j0, g, t, xb0);
      if (MAXJ > 1 && j0 + 1 < j1) F::load_x(xp, sb0 + j0 + 1, g, t, xb1);
      loaded_kc = kc;
    }
    const uint32_t rg = st + off_g + static_cast<uint32_t>(j0 * F::kSBBytes);
    const uint32_t rg8 = st + off_g8 + static_cast<uint32_t>(j0 * F::kSBBytes);
    if (j0 < j1) F::tile(smem, rg, rg8, xb0, t, w0, w1, pg, pg8);
    if (MAXJ > 1 && j0 + 1 < j1) F::tile(smem, rg + F::kSBBytes, rg8 + F::kSBBytes, xb1, t, w0, w1, pg, pg8);
    if (kc == a.NKC - 1) {
      pg += __shfl_xor_sync(0xFFFFFFFFu, pg, 1);
      pg += __shfl_xor_sync(0xFFFFFFFFu, pg, 2);
      pg8 += __shfl_xor_sync(0xFFFFFFFFu, pg8, 1);
      pg8 += __shfl_xor_sync(0xFFFFFFFFu, pg8, 2);
      if (t == 0) {
        float* rb = red + static_cast<size_t>(buf) * SR * WK;
        rb[(16 * ti + rr) * WK + wk] = pg;
        rb[(16 * ti + rr8) * WK + wk] = pg8;
      }
      pg = pg8 = 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
    if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    if (++kc == a.NKC) kc = 0;
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
static cudaError_t launch_mma_kernel(const MmaArgs& a, int grid, int threads, size_t smem, cudaStream_t st, bool pdl) {
  cudaError_t e = set_smem_once<Kern>(smem);
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

int mma_sb_bytes(int fmt) {
  switch (fmt) {
    case 12: return MmaQ4K::kSBBytes;
    case 14: return MmaQ6K::kSBBytes;
    case 8: return MmaQ80::kSBBytes;
    case 2: return MmaQ40::kSBBytes;
    default: return 0;
  }
}

template <class F, bool FUSED>
static cudaError_t launch_mma_cfg(const MmaArgs& a, int tps, int wk, int grid, size_t smem, cudaStream_t st,
                                  bool pdl) {
  if (wk == 16) return launch_mma_kernel<k_gemv_mma<F, 1, 16, FUSED>>(a, grid, 32 * 17, smem, st, pdl);
  if (tps == 2) return launch_mma_kernel<k_gemv_mma<F, 2, 8, FUSED>>(a, grid, 32 * 17, smem, st, pdl);
  return launch_mma_kernel<k_gemv_mma<F, 1, 8, FUSED>>(a, grid, 32 * 9, smem, st, pdl);
}

template <class F>
static cudaError_t launch_mma_fmt(const MmaArgs& a, int tps, int wk, int grid, size_t smem, cudaStream_t st,
                                  bool pdl) {
  const bool fused = a.xmode != kXPlain || a.res || a.argmax_key || a.xfirst || a.swiglu || a.npeer || a.wait_cnt;
  return fused ? launch_mma_cfg<F, true>(a, tps, wk, grid, smem, st, pdl)
               : launch_mma_cfg<F, false>(a, tps, wk, grid, smem, st, pdl);
}

cudaError_t launch_gemv_mma(int fmt, const MmaArgs& a, int tps, int wk, int grid, size_t smem, cudaStream_t st,
                            bool pdl) {
  switch (fmt) {
    case 12: return launch_mma_fmt<MmaQ4K>(a, tps, wk, grid, smem, st, pdl);
    case 14: return launch_mma_fmt<MmaQ6K>(a, tps, wk, grid, smem, st, pdl);
    case 8: return launch_mma_fmt<MmaQ80>(a, tps, wk, grid, smem, st, pdl);
    case 2: return launch_mma_fmt<MmaQ40>(a, tps, wk, grid, smem, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// ================================================================ batched GEMV, 8 columns per pass
//
// Y[b][r] = sum_k X[b][k] W[r][k] for up to 8 rows of X per launch (Q4_K).
// k_xprep8 quantises X once into one record per 256-element super-block: the
// three int8 slices of every column (the B = 1 kernel's representation), the
// 32-element group sums and the column scales.  k_gemm8_q4k walks the K
// chunks outermost: one TMA bulk copy brings a chunk's records into shared
// memory for all of the CTA's row tiles, the 8 consumer warps each take one
// super-block of the staged 16-row tile and run three m16n8k32 MMAs per
// sub-block (one per slice) with the 8 columns as N, and the producer adds
// the warps' partials into per-(row, column) sums in shared memory, writing Y
// after the last chunk.  Same integer math and fp32 epilogue as k_gemv_mma.
constexpr int kXB = 8;                                 // columns per pass
constexpr int kXRecSlices = 8 * 3 * kXB * 32;          // [sub-block j][slice][column][32]
constexpr int kXRecSum = kXRecSlices;                  // f32 [j][column]
constexpr int kXRecScale = kXRecSum + 8 * kXB * 4;     // f32 [column]
constexpr int kXRec = kXRecScale + kXB * 4;            // 6432 bytes per super-block

__global__ void __launch_bounds__(256) k_xprep8(const float* __restrict__ x, int cols, int in_dim,
                                                uint8_t* __restrict__ out) {
  const int sb = blockIdx.x, b = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (b < cols) {
    const float4* p4 = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * in_dim + 256 * sb + 8 * lane);
    const float4 v0 = __ldg(p4), v1 = __ldg(p4 + 1);
    v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
    v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
  }
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
    const float q = v[i] * inv;
    const float q0 = rintf(q);
    const float u1 = (q - q0) * 254.0f;
    const float q1 = rintf(u1);
    const float q2 = rintf((u1 - q1) * 254.0f);
    const int sh = 8 * (i & 3);
    s0[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q0)) & 0xFFu) << sh;
    s1[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q1)) & 0xFFu) << sh;
    s2[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(q2)) & 0xFFu) << sh;
  }
  uint8_t* rec = out + static_cast<size_t>(sb) * kXRec;
  const int j = lane >> 2;
  uint8_t* dst = rec + ((j * 3) * kXB + b) * 32 + 8 * (lane & 3);
  *reinterpret_cast<uint2*>(dst) = make_uint2(s0[0], s0[1]);
  *reinterpret_cast<uint2*>(dst + kXB * 32) = make_uint2(s1[0], s1[1]);
  *reinterpret_cast<uint2*>(dst + 2 * kXB * 32) = make_uint2(s2[0], s2[1]);
  float p32 = part + __shfl_xor_sync(0xFFFFFFFFu, part, 1);
  p32 += __shfl_xor_sync(0xFFFFFFFFu, p32, 2);
  if ((lane & 3) == 0) reinterpret_cast<float*>(rec + kXRecSum)[j * kXB + b] = p32;
  if (lane == 0) reinterpret_cast<float*>(rec + kXRecScale)[b] = amax > 0.f ? amax / 127.0f : 0.f;
}

static_assert(kXRec == kGemm8RecBytes, "prepared-x record size");
static_assert(kXB == kGemm8Cols, "columns per pass");

// One 16-row Q4_K super-block tile against 8 columns, the x operands read
// from the prepared record `rec` in shared memory as they are used: v[0],
// v[1] = row g and columns 2t, 2t+1; v[2], v[3] = row g + 8.
__device__ __forceinline__ void tile8_q4k(const uint8_t* sm, uint32_t rg, uint32_t rg8, uint32_t rec, int g,
                                          int t, float (&v)[4]) {
  const uint4 hg = lds128(sm, rg);
  const uint4 hg8 = lds128(sm, rg8);
  const uint32_t qo = rg + 16 + 8 * t, qo8 = rg8 + 16 + 8 * t;
  uint32_t scl, sch, ml, mh, scl8, sch8, ml8, mh8;
  MmaQ4K::sc_words(hg, scl, sch, ml, mh);
  MmaQ4K::sc_words(hg8, scl8, sch8, ml8, mh8);
  const uint32_t xb = rec + g * 32 + 8 * t;  // B fragment of (j, slice s): xb + (j * 3 + s) * kXB * 32
  int alo[3][4], ahi[3][4];
#pragma unroll
  for (int s = 0; s < 3; ++s)
#pragma unroll
    for (int i = 0; i < 4; ++i) alo[s][i] = ahi[s][i] = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint2 q = lds64(sm, qo + 32 * c);
    const uint2 q8 = lds64(sm, qo8 + 32 * c);
    const uint32_t w = c < 2 ? scl : sch, w8 = c < 2 ? scl8 : sch8;
    int sa, sb, sa8, sb8;
    if (c & 1) {
      sa = ubyte<2>(w); sb = ubyte<3>(w); sa8 = ubyte<2>(w8); sb8 = ubyte<3>(w8);
    } else {
      sa = ubyte<0>(w); sb = ubyte<1>(w); sa8 = ubyte<0>(w8); sb8 = ubyte<1>(w8);
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const uint2 blo = lds64(sm, xb + ((2 * c) * 3 + s) * kXB * 32);
      const uint2 bhi = lds64(sm, xb + ((2 * c + 1) * 3 + s) * kXB * 32);
      int dlo[4], dhi[4];
      mma_k32_u8s8(q.x & 0x0F0F0F0Fu, q8.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q8.y & 0x0F0F0F0Fu, blo.x, blo.y, dlo);
      mma_k32_u8s8(q.x & 0xF0F0F0F0u, q8.x & 0xF0F0F0F0u, q.y & 0xF0F0F0F0u, q8.y & 0xF0F0F0F0u, bhi.x, bhi.y, dhi);
      alo[s][0] += sa * dlo[0];
      alo[s][1] += sa * dlo[1];
      alo[s][2] += sa8 * dlo[2];
      alo[s][3] += sa8 * dlo[3];
      ahi[s][0] += sb * dhi[0];
      ahi[s][1] += sb * dhi[1];
      ahi[s][2] += sb8 * dhi[2];
      ahi[s][3] += sb8 * dhi[3];
    }
  }
  const float d = f16_to_f32(hg.x), dmin = f16_to_f32(hg.x >> 16);
  const float d8 = f16_to_f32(hg8.x), dmin8 = f16_to_f32(hg8.x >> 16);
  // min term dmin * sum_j m_j * sum(x_j), per row and column
  float mg[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t mw = j < 4 ? ml : mh, mw8 = j < 4 ? ml8 : mh8;
    const int k = j & 3;
    const float m = static_cast<float>((mw >> (8 * k)) & 0xFFu);
    const float m8 = static_cast<float>((mw8 >> (8 * k)) & 0xFFu);
    const float2 sj = *reinterpret_cast<const float2*>(sm + rec + kXRecSum + (j * kXB + 2 * t) * 4);
    mg[0] = fmaf(m, sj.x, mg[0]);
    mg[1] = fmaf(m, sj.y, mg[1]);
    mg[2] = fmaf(m8, sj.x, mg[2]);
    mg[3] = fmaf(m8, sj.y, mg[3]);
  }
  const float2 sc = *reinterpret_cast<const float2*>(sm + rec + kXRecScale + 2 * t * 4);
  const float sx0 = sc.x * (1.0f / 16.0f), sx1 = sc.y * (1.0f / 16.0f);
  float main[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    main[i] = static_cast<float>(16 * alo[0][i] + ahi[0][i]) +
              static_cast<float>(16 * alo[1][i] + ahi[1][i]) * (1.0f / 254.0f) +
              static_cast<float>(16 * alo[2][i] + ahi[2][i]) * (1.0f / 64516.0f);
  v[0] = fmaf(d * sx0, main[0], -dmin * mg[0]);
  v[1] = fmaf(d * sx1, main[1], -dmin * mg[1]);
  v[2] = fmaf(d8 * sx0, main[2], -dmin8 * mg[2]);
  v[3] = fmaf(d8 * sx1, main[3], -dmin8 * mg[3]);
}

// Block = 1 producer warp + 8 consumer warps; a stage holds TPS = 8 / KC
// row tiles of 16 rows x KC super-blocks, consumer warp w takes tile w / KC
// and super-block w % KC.  Sized for two CTAs per SM.
__global__ void __launch_bounds__(288, 2) k_gemm8_q4k(const Gemm8Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long row0 = static_cast<long long>(blockIdx.x) * a.rows_per_cta;
  long long row_end = row0 + a.rows_per_cta;
  if (row_end > a.rows) row_end = a.rows;
  if (row0 >= row_end) return;  // uniform across the CTA
  const int TPS = 8 / a.KC, SR = 16 * TPS;
  const int nrows = static_cast<int>(row_end - row0);
  const int ngroups = (nrows + SR - 1) / SR;
  const int nst = ngroups * a.NKC;  // stage s = (chunk s / ngroups, row group s % ngroups)
  const uint32_t XC = static_cast<uint32_t>(a.KC) * kXRec;
  const uint32_t stage_bytes = static_cast<uint32_t>(SR) * static_cast<uint32_t>(a.GS);
  const int red_stage = SR * kXB * a.KC;  // floats: [KC warps][SR rows][8 columns]
  float* red = reinterpret_cast<float*>(smem + a.off_red);
  float* acc = reinterpret_cast<float*>(smem + a.off_acc);  // [nrows][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  uint64_t* empty = full + a.NS;
  uint64_t* xfull = empty + a.NS;
  uint64_t* xempty = xfull + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xempty + 2);
  if (tid == 0) {
    for (int s = 0; s < a.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < nrows * kXB; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------ producer warp
    uint64_t policy = 0;
    if (lane == 0) policy = l2_evict_first_policy();
    policy = __shfl_sync(0xFFFFFFFFu, policy, 0);
    auto issue_x = [&](int kc) {
      const int nsb = min(a.KC, a.NSB - kc * a.KC);
      if (lane == 0) {
        mbar_arrive_expect_tx(&xfull[kc & 1], static_cast<uint32_t>(nsb * kXRec));
        bulk_g2s(smem + (kc & 1) * XC, a.xq + static_cast<size_t>(kc) * a.KC * kXRec,
                 static_cast<uint32_t>(nsb * kXRec), &xfull[kc & 1], 0ull);
      }
      __syncwarp();
    };
    auto issue = [&](int s) {
      const int kc = s / ngroups, grp = s - kc * ngroups;
      const int rows_g = min(SR, nrows - SR * grp);
      const int seg = min(a.KC, a.NSB - kc * a.KC) * MmaQ4K::kSBBytes;
      const int b = s % a.NS;
      if (lane == 0) mbar_arrive_expect_tx(&full[b], static_cast<uint32_t>(rows_g * seg));
      __syncwarp();
      for (int r = lane; r < rows_g; r += 32) {
        const long long row = row0 + SR * grp + r;
        bulk_g2s(smem + a.off_stage + b * stage_bytes + static_cast<size_t>(r) * a.GS,
                 a.w + row * a.RB + static_cast<long long>(kc) * a.KC * MmaQ4K::kSBBytes, static_cast<uint32_t>(seg),
                 &full[b], policy);
      }
    };
    issue_x(0);
    if (a.NKC > 1) issue_x(1);
    for (int s = 0; s < min(a.NS, nst); ++s) issue(s);
    int buf = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int s = 0; s < nst && ok; ++s) {
      ok = mbar_wait_bounded(&empty[buf], ph, kMmaTimeoutNs, abort_flag);
      if (!ok) break;
      const int kc = s / ngroups, grp = s - kc * ngroups;
      if (s + a.NS < nst) {
        if (lane == 0) fence_proxy_async_smem();
        issue(s + a.NS);
      }
      if (grp == ngroups - 1 && kc + 2 < a.NKC) {  // chunk kc fully consumed: its buffer takes chunk kc + 2
        ok = mbar_wait_bounded(&xempty[kc & 1], (kc >> 1) & 1, kMmaTimeoutNs, abort_flag);
        if (!ok) break;
        if (lane == 0) fence_proxy_async_smem();
        issue_x(kc + 2);
      }
      if (++buf == a.NS) { buf = 0; ph ^= 1u; }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusCopyTimeout);
      for (int s = 0; s < a.NS; ++s) (void)mbar_wait_bounded(&full[s], 0u, kMmaTimeoutNs / 8);
      for (int i = 0; i < 2; ++i) (void)mbar_wait_bounded(&xfull[i], 0u, kMmaTimeoutNs / 8);
    }
    return;
  }

  // -------------------------------------------------- consumer warps
  const int cw = warp - 1;
  const int ti = cw / a.KC, sbw = cw % a.KC;  // row tile of the stage, super-block of the chunk
  const int g = lane >> 2, t = lane & 3;
  const uint32_t off_g = static_cast<uint32_t>((16 * ti + g) * a.GS + sbw * MmaQ4K::kSBBytes);
  const uint32_t off_g8 = static_cast<uint32_t>((16 * ti + g + 8) * a.GS + sbw * MmaQ4K::kSBBytes);
  int buf = 0, loaded_kc = -1;
  uint32_t ph = 0;
  bool active = false;
  for (int s = 0; s < nst; ++s) {
    const int kc = s / ngroups;
    if (kc != loaded_kc) {
      if (loaded_kc >= 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&xempty[loaded_kc & 1]);
      }
      // A wait that gives up flags the CTA and the loop runs on without the
      // data, so every warp still reaches every named barrier below.
      if (!mbar_wait_bounded(&xfull[kc & 1], (kc >> 1) & 1, kMmaTimeoutNs, abort_flag) && lane == 0) {
        *abort_flag = 1;
        atomicOr(a.status, kStatusCopyTimeout);
      }
      active = sbw < min(a.KC, a.NSB - kc * a.KC);
      loaded_kc = kc;
    }
    if (!mbar_wait_bounded(&full[buf], ph, kMmaTimeoutNs, abort_flag) && lane == 0) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusCopyTimeout);
    }
    __syncwarp();
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t st = static_cast<uint32_t>(a.off_stage) + static_cast<uint32_t>(buf) * stage_bytes;
    if (active) tile8_q4k(smem, st + off_g, st + off_g8, (kc & 1) * XC + sbw * kXRec, g, t, v);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);  // the weights are consumed: the producer may refill
    // partials [warp][row][column]: a warp's 32 lanes write 32 consecutive words per store
    float* rb = red + static_cast<size_t>(buf) * red_stage;
    const int r0 = 16 * ti + g, r8 = r0 + 8;
    *reinterpret_cast<float2*>(rb + sbw * (SR * kXB) + r0 * kXB + 2 * t) = make_float2(v[0], v[1]);
    *reinterpret_cast<float2*>(rb + sbw * (SR * kXB) + r8 * kXB + 2 * t) = make_float2(v[2], v[3]);
    // The 8 consumer warps reduce the stage's partials together (fixed order,
    // deterministic).  red[buf] is written again NS >= 2 stages later, after
    // every warp has passed the next stage's barrier.
    named_bar_sync(1, 256);
    const int grp = s - kc * ngroups;
    const int rows_g = min(SR, nrows - SR * grp);
    for (int idx = cw * 32 + lane; idx < SR * kXB; idx += 256) {
      const int r = idx >> 3, b = idx & 7;
      if (r < rows_g) {
        float sum = 0.f;
        for (int w = 0; w < a.KC; ++w) sum += rb[w * (SR * kXB) + idx];
        const int ar = (SR * grp + r) * kXB + b;
        const float tot = acc[ar] + sum;
        acc[ar] = tot;
        if (kc == a.NKC - 1 && b < a.cols) a.y[static_cast<long long>(b) * a.ldy + row0 + SR * grp + r] = tot;
      }
    }
    if (++buf == a.NS) { buf = 0; ph ^= 1u; }
  }
}

cudaError_t launch_xprep8(const float* x, int cols, int in_dim, uint8_t* out, cudaStream_t st) {
  k_xprep8<<<in_dim / 256, 256, 0, st>>>(x, cols, in_dim, out);
  return cudaGetLastError();
}

cudaError_t launch_gemm8_q4k(const Gemm8Args& a, int grid, size_t smem, cudaStream_t st) {
  cudaError_t e = set_smem_once<k_gemm8_q4k>(smem);
  if (e != cudaSuccess) return e;
  k_gemm8_q4k<<<grid, 288, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace m3g
