// m3g_formats.cuh -- the four GGUF block formats of the fused GEMV path.
//
// Each format describes one "unit": the slice of a block that one thread
// decodes and dots against x for every output row it visits.  A thread keeps
// the x values of its unit in registers (the unit's K positions are fixed
// across rows), so the inner loop touches only weight bytes.
//
// Numerics: every quant becomes its exact float (the PRMT/FADD trick of
// m3g_device.cuh), products with x are summed in fp32 with FMA, and the block
// scales are applied once per group:
//   Q4_K: sum_l (d*sc*q_l - dmin*m) x_l = (d*sc) * sum_l q_l x_l - (dmin*m) * sum_l x_l
//   Q6_K: sum_l d*s*(q_l-32) x_l      = (d*s) * sum_l (q_l-32) x_l
//   Q8_0 / Q4_0: d * sum_l q_l x_l
// which is the reference's sum (src/matvec_quant.rs:249-356 and :124-216)
// re-associated; the difference is bounded by the fp32 rounding of the sums.
#pragma once
#include "m3g_device.cuh"

namespace m3g {

// ---------------------------------------------------------------- Q4_K
// 144-byte super-block [d f16][dmin f16][scales 12][qs 128] of 256 weights
// (src/quant.rs:41-71).  Unit = 32-byte chunk c of qs: low nibbles are the 32
// weights of sub-block 2c, high nibbles those of sub-block 2c+1, i.e. the 64
// contiguous elements 64c .. 64c+63 of the block.
struct FmtQ4K {
  static constexpr int kBlockBytes = 144, kBlockElems = 256, kUnitsPerBlock = 4, kUnitElems = 64, kExtra = 2;

  __device__ static __forceinline__ int xpos(int u, int i) { return 256 * (u >> 2) + 64 * (u & 3) + i; }

  __device__ static __forceinline__ void prep(const float (&x)[kUnitElems], float (&e)[kExtra]) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { a += x[i]; b += x[32 + i]; }
    e[0] = a;
    e[1] = b;
  }

  // 6-bit scale/min pair j of a block from its 12 scale bytes held as three
  // little-endian words (get_scale_min_k4, src/quant.rs:28-36), computed for
  // the pair (2c, 2c+1) without branching on c.
  __device__ static __forceinline__ void scales(uint32_t s0, uint32_t s1, uint32_t s2, int c, uint32_t& sc_a,
                                                uint32_t& m_a, uint32_t& sc_b, uint32_t& m_b) {
    // j < 4: sc = q[j] & 63, m = q[j+4] & 63
    const uint32_t sc_lo = s0 & 0x3F3F3F3Fu, m_lo = s1 & 0x3F3F3F3Fu;
    // j >= 4: sc = (q[j+4] & 0xF) | (q[j-4] >> 6) << 4, m = (q[j+4] >> 4) | (q[j] >> 6) << 4
    const uint32_t sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    const uint32_t scw = c < 2 ? sc_lo : sc_hi;
    const uint32_t mw = c < 2 ? m_lo : m_hi;
    const uint32_t sh = static_cast<uint32_t>(c & 1) * 16u;
    sc_a = (scw >> sh) & 0xFFu;
    sc_b = (scw >> (sh + 8u)) & 0xFFu;
    m_a = (mw >> sh) & 0xFFu;
    m_b = (mw >> (sh + 8u)) & 0xFFu;
  }

  __device__ static __forceinline__ float dot(const uint8_t* row, int u, const float (&x)[kUnitElems],
                                              const float (&e)[kExtra]) {
    const int b = u >> 2, c = u & 3;
    const uint8_t* blk = row + b * kBlockBytes;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
    const float d = f16_to_f32(hdr.x), dmin = f16_to_f32(hdr.x >> 16);
    uint32_t sc_a, m_a, sc_b, m_b;
    scales(hdr.y, hdr.z, hdr.w, c, sc_a, m_a, sc_b, m_b);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    float lo0 = 0.f, lo1 = 0.f, hi0 = 0.f, hi1 = 0.f;  // four short FMA chains
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t l = q[w] & 0x0F0F0F0Fu;
      const uint32_t h = (q[w] >> 4) & 0x0F0F0F0Fu;
      lo0 = fmaf(byte_2p23<0>(l) - k2p23, x[4 * w + 0], lo0);
      lo1 = fmaf(byte_2p23<1>(l) - k2p23, x[4 * w + 1], lo1);
      lo0 = fmaf(byte_2p23<2>(l) - k2p23, x[4 * w + 2], lo0);
      lo1 = fmaf(byte_2p23<3>(l) - k2p23, x[4 * w + 3], lo1);
      hi0 = fmaf(byte_2p23<0>(h) - k2p23, x[32 + 4 * w + 0], hi0);
      hi1 = fmaf(byte_2p23<1>(h) - k2p23, x[32 + 4 * w + 1], hi1);
      hi0 = fmaf(byte_2p23<2>(h) - k2p23, x[32 + 4 * w + 2], hi0);
      hi1 = fmaf(byte_2p23<3>(h) - k2p23, x[32 + 4 * w + 3], hi1);
    }
    const float lo = lo0 + lo1, hi = hi0 + hi1;
    const float d1 = d * (float)sc_a, d2 = d * (float)sc_b;
    const float m1 = dmin * (float)m_a, m2 = dmin * (float)m_b;
    return (d1 * lo - m1 * e[0]) + (d2 * hi - m2 * e[1]);
  }
};

// ---------------------------------------------------------------- Q6_K
// 210-byte super-block [ql 128][qh 64][scales 16 x i8][d f16] (src/quant.rs:76-116).
// Unit t = 2n + g (half n, l in [16g, 16g+16)): the four 16-element groups
// 128n + 16g + 32k + i (k = 0..3) with scales s[8n + g + 2k], built from
// ql[64n+16g ..+16] (k = 0, 2), ql[64n+32+16g ..+16] (k = 1, 3) and qh[32n+16g ..+16].
struct FmtQ6K {
  static constexpr int kBlockBytes = 210, kBlockElems = 256, kUnitsPerBlock = 4, kUnitElems = 64, kExtra = 1;

  __device__ static __forceinline__ int xpos(int u, int i) {
    const int b = u >> 2, n = (u >> 1) & 1, g = u & 1;
    return 256 * b + 128 * n + 16 * g + 32 * (i >> 4) + (i & 15);
  }
  __device__ static __forceinline__ void prep(const float (&)[kUnitElems], float (&e)[kExtra]) { e[0] = 0.f; }

  __device__ static __forceinline__ float dot(const uint8_t* row, int u, const float (&x)[kUnitElems],
                                              const float (&)[kExtra]) {
    const int b = u >> 2, n = (u >> 1) & 1, g = u & 1;
    const uint8_t* blk = row + b * kBlockBytes;
    uint32_t A[4], B[4], C[4], S[2];
    lds_words<4>(blk + 64 * n + 16 * g, A);
    lds_words<4>(blk + 64 * n + 32 + 16 * g, B);
    lds_words<4>(blk + 128 + 32 * n + 16 * g, C);
    lds_words<2>(blk + 192 + 8 * n, S);
    const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
    constexpr float kBias = 8388608.0f + 32.0f;
    float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t q1 = (A[w] & 0x0F0F0F0Fu) | ((C[w] << 4) & 0x30303030u);
      const uint32_t q2 = (B[w] & 0x0F0F0F0Fu) | ((C[w] << 2) & 0x30303030u);
      const uint32_t q3 = ((A[w] >> 4) & 0x0F0F0F0Fu) | (C[w] & 0x30303030u);
      const uint32_t q4 = ((B[w] >> 4) & 0x0F0F0F0Fu) | ((C[w] >> 2) & 0x30303030u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        g0 = fmaf(byte_2p23_rt(q1, k) - kBias, x[4 * w + k], g0);
        g1 = fmaf(byte_2p23_rt(q2, k) - kBias, x[16 + 4 * w + k], g1);
        g2 = fmaf(byte_2p23_rt(q3, k) - kBias, x[32 + 4 * w + k], g2);
        g3 = fmaf(byte_2p23_rt(q4, k) - kBias, x[48 + 4 * w + k], g3);
      }
    }
    // int8 scales s[8n + g + 2k]: bytes g, g+2 of S[0] and g, g+2 of S[1]
    const int sh = 8 * g;
    const float s0 = (float)(int8_t)((S[0] >> sh) & 0xFFu);
    const float s1 = (float)(int8_t)((S[0] >> (sh + 16)) & 0xFFu);
    const float s2 = (float)(int8_t)((S[1] >> sh) & 0xFFu);
    const float s3 = (float)(int8_t)((S[1] >> (sh + 16)) & 0xFFu);
    return d * ((s0 * g0 + s1 * g1) + (s2 * g2 + s3 * g3));
  }
};

// ---------------------------------------------------------------- Q8_0
// 34-byte block [d f16][32 x i8] (src/quant.rs:156-170).  Unit = one block.
struct FmtQ80 {
  static constexpr int kBlockBytes = 34, kBlockElems = 32, kUnitsPerBlock = 1, kUnitElems = 32, kExtra = 1;

  __device__ static __forceinline__ int xpos(int u, int i) { return 32 * u + i; }
  __device__ static __forceinline__ void prep(const float (&)[kUnitElems], float (&e)[kExtra]) { e[0] = 0.f; }

  __device__ static __forceinline__ float dot(const uint8_t* row, int u, const float (&x)[kUnitElems],
                                              const float (&)[kExtra]) {
    const uint8_t* blk = row + u * kBlockBytes;
    uint32_t Q[8];
    lds_words<8>(blk + 2, Q);
    const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk));
    constexpr float kBias = 8388608.0f + 128.0f;  // int8 q stored as (q ^ 0x80) = q + 128
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t v = Q[w] ^ 0x80808080u;
      s0 = fmaf(byte_2p23<0>(v) - kBias, x[4 * w + 0], s0);
      s1 = fmaf(byte_2p23<1>(v) - kBias, x[4 * w + 1], s1);
      s0 = fmaf(byte_2p23<2>(v) - kBias, x[4 * w + 2], s0);
      s1 = fmaf(byte_2p23<3>(v) - kBias, x[4 * w + 3], s1);
    }
    return d * (s0 + s1);
  }
};

// ---------------------------------------------------------------- Q4_0
// 18-byte block [d f16][16 bytes of nibbles]: low nibbles are elements 0..15,
// high nibbles 16..31, each q - 8 (src/quant.rs:9-24).  Unit = one block.
struct FmtQ40 {
  static constexpr int kBlockBytes = 18, kBlockElems = 32, kUnitsPerBlock = 1, kUnitElems = 32, kExtra = 1;

  __device__ static __forceinline__ int xpos(int u, int i) { return 32 * u + i; }
  __device__ static __forceinline__ void prep(const float (&)[kUnitElems], float (&e)[kExtra]) { e[0] = 0.f; }

  __device__ static __forceinline__ float dot(const uint8_t* row, int u, const float (&x)[kUnitElems],
                                              const float (&)[kExtra]) {
    const uint8_t* blk = row + u * kBlockBytes;
    uint32_t Q[4];
    lds_words<4>(blk + 2, Q);
    const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk));
    constexpr float kBias = 8388608.0f + 8.0f;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t l = Q[w] & 0x0F0F0F0Fu, h = (Q[w] >> 4) & 0x0F0F0F0Fu;
      s0 = fmaf(byte_2p23<0>(l) - kBias, x[4 * w + 0], s0);
      s1 = fmaf(byte_2p23<1>(l) - kBias, x[4 * w + 1], s1);
      s0 = fmaf(byte_2p23<2>(l) - kBias, x[4 * w + 2], s0);
      s1 = fmaf(byte_2p23<3>(l) - kBias, x[4 * w + 3], s1);
      s0 = fmaf(byte_2p23<0>(h) - kBias, x[16 + 4 * w + 0], s0);
      s1 = fmaf(byte_2p23<1>(h) - kBias, x[16 + 4 * w + 1], s1);
      s0 = fmaf(byte_2p23<2>(h) - kBias, x[16 + 4 * w + 2], s0);
      s1 = fmaf(byte_2p23<3>(h) - kBias, x[16 + 4 * w + 3], s1);
    }
    return d * (s0 + s1);
  }
};

// ---------------------------------------------------------------- exact block decode
// Element e of a block as the reference decoders produce it, bit for bit.
// Products that the reference rounds are spelled with __fmul_rn/__fsub_rn so
// that no FMA contraction changes them (they are exact anyway, see below).
//
// Q4_K: d*sc (<= 17 significant bits) and (d*sc)*q (<= 21) are exact in f32,
// so the only rounding is the final subtraction, as in the reference.
__device__ __forceinline__ float q4k_elem(const uint8_t* blk, int e) {
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk);
  const float d = f16_to_f32(w0), dmin = f16_to_f32(w0 >> 16);
  const uint8_t* sc = blk + 4;
  const int c = e >> 6, l = e & 63, j = 2 * c + (l >> 5);
  uint32_t s, m;
  if (j < 4) {
    s = sc[j] & 63u;
    m = sc[j + 4] & 63u;
  } else {
    s = (sc[j + 4] & 0xFu) | ((sc[j - 4] >> 6) << 4);
    m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  const uint8_t qb = blk[16 + 32 * c + (l & 31)];
  const uint32_t q = (l < 32) ? (qb & 0xFu) : (qb >> 4);
  return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
}

// Q6_K: (d*s)*q has at most 11+7+5 significant bits, so it is exact.
__device__ __forceinline__ float q6k_elem(const uint8_t* blk, int e) {
  const int n = e >> 7, r = e & 127, k = r >> 5, l = r & 31;
  const uint8_t qlb = blk[64 * n + l + ((k & 1) ? 32 : 0)];
  const uint8_t qhb = blk[128 + 32 * n + l];
  const uint32_t low = (k < 2) ? (qlb & 0xFu) : (qlb >> 4);
  const int q = (int)(low | (((qhb >> (2 * k)) & 3u) << 4)) - 32;
  const float s = (float)(int8_t)blk[192 + 8 * n + (l >> 4) + 2 * k];
  const float d = f16_to_f32(blk[208] | (blk[209] << 8));
  return __fmul_rn(__fmul_rn(d, s), (float)q);
}

__device__ __forceinline__ float q8_0_elem(const uint8_t* blk, int e) {
  const float d = f16_to_f32(blk[0] | (blk[1] << 8));
  return __fmul_rn((float)(int8_t)blk[2 + e], d);
}

__device__ __forceinline__ float q4_0_elem(const uint8_t* blk, int e) {
  const float d = f16_to_f32(blk[0] | (blk[1] << 8));
  const uint8_t qb = blk[2 + (e & 15)];
  const int q = (int)((e < 16) ? (qb & 0xFu) : (qb >> 4)) - 8;
  return __fmul_rn((float)q, d);
}

}  // namespace m3g
