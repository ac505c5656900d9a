/*
 * m3q_oracle.c -- CPU oracle for the fused quantised GEMV path of m3_avm.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the reference's
 * CPU algorithm for the GGUF block decoders and the fused dequantise-and-matvec
 * so that the CUDA library can be checked against it.  Only tests, the smoke
 * check and the CPU-baseline leg of the benchmark may load it; the product
 * library never links or calls it.
 *
 * Parity anchor: the reference is pure Rust and cannot be built here, so this
 * restatement is pinned by (1) every known-answer test the reference's own
 * unit tests hold for this path (src/quant.rs:277-448,
 * src/matvec_quant.rs:384-582, src/matvec.rs:101-120), ported as pytest cases,
 * and (2) the independent ggml-format decoders of the `gguf` Python package
 * (the reference cites ggml-quants.c as its source format).
 *
 * Floating point follows Rust's strict rules: build with -O3
 * -ffp-contract=off and without -ffast-math, so every `a*b + c` rounds twice
 * and no loop is reassociated.  f16 -> f32 is the exact IEEE widening that
 * `half` 2.7.1 `f16::to_f32` performs.
 *
 * Return conventions (the reference's Option/bool/assert! mapped to C):
 *   1  = Some / true,   0 = None / false,   -1 = the reference would panic
 *   (an assert! on the block count or the source length).
 */
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <omp.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define OR_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- f16 / bf16 */

static inline float u32_as_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_as_u32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Exact IEEE binary16 -> binary32 widening (what half::f16::to_f32 computes). */
OR_API float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return u32_as_f32(sign);
        /* subnormal half: renormalise into a normal float */
        int e = -1;
        do { e++; man <<= 1; } while ((man & 0x400u) == 0);
        man &= 0x3FFu;
        return u32_as_f32(sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13));
    }
    if (exp == 31) return u32_as_f32(sign | 0x7F800000u | (man << 13));
    return u32_as_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16 with round-to-nearest-even (half::f16::from_f32). */
OR_API uint16_t or_f32_to_f16_bits(float f) {
    uint32_t x = f32_as_u32(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) {
        if (man == 0) return sign | 0x7C00u;
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return sign | 0x7C00u;
    if (e <= 0) {
        if (e < -10) return sign;
        man |= 0x800000u;
        int shift = 14 - e;                 /* 14..24 */
        uint32_t hm = man >> shift;
        uint32_t rb = 1u << (shift - 1);
        uint32_t rest = man & ((1u << shift) - 1u);
        if (rest > rb || (rest == rb && (hm & 1u))) hm += 1;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = man >> 13;
    uint32_t rest = man & 0x1FFFu;
    uint32_t out = ((uint32_t)e << 10) | hm;
    if (rest > 0x1000u || (rest == 0x1000u && (hm & 1u))) out += 1;  /* carry may bump exp */
    return (uint16_t)(sign | out);
}

static inline float rd_f16(const uint8_t* p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* f32 -> bf16 bits, RNE with a quiet-NaN guard (src/quant.rs:186-194). */
OR_API uint16_t or_f32_to_bf16_bits(float x) {
    uint32_t b = f32_as_u32(x);
    uint32_t bias = 0x7FFFu + ((b >> 16) & 1u);
    uint16_t bf = (uint16_t)((b + bias) >> 16);
    if (isnan(x)) bf |= 0x0040u;
    return bf;
}

/* bf16 bits -> f32 (src/quant.rs:197-199). */
OR_API float or_bf16_bits_to_f32(uint16_t b) { return u32_as_f32((uint32_t)b << 16); }

/* ---------------------------------------------------------------- decoders */

/* Q4_0, 18-byte blocks of 32 (src/quant.rs:9-24). */
OR_API int or_dequant_q4_0(const uint8_t* src, size_t src_len, float* dst, size_t n) {
    if (n % 32 != 0) return -1;
    size_t nb = n / 32;
    if (src_len < nb * 18) return -1;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = src + b * 18;
        float d = rd_f16(blk);
        for (int i = 0; i < 16; i++) {
            uint8_t q = blk[2 + i];
            int lo = (int)(q & 0x0F) - 8;
            int hi = (int)(q >> 4) - 8;
            dst[b * 32 + i] = (float)lo * d;
            dst[b * 32 + 16 + i] = (float)hi * d;
        }
    }
    return 1;
}

/* ggml 6-bit scale/min unpack (src/quant.rs:28-36). */
OR_API void or_get_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q4_K super-block [d f16][dmin f16][scales 12][qs 128] (src/quant.rs:41-71). */
static void q4k_block(const uint8_t* blk, float* out) {
    float d = rd_f16(blk);
    float dmin = rd_f16(blk + 2);
    const uint8_t* sc = blk + 4;
    const uint8_t* qs = blk + 16;
    for (int c = 0; c < 4; c++) {
        uint8_t s, m;
        or_get_scale_min_k4(2 * c, sc, &s, &m);
        float d1 = d * (float)s, m1 = dmin * (float)m;
        or_get_scale_min_k4(2 * c + 1, sc, &s, &m);
        float d2 = d * (float)s, m2 = dmin * (float)m;
        for (int l = 0; l < 32; l++) {
            out[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0xF) - m1;
            out[64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - m2;
        }
    }
}

OR_API int or_dequant_q4_k(const uint8_t* src, size_t src_len, float* dst, size_t n) {
    if (n % 256 != 0) return -1;
    size_t nb = n / 256;
    if (src_len < nb * 144) return -1;
    for (size_t b = 0; b < nb; b++) q4k_block(src + b * 144, dst + b * 256);
    return 1;
}

/* Q6_K super-block [ql 128][qh 64][scales 16 x i8][d f16] (src/quant.rs:76-116). */
static void q6k_block(const uint8_t* blk, float* out) {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* sc = (const int8_t*)(blk + 192);
    float d = rd_f16(blk + 208);
    for (int h = 0; h < 2; h++) {
        const uint8_t* l0 = ql + 64 * h;
        const uint8_t* h0 = qh + 32 * h;
        const int8_t* s0 = sc + 8 * h;
        float* y = out + 128 * h;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)((l0[l] & 0xF) | (((h0[l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)((l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32;
            /* evaluated left to right: (d * s) * q, as the reference does */
            y[l] = d * (float)s0[is] * (float)q1;
            y[l + 32] = d * (float)s0[is + 2] * (float)q2;
            y[l + 64] = d * (float)s0[is + 4] * (float)q3;
            y[l + 96] = d * (float)s0[is + 6] * (float)q4;
        }
    }
}

OR_API int or_dequant_q6_k(const uint8_t* src, size_t src_len, float* dst, size_t n) {
    if (n % 256 != 0) return -1;
    size_t nb = n / 256;
    if (src_len < nb * 210) return -1;
    for (size_t b = 0; b < nb; b++) q6k_block(src + b * 210, dst + b * 256);
    return 1;
}

/* Q8_0 block [d f16][32 x i8] (src/quant.rs:156-170, src/matvec_quant.rs:376-381). */
static void q8_0_block(const uint8_t* blk, float* out) {
    float d = rd_f16(blk);
    for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)blk[2 + i] * d;
}

static void q4_0_block(const uint8_t* blk, float* out) { or_dequant_q4_0(blk, 18, out, 32); }

/* ggml-dtype dispatcher (src/quant.rs:120-173).  Note the reference maps
 * dtype 13 (Q5_K) onto the Q4_K decoder. */
OR_API int or_dequantize(const uint8_t* src, size_t src_len, uint32_t dtype, float* dst, size_t n) {
    switch (dtype) {
    case 0:
        if (src_len < n * 4) return 0;
        for (size_t i = 0; i < n; i++) { float v; memcpy(&v, src + 4 * i, 4); dst[i] = v; }
        return 1;
    case 1:
        if (src_len < n * 2) return 0;
        for (size_t i = 0; i < n; i++) dst[i] = rd_f16(src + 2 * i);
        return 1;
    case 2:
        if (n % 32 != 0) return 0;
        return or_dequant_q4_0(src, src_len, dst, n);     /* may "panic" (-1) on a short src */
    case 12: case 13:
        if (n % 256 != 0) return 0;
        return or_dequant_q4_k(src, src_len, dst, n);     /* may "panic" (-1) */
    case 14:
        if (n % 256 != 0) return 0;
        if (src_len < (n / 256) * 210) return 0;
        return or_dequant_q6_k(src, src_len, dst, n);
    case 8: {
        if (n % 32 != 0) return 0;
        size_t nb = n / 32;
        if (src_len < nb * 34) return 0;
        for (size_t b = 0; b < nb; b++) q8_0_block(src + b * 34, dst + b * 32);
        return 1;
    }
    default:
        return 0;
    }
}

/* ---------------------------------------------------------------- encoders */

/* Rust `f32 as i32`: saturating, NaN -> 0. */
static inline int32_t sat_i32(float v) {
    if (isnan(v)) return 0;
    if (v >= 2147483647.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}
static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* 32 f32 -> one Q4_0 block (src/quant.rs:206-234). 1 = true, 0 = false. */
OR_API int or_quantize_q4_0(const float* src, size_t src_len, uint8_t* dst, size_t dst_len) {
    if (src_len != 32 || dst_len < 18) return 0;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        if (!isfinite(src[i])) return 0;
        amax = fmaxf(amax, fabsf(src[i]));
    }
    uint16_t dbits = or_f32_to_f16_bits(amax == 0.0f ? 0.0f : amax / 7.0f);
    float ds = or_f16_to_f32(dbits);
    dst[0] = (uint8_t)(dbits & 0xFF); dst[1] = (uint8_t)(dbits >> 8);
    if (amax == 0.0f) { for (int i = 2; i < 18; i++) dst[i] = 0x88; return 1; }
    for (int i = 0; i < 16; i++) {
        int32_t ql = clampi(sat_i32(roundf(src[i] / ds)), -8, 7) + 8;
        int32_t qh = clampi(sat_i32(roundf(src[i + 16] / ds)), -8, 7) + 8;
        dst[2 + i] = (uint8_t)((uint8_t)ql | (uint8_t)(qh << 4));
    }
    return 1;
}

/* 32 f32 -> one Q8_0 block (src/quant.rs:239-264). */
OR_API int or_quantize_q8_0(const float* src, size_t src_len, uint8_t* dst, size_t dst_len) {
    if (src_len != 32 || dst_len < 34) return 0;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        if (!isfinite(src[i])) return 0;
        amax = fmaxf(amax, fabsf(src[i]));
    }
    uint16_t dbits = or_f32_to_f16_bits(amax == 0.0f ? 0.0f : amax / 127.0f);
    float ds = or_f16_to_f32(dbits);
    dst[0] = (uint8_t)(dbits & 0xFF); dst[1] = (uint8_t)(dbits >> 8);
    if (amax == 0.0f) { memset(dst + 2, 0, 32); return 1; }
    for (int i = 0; i < 32; i++) {
        int32_t q = clampi(sat_i32(roundf(src[i] / ds)), -127, 127);
        dst[2 + i] = (uint8_t)(int8_t)q;
    }
    return 1;
}

/* (elems, bytes) for the symmetric encode/decode pairs (src/quant.rs:269-275).
 * Note the reference keys this table by memory::DType numbering (4 = Q4_0). */
OR_API int or_quant_block_info(uint32_t dtype, size_t* elems, size_t* bytes) {
    if (dtype == 4) { *elems = 32; *bytes = 18; return 1; }
    if (dtype == 8) { *elems = 32; *bytes = 34; return 1; }
    return 0;
}

/* ---------------------------------------------------------------- fused GEMV */

/* Bytes for n elements of a fused-kernel dtype (src/matvec_quant.rs:51-83). */
OR_API int or_quant_raw_len(uint32_t dtype, size_t n, size_t* out) {
    switch (dtype) {
    case 2: if (n % 32) return 0; *out = (n / 32) * 18; return 1;
    case 12: case 13: if (n % 256) return 0; *out = (n / 256) * 144; return 1;
    case 14: if (n % 256) return 0; *out = (n / 256) * 210; return 1;
    case 8: if (n % 32) return 0; *out = (n / 32) * 34; return 1;
    default: return 0;
    }
}

typedef void (*block_decoder)(const uint8_t*, float*);

/* The run loop shared by the serial and parallel kernels: one decoded block
 * contributes a dot per output row it overlaps, in the GGUF flat order
 * k = i + j*in_dim (src/matvec_quant.rs:136-157 and :181-203). */
static void block_runs(const float* x, const float* buf, size_t b, size_t in_dim,
                       size_t be, float* acc) {
    size_t base = b * be;
    size_t t = 0, j = base / in_dim, i = base % in_dim;
    while (t < be) {
        size_t run = in_dim - i < be - t ? in_dim - i : be - t;
        float s = 0.0f;
        for (size_t r = 0; r < run; r++) s += x[i + r] * buf[t + r];
        acc[j] += s;
        t += run;
        i += run;
        if (i == in_dim) { i = 0; j++; }
    }
}

/* matvec_blocked_serial (src/matvec_quant.rs:124-159). */
static void matvec_blocked_serial(const float* x, const uint8_t* raw, size_t in_dim, size_t out_dim,
                                  size_t be, size_t bb, block_decoder dec, float* y) {
    size_t nb = (in_dim * out_dim) / be;
    float buf[256];
    memset(y, 0, out_dim * sizeof(float));
    for (size_t b = 0; b < nb; b++) {
        dec(raw + b * bb, buf);
        block_runs(x, buf, b, in_dim, be, y);
    }
}

/* matvec_blocked (src/matvec_quant.rs:165-216): rayon fold of private `y`
 * vectors over super-blocks, then an element-wise reduce.  Restated as one
 * contiguous range of blocks per OpenMP thread and a reduce in thread order,
 * so the result is deterministic for a given thread count. */
static void matvec_blocked(const float* x, const uint8_t* raw, size_t in_dim, size_t out_dim,
                           size_t be, size_t bb, block_decoder dec, float* y, int nthreads) {
    size_t nb = (in_dim * out_dim) / be;
    if (nthreads < 1) nthreads = 1;
    float* accs = (float*)calloc((size_t)nthreads * out_dim, sizeof(float));
    #pragma omp parallel num_threads(nthreads)
    {
        int t = omp_get_thread_num(), nt = omp_get_num_threads();
        size_t lo = nb * (size_t)t / (size_t)nt, hi = nb * (size_t)(t + 1) / (size_t)nt;
        float* acc = accs + (size_t)t * out_dim;
        float buf[256];
        for (size_t b = lo; b < hi; b++) {
            dec(raw + b * bb, buf);
            block_runs(x, buf, b, in_dim, be, acc);
        }
    }
    memset(y, 0, out_dim * sizeof(float));
    for (int t = 0; t < nthreads; t++) {
        const float* acc = accs + (size_t)t * out_dim;
        for (size_t j = 0; j < out_dim; j++) y[j] += acc[j];
    }
    free(accs);
}

#if defined(__x86_64__)
/* dot_q4k_superblock (src/matvec_quant.rs:290-356): the same AVX2 sequence,
 * cvtepi8 -> cvtepi32_ps, q*d - m, then acc += v*x with no FMA, then the
 * 256 -> 128 -> 64 -> 32 horizontal sum. */
__attribute__((target("avx2")))
static float dot_q4k_superblock(const uint8_t* qs, const uint8_t* scales, float d, float dmin,
                                const float* xseg) {
    const __m128i nib = _mm_set1_epi8(0x0F);
    __m256 acc = _mm256_setzero_ps();
    for (int c = 0; c < 4; c++) {
        uint8_t sc0, m0, sc1, m1;
        or_get_scale_min_k4(2 * c, scales, &sc0, &m0);
        or_get_scale_min_k4(2 * c + 1, scales, &sc1, &m1);
        __m256 d0 = _mm256_set1_ps(d * (float)sc0);
        __m256 mv0 = _mm256_set1_ps(dmin * (float)m0);
        __m256 d1 = _mm256_set1_ps(d * (float)sc1);
        __m256 mv1 = _mm256_set1_ps(dmin * (float)m1);
        const uint8_t* qp = qs + 32 * c;
        __m128i q0 = _mm_loadu_si128((const __m128i*)qp);
        __m128i q1 = _mm_loadu_si128((const __m128i*)(qp + 16));
        __m128i nibs[4] = {
            _mm_and_si128(q0, nib), _mm_and_si128(q1, nib),
            _mm_and_si128(_mm_srli_epi16(q0, 4), nib), _mm_and_si128(_mm_srli_epi16(q1, 4), nib),
        };
        const float* xb = xseg + 64 * c;
        for (int job = 0; job < 8; job++) {
            int ko = 8 * job;                      /* 0,8,...,56 */
            __m128i src = nibs[job / 2];
            __m128i part = (ko % 16 == 0) ? src : _mm_srli_si128(src, 8);
            __m256 dv = job < 4 ? d0 : d1;
            __m256 mv = job < 4 ? mv0 : mv1;
            __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(part));
            __m256 v = _mm256_sub_ps(_mm256_mul_ps(qf, dv), mv);
            __m256 xv = _mm256_loadu_ps(xb + ko);
            acc = _mm256_add_ps(acc, _mm256_mul_ps(v, xv));
        }
    }
    __m128 hi = _mm256_extractf128_ps(acc, 1);
    __m128 lo = _mm256_castps256_ps128(acc);
    __m128 s4 = _mm_add_ps(lo, hi);
    __m128 s2 = _mm_add_ps(s4, _mm_movehl_ps(s4, s4));
    __m128 s1 = _mm_add_ss(s2, _mm_shuffle_ps(s2, s2, 0x1));
    return _mm_cvtss_f32(s1);
}

/* matvec_q4k_avx2 (src/matvec_quant.rs:249-285); requires in_dim % 256 == 0. */
OR_API void or_matvec_q4k_avx2(const float* x, const uint8_t* raw, size_t in_dim, size_t out_dim,
                               float* y, int nthreads) {
    size_t nb = (in_dim * out_dim) / 256;
    if (nthreads < 1) nthreads = 1;
    float* accs = (float*)calloc((size_t)nthreads * out_dim, sizeof(float));
    #pragma omp parallel num_threads(nthreads)
    {
        int t = omp_get_thread_num(), nt = omp_get_num_threads();
        size_t lo = nb * (size_t)t / (size_t)nt, hi = nb * (size_t)(t + 1) / (size_t)nt;
        float* acc = accs + (size_t)t * out_dim;
        for (size_t b = lo; b < hi; b++) {
            const uint8_t* blk = raw + b * 144;
            float d = rd_f16(blk), dmin = rd_f16(blk + 2);
            size_t base = b * 256;
            acc[base / in_dim] += dot_q4k_superblock(blk + 16, blk + 4, d, dmin, x + base % in_dim);
        }
    }
    memset(y, 0, out_dim * sizeof(float));
    for (int t = 0; t < nthreads; t++) {
        const float* acc = accs + (size_t)t * out_dim;
        for (size_t j = 0; j < out_dim; j++) y[j] += acc[j];
    }
    free(accs);
}
#endif

static void dec_q4k(const uint8_t* b, float* o) { q4k_block(b, o); }
static void dec_q6k(const uint8_t* b, float* o) { q6k_block(b, o); }
static void dec_q4_0(const uint8_t* b, float* o) { q4_0_block(b, o); }
static void dec_q8_0(const uint8_t* b, float* o) { q8_0_block(b, o); }

/* M3_PAR_MIN gate (src/matvec_quant.rs:116-121), default 1 048 576 elements. */
static size_t par_min_elems(void) {
    const char* s = getenv("M3_PAR_MIN");
    if (s && *s) {
        char* end = NULL;
        unsigned long long v = strtoull(s, &end, 10);
        if (end && *end == 0) return (size_t)v;
    }
    return 1048576;
}

/* matvec_q4k_impl (src/matvec_quant.rs:228-243). */
OR_API void or_matvec_q4k_impl(const float* x, const uint8_t* raw, size_t in_dim, size_t out_dim,
                               int use_avx2, float* y, int nthreads) {
    if (in_dim * out_dim < par_min_elems()) {
        matvec_blocked_serial(x, raw, in_dim, out_dim, 256, 144, dec_q4k, y);
        return;
    }
#if defined(__x86_64__)
    /* cpu_has_avx2 (src/matvec_quant.rs:37-47) is folded into use_avx2 here */
    if (use_avx2 && __builtin_cpu_supports("avx2") && in_dim % 256 == 0 && (in_dim * out_dim) % 256 == 0) {
        or_matvec_q4k_avx2(x, raw, in_dim, out_dim, y, nthreads);
        return;
    }
#endif
    matvec_blocked(x, raw, in_dim, out_dim, 256, 144, dec_q4k, y, nthreads);
}

OR_API void or_matvec_blocked(const float* x, const uint8_t* raw, uint32_t dtype, size_t in_dim,
                              size_t out_dim, float* y, int nthreads, int serial) {
    size_t be = 256, bb = 144; block_decoder dec = dec_q4k;
    if (dtype == 14) { bb = 210; dec = dec_q6k; }
    else if (dtype == 2) { be = 32; bb = 18; dec = dec_q4_0; }
    else if (dtype == 8) { be = 32; bb = 34; dec = dec_q8_0; }
    if (serial) matvec_blocked_serial(x, raw, in_dim, out_dim, be, bb, dec, y);
    else matvec_blocked(x, raw, in_dim, out_dim, be, bb, dec, y, nthreads);
}

/* matvec_quant dispatcher (src/matvec_quant.rs:87-109). 1 = Some(y), 0 = None. */
OR_API int or_matvec_quant(const float* x, size_t x_len, const uint8_t* raw, size_t raw_len,
                           uint32_t dtype, size_t in_dim, size_t out_dim, float* y, int nthreads) {
    if (x_len != in_dim || in_dim == 0 || out_dim == 0) return 0;
    if (out_dim != 0 && in_dim > SIZE_MAX / out_dim) return 0;
    size_t need;
    if (!or_quant_raw_len(dtype, in_dim * out_dim, &need)) return 0;
    if (raw_len < need) return 0;
    switch (dtype) {
    case 12: case 13: or_matvec_q4k_impl(x, raw, in_dim, out_dim, 1, y, nthreads); return 1;
    case 14: case 2: case 8: or_matvec_blocked(x, raw, dtype, in_dim, out_dim, y, nthreads, 0); return 1;
    default: return 0;
    }
}

/* Dense GEMV in the GGUF orientation, y[j] = sum_i x[i] * w[i + j*in_dim]
 * (src/matvec.rs:24-33), summed sequentially per row. */
OR_API void or_matvec_dense(const float* x, const float* w, size_t in_dim, size_t out_dim, float* y) {
    for (size_t j = 0; j < out_dim; j++) {
        float s = 0.0f;
        for (size_t i = 0; i < in_dim; i++) s += x[i] * w[i + j * in_dim];
        y[j] = s;
    }
}

/* Per-row L1 norm of the dequantised weights, sum_i |w[i + j*in_dim]|, in
 * double: the scale of the GEMV error bound 1e-5 * ||row||_1 * ||x||_inf. */
OR_API int or_row_l1(const uint8_t* raw, size_t raw_len, uint32_t dtype, size_t in_dim, size_t out_dim,
                     double* l1) {
    size_t n = in_dim * out_dim;
    float* w = (float*)malloc(n * sizeof(float));
    if (!w) return 0;
    int ok = or_dequantize(raw, raw_len, dtype == 13 ? 12 : dtype, w, n);
    if (ok == 1) {
        for (size_t j = 0; j < out_dim; j++) {
            double s = 0.0;
            for (size_t i = 0; i < in_dim; i++) s += fabs((double)w[i + j * in_dim]);
            l1[j] = s;
        }
    }
    free(w);
    return ok == 1;
}

OR_API int or_max_threads(void) { return omp_get_max_threads(); }
