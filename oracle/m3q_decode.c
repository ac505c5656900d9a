/*
 * m3q_decode.c -- CPU oracle for one greedy decode step of m3_avm's
 * Llama-style transformer (RealInference::forward_one, src/inference.rs:953-1152).
 *
 * TEST INFRASTRUCTURE ONLY.  This restates, in plain C, the reference's CPU
 * forward pass with every MATVEC on its CPU path (matvec_quant for the
 * quantised GGUF weights, the f32-cached sequential loop for the vocab head),
 * so that the device decode engine of the CUDA library can be checked against
 * it.  Only tests, the smoke check and the CPU-baseline leg of the benchmark
 * may load it; the product library never links or calls it.
 *
 * Followed step by step (reference file:line):
 *   embedding_row            src/inference.rs:903-944  (dequantise one row)
 *   rope frequencies         src/inference.rs:1000-1007 (pos * theta^(-2i/hd))
 *   rms_norm_into            src/inference.rs:1575-1585 (eps fixed at 1e-5)
 *   q/k/v GEMVs              src/inference.rs:1018-1021 -> matvec_quant
 *   apply_rope               src/inference.rs:1554-1572 (split-half pairs)
 *   repeat_kv_extend         src/inference.rs:448-470  (query head hh reads
 *                            KV head hh / (n_heads / n_kv_heads); the cache
 *                            here is stored compact, the values are the same)
 *   per-head attention       src/inference.rs:1052-1079 (sequential dot,
 *                            max-subtracted exp, divide by the running sum)
 *   o GEMV + residual        src/inference.rs:1082-1084
 *   SwiGLU FFN + residual    src/inference.rs:1086-1104
 *   final norm + head        src/inference.rs:1108-1120, logits_from_head_cached :735-764
 *   greedy sampling          sample_with_params :1315-1369 with top_k = 1
 *
 * Floating point follows Rust's strict rules (built with -ffp-contract=off,
 * no -ffast-math); expf/powf/cosf/sinf/sqrtf come from the same C math
 * library that Rust's f32 methods call on Linux.
 */
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <omp.h>

#define OR_API __attribute__((visibility("default")))

/* From m3q_oracle.c (same shared object). */
int or_dequantize(const uint8_t* src, size_t src_len, uint32_t dtype, float* dst, size_t n);
int or_matvec_quant(const float* x, size_t x_len, const uint8_t* raw, size_t raw_len, uint32_t dtype,
                    size_t in_dim, size_t out_dim, float* y, int nthreads);

/* Tensor slots: 0 token_embd, 1 output_norm (f32), 2 output (vocab head),
 * then 9 per layer: attn_norm (f32), q, k, v, o, ffn_norm (f32), gate, up, down. */
enum { SLOT_EMBD = 0, SLOT_OUT_NORM = 1, SLOT_OUT = 2, SLOT_LAYER0 = 3, SLOTS_PER_LAYER = 9 };
enum { L_ATTN_NORM = 0, L_Q, L_K, L_V, L_O, L_FFN_NORM, L_GATE, L_UP, L_DOWN };

typedef struct {
    const uint8_t* p;
    size_t len;
    uint32_t dtype;
} or_tensor;

typedef struct {
    int n_layers, hidden, ffn, n_heads, n_kv_heads, vocab, max_pos, pos;
    float rope_theta;
    or_tensor* t;   /* 3 + 9 * n_layers */
    float* kc;      /* [n_layers][max_pos][n_kv_heads * hd] */
    float* vc;
    float* head32;  /* the f32 head the CPU path caches (vocab x hidden) */
} or_decoder;

static int head_dim(const or_decoder* d) { return d->n_heads == 0 ? d->hidden : d->hidden / d->n_heads; }

OR_API or_decoder* or_decoder_create(int n_layers, int hidden, int ffn, int n_heads, int n_kv_heads, int vocab,
                                     float rope_theta, int max_pos) {
    if (n_layers <= 0 || hidden <= 0 || ffn <= 0 || n_heads <= 0 || n_kv_heads <= 0 || vocab <= 0 || max_pos <= 0)
        return NULL;
    if (hidden % n_heads || n_heads % n_kv_heads) return NULL;
    or_decoder* d = (or_decoder*)calloc(1, sizeof *d);
    if (!d) return NULL;
    d->n_layers = n_layers; d->hidden = hidden; d->ffn = ffn; d->n_heads = n_heads;
    d->n_kv_heads = n_kv_heads; d->vocab = vocab; d->rope_theta = rope_theta; d->max_pos = max_pos;
    const size_t kvh = (size_t)n_kv_heads * (size_t)(hidden / n_heads);
    d->t = (or_tensor*)calloc((size_t)(SLOT_LAYER0 + SLOTS_PER_LAYER * n_layers), sizeof(or_tensor));
    d->kc = (float*)calloc((size_t)n_layers * (size_t)max_pos * kvh, sizeof(float));
    d->vc = (float*)calloc((size_t)n_layers * (size_t)max_pos * kvh, sizeof(float));
    if (!d->t || !d->kc || !d->vc) {
        free(d->t); free(d->kc); free(d->vc); free(d);
        return NULL;
    }
    return d;
}

OR_API void or_decoder_destroy(or_decoder* d) {
    if (!d) return;
    free(d->t); free(d->kc); free(d->vc); free(d->head32); free(d);
}

/* The caller keeps `p` alive for the decoder's lifetime.  1 = ok. */
OR_API int or_decoder_set(or_decoder* d, int slot, const void* p, size_t len, uint32_t dtype) {
    if (slot < 0 || slot >= SLOT_LAYER0 + SLOTS_PER_LAYER * d->n_layers) return 0;
    d->t[slot].p = (const uint8_t*)p;
    d->t[slot].len = len;
    d->t[slot].dtype = dtype;
    if (slot == SLOT_OUT) { free(d->head32); d->head32 = NULL; }
    return 1;
}

OR_API int or_decoder_pos(const or_decoder* d) { return d->pos; }
OR_API void or_decoder_reset(or_decoder* d) { d->pos = 0; }
/* truncate_kv_cache (src/inference.rs) keeps the first n positions. */
OR_API void or_decoder_truncate(or_decoder* d, int n) { if (n >= 0 && n < d->pos) d->pos = n; }

/* rms_norm_into (src/inference.rs:1575-1585). */
OR_API void or_rms_norm_into(const float* x, const float* gamma, float* out, size_t n) {
    const float eps = 1e-5f;
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += x[i] * x[i];
    const float mean = sum / (float)n;
    const float rms = sqrtf(mean + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] / rms * (gamma ? gamma[i] : 1.0f);
}

/* (cos, sin) pairs for position `pos` (src/inference.rs:1000-1007). */
OR_API void or_rope_freqs(int pos, int hd, float theta, float* cs /* [hd/2][2] */) {
    const int half = (hd < 2 ? 2 : hd) / 2;
    for (int i = 0; i < half; i++) {
        const float f = (float)pos * powf(theta, -2.0f * (float)i / (float)(hd < 1 ? 1 : hd));
        cs[2 * i] = cosf(f);
        cs[2 * i + 1] = sinf(f);
    }
}

/* apply_rope (src/inference.rs:1554-1572): pair (i, i + half) of each head. */
OR_API void or_apply_rope(float* v, size_t len, int n_heads, int hd, const float* cs) {
    if (hd == 0 || hd % 2) return;
    const int half = hd / 2;
    for (int hh = 0; hh < n_heads; hh++) {
        const size_t base = (size_t)hh * (size_t)hd;
        if (base + (size_t)hd > len) break;
        for (int i = 0; i < half; i++) {
            const float c = cs[2 * i], s = cs[2 * i + 1];
            const float a = v[base + i], b = v[base + i + half];
            v[base + i] = a * c - b * s;
            v[base + i + half] = a * s + b * c;
        }
    }
}

/* Greedy pick of sample_with_params with top_k = 1 and no repetition
 * penalty: a stable descending sort keeps the first of equal maxima, so the
 * result is the lowest index holding the largest logit. */
OR_API uint32_t or_greedy(const float* logits, size_t n) {
    if (n == 0) return 0;
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (logits[i] > logits[best]) best = i;
    return (uint32_t)best;
}

/* One attention head over positions [0, npos) of a compact KV cache
 * (src/inference.rs:1052-1079). */
OR_API void or_attention_head(const float* q, const float* kc, const float* vc, size_t row_stride, int npos, int hd,
                              float* out, float* scores) {
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = 0; i < npos; i++) {
        const float* kb = kc + (size_t)i * row_stride;
        float dot = 0.0f;
        for (int j = 0; j < hd; j++) dot += q[j] * kb[j];
        scores[i] = dot * scale;
    }
    float mx = -INFINITY;
    for (int i = 0; i < npos; i++) mx = fmaxf(mx, scores[i]);
    float sum = 0.0f;
    for (int i = 0; i < npos; i++) { scores[i] = expf(scores[i] - mx); sum += scores[i]; }
    for (int i = 0; i < npos; i++) scores[i] /= sum;
    for (int i = 0; i < npos; i++) {
        const float* vb = vc + (size_t)i * row_stride;
        const float w = scores[i];
        for (int j = 0; j < hd; j++) out[j] += w * vb[j];
    }
}

static int matvec(const or_tensor* t, const float* x, size_t in_dim, size_t out_dim, float* y, int nthreads) {
    if (!t->p) return 0;
    return or_matvec_quant(x, in_dim, t->p, t->len, t->dtype, in_dim, out_dim, y, nthreads) == 1;
}

/* Block geometry embedding_row slices by (src/inference.rs:924-930). */
static int row_block(uint32_t dtype, size_t* be, size_t* bb) {
    switch (dtype) {
    case 2: *be = 32; *bb = 18; return 1;
    case 8: *be = 32; *bb = 34; return 1;
    case 12: case 13: *be = 256; *bb = 144; return 1;
    case 14: *be = 256; *bb = 210; return 1;
    default: return 0;
    }
}

/* embedding_row: dequantise only the blocks of row `row`. */
static int embedding_row(const or_tensor* t, size_t row, size_t h, size_t n_rows, float* dst) {
    if (!t->p || row >= n_rows) return 0;
    const size_t base = row * h;
    if (t->dtype == 0) { memcpy(dst, t->p + base * 4, h * 4); return 1; }
    size_t be = 0, bb = 0;
    if (t->dtype == 1) {
        return or_dequantize(t->p + base * 2, h * 2, 1, dst, h) == 1;
    }
    if (!row_block(t->dtype, &be, &bb)) return 0;
    if (base % be || h % be) return 0;
    const size_t b0 = base / be, nb = h / be;
    if ((b0 + nb) * bb > t->len) return 0;
    return or_dequantize(t->p + b0 * bb, nb * bb, t->dtype, dst, h) == 1;
}

/* The CPU head caches the dequantised f32 matrix once, then sums each row
 * sequentially (logits_from_head_cached). */
static int head_logits(or_decoder* d, const float* xn, float* logits, int nthreads) {
    const size_t h = (size_t)d->hidden, V = (size_t)d->vocab;
    const or_tensor* t = &d->t[SLOT_OUT];
    if (!t->p) return 0;
    if (!d->head32) {
        d->head32 = (float*)malloc(V * h * sizeof(float));
        if (!d->head32) return 0;
        if (or_dequantize(t->p, t->len, t->dtype == 13 ? 12 : t->dtype, d->head32, V * h) != 1) {
            free(d->head32); d->head32 = NULL;
            return 0;
        }
    }
    const float* W = d->head32;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : omp_get_max_threads())
    for (size_t i = 0; i < V; i++) {
        float sum = 0.0f;
        for (size_t j = 0; j < h; j++) sum += xn[j] * W[i * h + j];
        logits[i] = sum;
    }
    return 1;
}

/* One forward_one step: embeds `token` at position pos, appends its K/V and
 * writes vocab logits.  1 = ok, 0 = a missing tensor, a bad token or a full
 * cache. */
OR_API int or_decoder_forward(or_decoder* d, uint32_t token, float* logits, int nthreads) {
    const int h = d->hidden, F = d->ffn, hd = head_dim(d);
    const int kvh = d->n_kv_heads * hd, groups = d->n_heads / d->n_kv_heads;
    if (d->pos >= d->max_pos || token >= (uint32_t)d->vocab) return 0;
    const int pos = d->pos;
    int ok = 1;
    float* hidden = (float*)calloc((size_t)h, 4);
    float* hidden2 = (float*)calloc((size_t)h, 4);
    float* xn = (float*)calloc((size_t)(F > h ? F : h), 4);
    float* q = (float*)calloc((size_t)h, 4);
    float* k = (float*)calloc((size_t)kvh, 4);
    float* v = (float*)calloc((size_t)kvh, 4);
    float* att = (float*)calloc((size_t)h, 4);
    float* tmp = (float*)calloc((size_t)h, 4);
    float* gate = (float*)calloc((size_t)F, 4);
    float* up = (float*)calloc((size_t)F, 4);
    float* scores = (float*)calloc((size_t)d->max_pos, 4);
    float* cs = (float*)calloc((size_t)(hd < 2 ? 2 : hd), 4);
    if (!hidden || !hidden2 || !xn || !q || !k || !v || !att || !tmp || !gate || !up || !scores || !cs) {
        ok = 0;
        goto done;
    }
    if (!embedding_row(&d->t[SLOT_EMBD], token, (size_t)h, (size_t)d->vocab, hidden)) { ok = 0; goto done; }
    or_rope_freqs(pos, hd, d->rope_theta, cs);
    for (int l = 0; l < d->n_layers; l++) {
        const or_tensor* T = &d->t[SLOT_LAYER0 + SLOTS_PER_LAYER * l];
        const float* g_attn = (const float*)T[L_ATTN_NORM].p;
        const float* g_ffn = (const float*)T[L_FFN_NORM].p;
        or_rms_norm_into(hidden, g_attn, xn, (size_t)h);
        if (!matvec(&T[L_Q], xn, h, h, q, nthreads) || !matvec(&T[L_K], xn, h, kvh, k, nthreads) ||
            !matvec(&T[L_V], xn, h, kvh, v, nthreads)) { ok = 0; goto done; }
        or_apply_rope(q, (size_t)h, d->n_heads, hd, cs);
        or_apply_rope(k, (size_t)kvh, d->n_kv_heads, hd, cs);
        float* Kl = d->kc + (size_t)l * (size_t)d->max_pos * (size_t)kvh;
        float* Vl = d->vc + (size_t)l * (size_t)d->max_pos * (size_t)kvh;
        memcpy(Kl + (size_t)pos * kvh, k, (size_t)kvh * 4);
        memcpy(Vl + (size_t)pos * kvh, v, (size_t)kvh * 4);
        memset(att, 0, (size_t)h * 4);
        for (int hh = 0; hh < d->n_heads; hh++) {
            const int kv = hh / groups;
            or_attention_head(q + (size_t)hh * hd, Kl + (size_t)kv * hd, Vl + (size_t)kv * hd, (size_t)kvh, pos + 1, hd,
                              att + (size_t)hh * hd, scores);
        }
        if (!matvec(&T[L_O], att, h, h, tmp, nthreads)) { ok = 0; goto done; }
        for (int i = 0; i < h; i++) hidden2[i] = hidden[i] + tmp[i];
        or_rms_norm_into(hidden2, g_ffn, xn, (size_t)h);
        if (!matvec(&T[L_GATE], xn, h, F, gate, nthreads) || !matvec(&T[L_UP], xn, h, F, up, nthreads)) {
            ok = 0;
            goto done;
        }
        for (int i = 0; i < F; i++) {
            const float g = gate[i];
            const float sig = 1.0f / (1.0f + expf(-g));
            xn[i] = g * sig * up[i];
        }
        if (!matvec(&T[L_DOWN], xn, F, h, tmp, nthreads)) { ok = 0; goto done; }
        for (int i = 0; i < h; i++) hidden[i] = hidden2[i] + tmp[i];
    }
    or_rms_norm_into(hidden, (const float*)d->t[SLOT_OUT_NORM].p, xn, (size_t)h);
    if (!head_logits(d, xn, logits, nthreads)) { ok = 0; goto done; }
    d->pos = pos + 1;
done:
    free(hidden); free(hidden2); free(xn); free(q); free(k); free(v); free(att); free(tmp);
    free(gate); free(up); free(scores); free(cs);
    return ok;
}
