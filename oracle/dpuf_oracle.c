/*
 * dpuf_oracle.c - CPU restatement of DPUF's mode-12 per-token language-model loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA engine: it is
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg, never by
 * the product.  It restates, in plain scalar C, the arithmetic of the reference engine with
 * the reference's exact fp32 operation order, so that results are bit-identical:
 *
 *   - AVX2 8-lane reductions are emulated lane by lane: lane j accumulates elements
 *     i = j, j+8, j+16, ... and the horizontal sums use the reference's two trees
 *       hsum8_split  ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))   eng_hsum256_ps  dpuf_engine.c:37-46
 *       hsum8_pairs  ((l0+l1)+(l2+l3)) + ((l4+l5)+(l6+l7))   hsum4_256_ps    dpuf_engine.c:318-323
 *   - every fused multiply-add of the reference (_mm256_fmadd/fmsub/fnmadd) is an explicit
 *     fmaf(); nothing else is contracted (build with -ffp-contract=off).
 *
 * Pinned against the reference itself: tests/golden/ holds outputs of the reference library
 * (built from its sources by oracle/build_ref.sh) for seeded models, and the oracle must
 * reproduce them bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/dpuf_kernels.h"

#define ORC_EXPORT __attribute__((visibility("default")))
#define ORC_MAX_BATCH 256

/* ------------------------------------------------------------------ scalar helpers */

static float f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t x;
    if (ex == 0) {
        if (man == 0) {
            x = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (ex == 31) {
        x = sign | 0x7F800000u | (man << 13);
    } else {
        x = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static float hsum8_split(const float* l) {
    float a0 = l[0] + l[4], a1 = l[1] + l[5], a2 = l[2] + l[6], a3 = l[3] + l[7];
    return (a0 + a1) + (a2 + a3);
}

static float hsum8_pairs(const float* l) {
    return ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
}

static float maxf_ps(float a, float b) { return (a > b) ? a : b; } /* _mm_max_ps(a,b) for non-NaN */
static float minf_ps(float a, float b) { return (a < b) ? a : b; }

/* The reference's exp approximation eng_avx2_exp_ps (dpuf_engine.c:297-316), one lane. */
static float exp_poly(float x) {
    x = maxf_ps(-45.0f, minf_ps(x, 45.0f));
    float fx = rintf(x * 1.44269504088896341f);
    float r = fmaf(-fx, 0.693359375f, x);
    r = fmaf(-fx, -2.12194440e-4f, r);
    float p = 1.9875691500e-4f;
    p = fmaf(p, r, 1.3981999507e-3f);
    p = fmaf(p, r, 8.3334519073e-3f);
    p = fmaf(p, r, 4.1665795894e-2f);
    p = fmaf(p, r, 1.6666665459e-1f);
    p = fmaf(p, r, 5.0000001201e-1f);
    float r2 = r * r;
    float er = fmaf(p, r2, r) + 1.0f;
    int32_t n = (int32_t)fx;
    uint32_t bits = (uint32_t)(n + 127) << 23;
    float sc;
    memcpy(&sc, &bits, 4);
    return er * sc;
}

/* ------------------------------------------------------------------ mode-12 prep */

/* Orthonormal FWHT of 64 values: strides 1..32 ascending, then x0.125
 * (fwht64_block_f32, dpuf_avx2.c:724-772; any ascending-stride order is bit-identical). */
static void fwht64(float* y) {
    for (int h = 1; h < 64; h <<= 1)
        for (int g = 0; g < 64; g += 2 * h)
            for (int i = g; i < g + h; i++) {
                float a = y[i], b = y[i + h];
                y[i] = a + b;
                y[i + h] = a - b;
            }
    for (int i = 0; i < 64; i++) y[i] = y[i] * 0.125f;
}

/* x -> sign flip -> FWHT-64 -> per-32 int8 quantisation (dpuf_prep_had4_packed_slab,
 * dpuf_avx2.c:2364-2449, plain layout).  q[cols], xs[cols/32], xsum8[cols/32]. */
ORC_EXPORT void orc_prep_mode12(int32_t cols, const float* x, const uint8_t* sign_bits,
                                int8_t* q, float* xs, int32_t* xsum8) {
    float* f = (float*)malloc((size_t)cols * sizeof(float));
    for (int32_t c = 0; c < cols; c++) {
        int neg = sign_bits ? ((sign_bits[c >> 3] >> (c & 7)) & 1) : 0;
        f[c] = neg ? -x[c] : x[c];
    }
    for (int32_t c = 0; c < cols; c += 64) fwht64(f + c);
    for (int32_t b = 0; b < (cols >> 5); b++) {
        const float* v = f + (size_t)b * 32u;
        float amax = 0.0f;
        for (int k = 0; k < 32; k++) amax = maxf_ps(amax, fabsf(v[k]));
        if (amax <= 1e-4f) {
            xs[b] = 0.0f;
            xsum8[b] = 0;
            memset(q + (size_t)b * 32u, 0, 32);
            continue;
        }
        float d = amax / 127.0f;
        float inv = (amax > 1e-12f) ? (127.0f / amax) : 0.0f;
        int32_t s = 0;
        for (int k = 0; k < 32; k++) {
            float t = rintf(v[k] * inv);
            int32_t qi = (int32_t)t;
            if (qi > 127) qi = 127;   /* signed saturation of the two packs */
            if (qi < -127) qi = -127; /* max_epi8 with -127 */
            q[(size_t)b * 32u + (size_t)k] = (int8_t)qi;
            s += qi;
        }
        xs[b] = d;
        xsum8[b] = s * 8;
    }
    free(f);
}

/* ------------------------------------------------------------------ mode-12 matvec */

/* out[r] for tiles [t0, t1): per row, acc = fma(float(dot_b - xsum8_b), ws_b * xs_b, acc)
 * over blocks b ascending, blocks with xs_b <= 0 skipped (dpuf_avx2.c:2601-2640).  The
 * integer dot is exact; dot_b = sum_k u_k * q_k with the stored nibble u = w + 8. */
static void matvec_tiles(int32_t cols, const uint8_t* tensor_base, const uint64_t* tile_offsets,
                         int32_t t0, int32_t t1, const int8_t* q, const float* xs, const int32_t* xsum8,
                         float* out) {
    const int32_t n_blk = cols >> 5;
    #pragma omp parallel for schedule(static)
    for (int32_t t = t0; t < t1; t++) {
        const uint8_t* tp = tensor_base + tile_offsets[t];
        int32_t n_r = (int32_t)(tp[4] | (tp[5] << 8));
        for (int32_t lr = 0; lr < n_r; lr++) {
            int32_t rg = lr >> 3, ri = lr & 7;
            const uint8_t* grp = tp + 16 + (size_t)rg * (size_t)n_blk * 144u;
            const uint8_t* sc = grp;
            const uint8_t* qg = grp + (size_t)n_blk * 16u;
            float acc = 0.0f;
            for (int32_t b = 0; b < n_blk; b++) {
                float bs = xs[b];
                if (bs <= 0.0f) continue;
                const uint8_t* qb = qg + (size_t)b * 128u;
                const int8_t* xb = q + (size_t)b * 32u;
                int32_t dot = 0;
                for (int c = 0; c < 4; c++)
                    for (int k = 0; k < 4; k++) {
                        uint8_t byte = qb[c * 32 + ri * 4 + k];
                        dot += (int32_t)(byte & 0x0F) * xb[c * 8 + k];
                        dot += (int32_t)(byte >> 4) * xb[c * 8 + 4 + k];
                    }
                dot -= xsum8[b];
                uint16_t hs = (uint16_t)(sc[(size_t)b * 16u + (size_t)ri * 2u] |
                                         (sc[(size_t)b * 16u + (size_t)ri * 2u + 1u] << 8));
                float s = f16_to_f32(hs) * bs;
                acc = fmaf((float)dot, s, acc);
            }
            out[t * 16 + lr] = acc;
        }
    }
}

/* Standalone op with the reference signature (dpuf_avx2.c:2678-2736). */
ORC_EXPORT void orc_matmul_mode12_f32(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                      const float* x_in, const uint8_t* tensor_base,
                                      const uint64_t* tile_offsets, const uint8_t* sign_bits, float* out) {
    int32_t n_blk = cols >> 5;
    int8_t* q = (int8_t*)malloc((size_t)cols);
    float* xs = (float*)malloc((size_t)n_blk * sizeof(float));
    int32_t* xm = (int32_t*)malloc((size_t)n_blk * sizeof(int32_t));
    for (int32_t m = 0; m < M; m++) {
        orc_prep_mode12(cols, x_in + (size_t)m * (size_t)cols, sign_bits, q, xs, xm);
        matvec_tiles(cols, tensor_base, tile_offsets, 0, n_tiles, q, xs, xm, out + (size_t)m * (size_t)rows);
    }
    free(q); free(xs); free(xm);
}

/* Modes 13 (QR_HAD4_ASYM) and 14 (QR_HAD6): dpuf_matmul_qr_had4_asym_f32 / _had6_f32
 * (dpuf_avx2.c:3084-3144, had_asym_tile_range_impl :2947-3066).  Same activation prep as mode 12
 * (dpuf_prep_had4_packed_slab).  A tile is a 16-byte header and, per 8-row group, n64 x
 * [8 fp16 d | 8 fp16 m] (per 64-block), then per 32-block 128 bytes of nibbles ordered
 * [chunk c][row r][e] (low nibble: weight of x[8c+e], high: x[8c+4+e]), then (mode 14) per
 * 32-block 64 bytes of high bit pairs (byte c*16 + half*8 + (r%2)*4 + e, bits 2*(r/2)).  The
 * block dots are exact integers (no int16 saturation or wrap at these ranges).  Per row and
 * 64-block g, in order: fdot = fma(d0, xs0, d1 * xs1), acc = fma(fdot, d, acc),
 * acc = fma(m, xm_s, acc) with xm_s = fma(xsum0, xs0, xsum1 * xs1) * 0.125: the reference's
 * scalar "(xsum0 * xs0 + xsum1 * xs1) * 0.125f" as its build (gcc, gnu11, -mfma: contraction
 * on by default) computes it - checked against the built reference, which the other two
 * orders do not match. */
static void had_tiles(int32_t is_had6, int32_t cols, const uint8_t* tensor_base, const uint64_t* tile_offsets,
                      int32_t t0, int32_t t1, const int8_t* q, const float* xs, const int32_t* xm, float* out) {
    const int32_t n_64 = cols >> 6;
    const size_t grp_bytes = is_had6 ? 416u : 288u;
    {
        for (int32_t t = t0; t < t1; t++) {
            const uint8_t* tp = tensor_base + tile_offsets[t];
            const int32_t n_r = tp[4] | (tp[5] << 8);
            for (int32_t rg = 0; rg * 8 < n_r; rg++) {
                const uint8_t* grp = tp + 16 + (size_t)rg * (size_t)n_64 * grp_bytes;
                const uint16_t* dm = (const uint16_t*)grp;
                const uint8_t* q4 = grp + (size_t)n_64 * 32u;
                const uint8_t* q2 = q4 + (size_t)n_64 * 256u;
                for (int32_t r = 0; r < 8 && rg * 8 + r < n_r; r++) {
                    float acc = 0.0f;
                    for (int32_t g = 0; g < n_64; g++) {
                        int32_t d[2];
                        for (int k = 0; k < 2; k++) {
                            const int32_t b = 2 * g + k;
                            int32_t dot = 0;
                            for (int c = 0; c < 4; c++)
                                for (int e = 0; e < 4; e++) {
                                    const uint8_t byte = q4[(size_t)b * 128u + c * 32 + r * 4 + e];
                                    int32_t ulo = byte & 15, uhi = byte >> 4;
                                    if (is_had6) {
                                        const int sh = 2 * (r >> 1);
                                        const uint8_t* hp = q2 + (size_t)b * 64u + c * 16 + (r & 1) * 4 + e;
                                        ulo |= ((hp[0] >> sh) & 3) << 4;
                                        uhi |= ((hp[8] >> sh) & 3) << 4;
                                    }
                                    dot += ulo * q[b * 32 + c * 8 + e] + uhi * q[b * 32 + c * 8 + 4 + e];
                                }
                            d[k] = dot;
                        }
                        const int32_t b0 = 2 * g, b1 = b0 + 1;
                        const float fdot = fmaf((float)d[0], xs[b0], (float)d[1] * xs[b1]);
                        const float xms = fmaf((float)xm[b0], xs[b0], (float)xm[b1] * xs[b1]) * 0.125f;
                        acc = fmaf(fdot, f16_to_f32(dm[g * 16 + r]), acc);
                        acc = fmaf(f16_to_f32(dm[g * 16 + 8 + r]), xms, acc);
                    }
                    out[(size_t)t * 16 + rg * 8 + r] = acc;
                }
            }
        }
    }
}

ORC_EXPORT void orc_matmul_had_asym_f32(int32_t is_had6, int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                        const float* x_in, const uint8_t* tensor_base,
                                        const uint64_t* tile_offsets, const uint8_t* sign_bits, float* out) {
    const int32_t n_blk = cols >> 5;
    int8_t* q = (int8_t*)malloc((size_t)cols);
    float* xs = (float*)malloc((size_t)n_blk * sizeof(float));
    int32_t* xm = (int32_t*)malloc((size_t)n_blk * sizeof(int32_t));
    for (int32_t m = 0; m < M; m++) {
        orc_prep_mode12(cols, x_in + (size_t)m * (size_t)cols, sign_bits, q, xs, xm);
        had_tiles(is_had6, cols, tensor_base, tile_offsets, 0, n_tiles, q, xs, xm, out + (size_t)m * (size_t)rows);
    }
    free(q); free(xs); free(xm);
}

/* Row lookup: nibbles -> (u-8)*ws -> FWHT-64 -> sign (dpuf_avx2.c:2738-2783). */
ORC_EXPORT void orc_embed_mode12_f32(int32_t n_tokens, int32_t cols, const int32_t* ids,
                                     const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                     const uint8_t* sign_bits, float* out) {
    const int32_t n_blk = cols >> 5;
    for (int32_t tok = 0; tok < n_tokens; tok++) {
        int32_t r = ids[tok];
        int32_t t = r / 16, lr = r % 16, rg = lr >> 3, ri = lr & 7;
        const uint8_t* grp = tensor_base + tile_offsets[t] + 16 + (size_t)rg * (size_t)n_blk * 144u;
        const uint8_t* qg = grp + (size_t)n_blk * 16u;
        float* dst = out + (size_t)tok * (size_t)cols;
        for (int32_t b = 0; b < n_blk; b++) {
            uint16_t hs = (uint16_t)(grp[(size_t)b * 16u + (size_t)ri * 2u] | (grp[(size_t)b * 16u + (size_t)ri * 2u + 1u] << 8));
            float ws = f16_to_f32(hs);
            for (int c = 0; c < 4; c++)
                for (int k = 0; k < 4; k++) {
                    uint8_t byte = qg[(size_t)b * 128u + (size_t)c * 32u + (size_t)ri * 4u + (size_t)k];
                    dst[b * 32 + c * 8 + k] = (float)((int32_t)(byte & 0x0F) - 8) * ws;
                    dst[b * 32 + c * 8 + 4 + k] = (float)((int32_t)(byte >> 4) - 8) * ws;
                }
        }
        for (int32_t c = 0; c < cols; c += 64) fwht64(dst + c);
        if (sign_bits)
            for (int32_t c = 0; c < cols; c++)
                if ((sign_bits[c >> 3] >> (c & 7)) & 1) dst[c] = -dst[c];
    }
}

/* Mode 13 / 14 row lookup (embed_qr_had_asym_impl, dpuf_avx2.c:3146-3221): per 64-block the
 * row's d and m, per element v = q * d + m, then FWHT-64 and the column signs.  q * d is exact
 * (q < 64, d an fp16: at most 17 significant bits), so a fused multiply-add gives the same
 * bits. */
ORC_EXPORT void orc_embed_had_asym_f32(int32_t is_had6, int32_t n_tokens, int32_t cols, const int32_t* ids,
                                       const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                       const uint8_t* sign_bits, float* out) {
    const int32_t n_64 = cols >> 6;
    const size_t grp_bytes = is_had6 ? 416u : 288u;
    for (int32_t tok = 0; tok < n_tokens; tok++) {
        const int32_t r = ids[tok], t = r / 16, lr = r % 16, rg = lr >> 3, ri = lr & 7;
        const uint8_t* grp = tensor_base + tile_offsets[t] + 16 + (size_t)rg * (size_t)n_64 * grp_bytes;
        const uint16_t* dm = (const uint16_t*)grp;
        const uint8_t* q4 = grp + (size_t)n_64 * 32u;
        const uint8_t* q2 = q4 + (size_t)n_64 * 256u;
        float* dst = out + (size_t)tok * (size_t)cols;
        for (int32_t g = 0; g < n_64; g++) {
            const float wd = f16_to_f32(dm[g * 16 + ri]), wm = f16_to_f32(dm[g * 16 + 8 + ri]);
            for (int k2 = 0; k2 < 2; k2++) {
                const int32_t b = 2 * g + k2;
                for (int c = 0; c < 4; c++)
                    for (int e = 0; e < 4; e++) {
                        const uint8_t byte = q4[(size_t)b * 128u + c * 32 + ri * 4 + e];
                        int32_t ulo = byte & 15, uhi = byte >> 4;
                        if (is_had6) {
                            const uint8_t* hp = q2 + (size_t)b * 64u + c * 16 + (ri & 1) * 4 + e;
                            ulo |= ((hp[0] >> (2 * (ri >> 1))) & 3) << 4;
                            uhi |= ((hp[8] >> (2 * (ri >> 1))) & 3) << 4;
                        }
                        float* d0 = dst + b * 32 + c * 8 + e;
                        d0[0] = (float)ulo * wd + wm;
                        d0[4] = (float)uhi * wd + wm;
                    }
            }
        }
        for (int32_t c = 0; c < cols; c += 64) fwht64(dst + c);
        if (sign_bits)
            for (int32_t c = 0; c < cols; c++)
                if ((sign_bits[c >> 3] >> (c & 7)) & 1) dst[c] = -dst[c];
    }
}

/* ------------------------------------------------------------------ pointwise ops */

/* x += res (if res); out = (x * inv) * w, inv = 1/sqrt(ss/n + eps) with ss the 8-lane fma
 * sum of squares (rms_norm_f32 / add_and_rms_norm_f32, dpuf_engine.c:225-272). */
ORC_EXPORT void orc_add_rmsnorm(int32_t n, float* x, const float* res, const float* w, float eps, float* out) {
    float lane[8] = {0};
    int32_t i = 0;
    for (; i + 7 < n; i += 8)
        for (int j = 0; j < 8; j++) {
            float s = res ? (x[i + j] + res[i + j]) : x[i + j];
            x[i + j] = s;
            lane[j] = fmaf(s, s, lane[j]);
        }
    float ss = hsum8_split(lane);
    for (; i < n; i++) {
        float s = res ? (x[i] + res[i]) : x[i];
        x[i] = s;
        ss += s * s;
    }
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (i = 0; i < n; i++) out[i] = (x[i] * inv) * w[i];
}

/* NeoX rotate-half with host tables (apply_rope_neox_f32, dpuf_engine.c:274-295). */
static void rope_apply(int32_t hd, float* v, const float* cs, const float* sn) {
    int32_t half = hd >> 1, j = 0;
    for (; j + 7 < half; j += 8)
        for (int l = 0; l < 8; l++) {
            float x1 = v[j + l], x2 = v[j + l + half], c = cs[j + l], s = sn[j + l];
            v[j + l] = fmaf(x1, c, -(x2 * s));
            v[j + l + half] = fmaf(x2, c, x1 * s);
        }
    for (; j < half; j++) {
        float x1 = v[j], x2 = v[j + half], c = cs[j], s = sn[j];
        v[j] = x1 * c - x2 * s;
        v[j + half] = x2 * c + x1 * s;
    }
}

/* Host RoPE tables (precompute_rope, dpuf_engine.c:183-223), same libm calls. */
ORC_EXPORT void orc_rope_tables(const DpufModelConfig* cfg, float* cos_tab, float* sin_tab) {
    int32_t hd = cfg->head_dim, half = hd >> 1;
    float* inv_freq = (float*)malloc((size_t)half * sizeof(float));
    for (int32_t j = 0; j < half; j++) {
        float freq = 1.0f / powf(cfg->rope_theta, (float)(2 * j) / (float)hd);
        if (cfg->use_llama3_rope) {
            float factor = cfg->rope_factor, low_f = cfg->rope_low_freq, high_f = cfg->rope_high_freq;
            float orig = (float)cfg->rope_orig_max_pos;
            float wavelen = (2.0f * (float)3.14159265358979323846) / freq;
            float low_w = orig / low_f, high_w = orig / high_f;
            if (wavelen > low_w) {
                freq /= factor;
            } else if (wavelen >= high_w) {
                float smooth = (orig / wavelen - low_f) / (high_f - low_f);
                freq = (1.0f - smooth) * (freq / factor) + smooth * freq;
            }
        }
        inv_freq[j] = freq;
    }
    for (int32_t p = 0; p < cfg->max_seq_len; p++) {
        float pf = (float)p;
        for (int32_t j = 0; j < half; j++) {
            float ang = pf * inv_freq[j];
            cos_tab[(size_t)p * half + j] = cosf(ang);
            sin_tab[(size_t)p * half + j] = sinf(ang);
        }
    }
    free(inv_freq);
}

/* SwiGLU with dead-zone for element idx of a flat [M*I] range split over nt threads
 * (swiglu_range_avx2, dpuf_engine.c:967-997, called at :1982-2016).  `vec` selects the
 * 8-wide vector formula vs the scalar tail formula. */
static float swiglu_vec(float g, float u, float dz) {
    float ng = maxf_ps(-40.0f, minf_ps(0.0f - g, 40.0f));
    float silu = g / (1.0f + exp_poly(ng));
    float r = silu * u;
    if (dz > 0.0f && !(fabsf(r) >= dz)) r = 0.0f;
    return r;
}

static float swiglu_scalar(float g, float u, float dz) {
    float silu = (g >= 40.0f) ? g : ((g <= -40.0f) ? 0.0f : (g / (1.0f + expf(-g))));
    float v = silu * u;
    if (dz > 0.0f && fabsf(v) < dz) v = 0.0f;
    return v;
}

/* Which formula the reference applies to flat element idx (total elements, nt threads). */
ORC_EXPORT int32_t orc_swiglu_is_vector(int64_t idx, int64_t total, int32_t nt) {
    int64_t tid = (idx * nt) / total; /* first guess, then fix up */
    while (tid > 0 && (total * tid) / nt > idx) tid--;
    while (tid + 1 < nt && (total * (tid + 1)) / nt <= idx) tid++;
    int64_t s0 = (total * tid) / nt, s1 = (total * (tid + 1)) / nt;
    return (idx - s0) < ((s1 - s0) & ~(int64_t)7);
}

/* ------------------------------------------------------------------ attention */

/* Causal attention of one token for the Q heads of one KV head (gqa_attn_head_pair_f32,
 * dpuf_engine.c:341-577): heads are taken in pairs (the pair path); an odd last head uses the
 * single-head path, whose score tail and PV order differ. */
static void attn_pair(int32_t hd, int32_t kv_len, float scale, const float* kc, const float* vc,
                      const float* q0, const float* q1, float* sc0, float* sc1, float* o0, float* o1) {
    int32_t t = 0;
    float mx0 = -1e30f, mx1 = -1e30f;
    if (q1 && (hd & 7) == 0) {
        for (; t + 3 < kv_len; t += 4) {
            for (int kk = 0; kk < 4; kk++) {
                const float* kp = kc + (size_t)(t + kk) * (size_t)hd;
                float a[8] = {0}, b[8] = {0};
                for (int32_t i = 0; i < hd; i += 8)
                    for (int l = 0; l < 8; l++) {
                        a[l] = fmaf(q0[i + l], kp[i + l], a[l]);
                        b[l] = fmaf(q1[i + l], kp[i + l], b[l]);
                    }
                sc0[t + kk] = hsum8_pairs(a) * scale;
                sc1[t + kk] = hsum8_pairs(b) * scale;
                mx0 = maxf_ps(mx0, sc0[t + kk]);
                mx1 = maxf_ps(mx1, sc1[t + kk]);
            }
        }
        for (; t < kv_len; t++) {
            const float* kp = kc + (size_t)t * (size_t)hd;
            float a[8] = {0}, b[8] = {0};
            for (int32_t i = 0; i < hd; i += 8)
                for (int l = 0; l < 8; l++) {
                    a[l] = fmaf(q0[i + l], kp[i + l], a[l]);
                    b[l] = fmaf(q1[i + l], kp[i + l], b[l]);
                }
            float s0 = hsum8_split(a) * scale, s1 = hsum8_split(b) * scale;
            sc0[t] = s0; if (s0 > mx0) mx0 = s0;
            sc1[t] = s1; if (s1 > mx1) mx1 = s1;
        }
        float* scs[2] = {sc0, sc1};
        float mxs[2] = {mx0, mx1};
        for (int h = 0; h < 2; h++) {
            float* s = scs[h];
            float lane[8] = {0};
            int32_t k = 0;
            for (; k + 7 < kv_len; k += 8)
                for (int l = 0; l < 8; l++) {
                    float e = exp_poly(s[k + l] - mxs[h]);
                    s[k + l] = e;
                    lane[l] = lane[l] + e;
                }
            float sp = hsum8_split(lane);
            for (; k < kv_len; k++) { float e = expf(s[k] - mxs[h]); s[k] = e; sp += e; }
            float inv = 1.0f / (sp + 1e-12f);
            for (k = 0; k < kv_len; k++) s[k] = s[k] * inv;
        }
        for (int32_t d = 0; d < hd; d++) {
            float a = 0.0f, b = 0.0f;
            for (int32_t k = 0; k < kv_len; k++) {
                float v = vc[(size_t)k * (size_t)hd + (size_t)d];
                a = fmaf(sc0[k], v, a);
                b = fmaf(sc1[k], v, b);
            }
            o0[d] = a;
            o1[d] = b;
        }
        return;
    }
    /* single head */
    if ((hd & 7) == 0) {
        for (; t + 3 < kv_len; t += 4)
            for (int kk = 0; kk < 4; kk++) {
                const float* kp = kc + (size_t)(t + kk) * (size_t)hd;
                float a[8] = {0};
                for (int32_t i = 0; i < hd; i += 8)
                    for (int l = 0; l < 8; l++) a[l] = fmaf(q0[i + l], kp[i + l], a[l]);
                sc0[t + kk] = hsum8_pairs(a) * scale;
                mx0 = maxf_ps(mx0, sc0[t + kk]);
            }
    }
    for (; t < kv_len; t++) {
        /* dot_f32_avx2 (dpuf_engine.c:325-339): two 8-lane accumulators over 16-wide steps */
        const float* kp = kc + (size_t)t * (size_t)hd;
        float a0[8] = {0}, a1[8] = {0};
        int32_t i = 0;
        for (; i + 15 < hd; i += 16)
            for (int l = 0; l < 8; l++) {
                a0[l] = fmaf(q0[i + l], kp[i + l], a0[l]);
                a1[l] = fmaf(q0[i + 8 + l], kp[i + 8 + l], a1[l]);
            }
        for (; i + 7 < hd; i += 8)
            for (int l = 0; l < 8; l++) a0[l] = fmaf(q0[i + l], kp[i + l], a0[l]);
        float sum[8];
        for (int l = 0; l < 8; l++) sum[l] = a0[l] + a1[l];
        float s = hsum8_split(sum);
        for (; i < hd; i++) s += q0[i] * kp[i];
        s = s * scale;
        sc0[t] = s;
        if (s > mx0) mx0 = s;
    }
    {
        float lane[8] = {0};
        int32_t k = 0;
        for (; k + 7 < kv_len; k += 8)
            for (int l = 0; l < 8; l++) {
                float e = exp_poly(sc0[k + l] - mx0);
                sc0[k + l] = e;
                lane[l] = lane[l] + e;
            }
        float sp = hsum8_split(lane);
        for (; k < kv_len; k++) { float e = expf(sc0[k] - mx0); sc0[k] = e; sp += e; }
        float inv = 1.0f / (sp + 1e-12f);
        for (k = 0; k < kv_len; k++) sc0[k] = sc0[k] * inv;
    }
    if ((hd & 63) == 0) {
        for (int32_t d = 0; d < hd; d++) {
            float a = 0.0f;
            int32_t k = 0;
            for (; k + 1 < kv_len; k += 2) {
                float t1 = fmaf(sc0[k + 1], vc[(size_t)(k + 1) * (size_t)hd + (size_t)d], a);
                a = fmaf(sc0[k], vc[(size_t)k * (size_t)hd + (size_t)d], t1);
            }
            if (k < kv_len) a = fmaf(sc0[k], vc[(size_t)k * (size_t)hd + (size_t)d], a);
            o0[d] = a;
        }
    } else {
        for (int32_t d = 0; d < hd; d++) o0[d] = 0.0f;
        int32_t hd8 = hd & ~7;
        for (int32_t k = 0; k < kv_len; k++) {
            const float* vp = vc + (size_t)k * (size_t)hd;
            for (int32_t d = 0; d < hd8; d++) o0[d] = fmaf(sc0[k], vp[d], o0[d]);
            for (int32_t d = hd8; d < hd; d++) o0[d] += sc0[k] * vp[d];
        }
    }
}

/* ------------------------------------------------------------------ Q8 KV cache (kv_type 1) */

/* _mm256_cvtps_epi32 (round to nearest even) followed by the saturating packs and the
 * max(-127) of quantize_vec_q8_blk32: a NaN or out-of-range product becomes the x86 "integer
 * indefinite" INT32_MIN, i.e. -127 after saturation. */
static int8_t q8_cvt(float y) {
    if (!(y == y) || y >= 2147483648.0f || y < -2147483648.0f) return -127;
    float r = nearbyintf(y);
    if (r > 127.0f) return 127;
    if (r < -127.0f) return -127;
    return (int8_t)r;
}

/* quantize_vec_q8_blk32 (dpuf_engine.c:751-781): per 32-element block, amax by the reference's
 * max tree (lanes j, j+8, j+16, j+24; then the 4-wide and 2-wide folds), scale = amax / 127,
 * q = cvt(x * (127 / amax)), or 0 when amax <= 1e-12. */
ORC_EXPORT void orc_quantize_q8_blk32(int32_t n, const float* src, int8_t* dst, float* scales) {
    for (int32_t b = 0; b < (n >> 5); b++) {
        const float* x = src + (b << 5);
        float ln[8];
        for (int l = 0; l < 8; l++)
            ln[l] = maxf_ps(maxf_ps(fabsf(x[l]), fabsf(x[8 + l])), maxf_ps(fabsf(x[16 + l]), fabsf(x[24 + l])));
        float m4[4];
        for (int l = 0; l < 4; l++) m4[l] = maxf_ps(ln[l], ln[4 + l]);
        float amax = maxf_ps(maxf_ps(m4[0], m4[2]), maxf_ps(m4[1], m4[3]));
        scales[b] = amax / 127.0f;
        float inv = (amax > 1e-12f) ? (127.0f / amax) : 0.0f;
        for (int i = 0; i < 32; i++) dst[(b << 5) + i] = q8_cvt(x[i] * inv);
    }
}

/* dot_f32_q8_blk32_avx2 (dpuf_engine.c:603-619): per block two lane accumulators (elements
 * l, l+16 and l+8, l+24), their sum times the block scale fused into the total; split tree. */
static float dot_q8_blk32(int32_t n, const float* q, const int8_t* kq, const float* ks) {
    float tot[8] = {0};
    for (int32_t b = 0; b < (n >> 5); b++) {
        const int32_t c0 = b << 5;
        for (int l = 0; l < 8; l++) {
            float a0 = fmaf(q[c0 + l], (float)kq[c0 + l], 0.0f);
            float a1 = fmaf(q[c0 + 8 + l], (float)kq[c0 + 8 + l], 0.0f);
            a0 = fmaf(q[c0 + 16 + l], (float)kq[c0 + 16 + l], a0);
            a1 = fmaf(q[c0 + 24 + l], (float)kq[c0 + 24 + l], a1);
            tot[l] = fmaf(a0 + a1, ks[b], tot[l]);
        }
    }
    return hsum8_split(tot);
}

/* vec_softmax_avx2 (dpuf_engine.c:579-601). */
static void softmax_ref(int32_t n, float* s, float mx) {
    float lane[8] = {0};
    int32_t k = 0;
    for (; k + 7 < n; k += 8)
        for (int l = 0; l < 8; l++) {
            float e = exp_poly(s[k + l] - mx);
            s[k + l] = e;
            lane[l] = lane[l] + e;
        }
    float sp = hsum8_split(lane);
    for (; k < n; k++) { float e = expf(s[k] - mx); s[k] = e; sp += e; }
    float inv = 1.0f / (sp + 1e-12f);
    for (k = 0; k < n; k++) s[k] = s[k] * inv;
}

/* gqa_attn_head_pair_q8 (dpuf_engine.c:621-749) over one KV head's int8 rows kc/vc [.][hd] and
 * block scales ksc/vsc [.][hd/32].  Pair path: keys two at a time, per block and lane
 * t = fma(q[l], k[l], fma(q[l+8], k[l+8], t)) over the two 16-wide halves, then the block
 * scale fused into the lane sum, pairs tree; an odd last key and the lone head use
 * dot_q8_blk32.  PV per output d: fma(p_k * vs_k[d/32], v_kd, acc) over k ascending. */
static void attn_pair_q8(int32_t hd, int32_t kv_len, float scale, const int8_t* kc, const float* ksc,
                         const int8_t* vc, const float* vsc, const float* q0, const float* q1, float* sc0,
                         float* sc1, float* o0, float* o1) {
    const int32_t nb = hd >> 5;
    float mx0 = -1e30f, mx1 = -1e30f;
    int32_t t = 0;
    if (q1) {
        for (; t + 1 < kv_len; t += 2) {
            float d[2][2];
            for (int kk = 0; kk < 2; kk++) {
                const int8_t* kp = kc + (size_t)(t + kk) * (size_t)hd;
                const float* ks = ksc + (size_t)(t + kk) * (size_t)nb;
                float a[8] = {0}, b[8] = {0};
                for (int32_t bl = 0; bl < nb; bl++) {
                    const int32_t c0 = bl << 5;
                    for (int l = 0; l < 8; l++) {
                        float ta = 0.0f, tb = 0.0f;
                        for (int j = 0; j < 32; j += 16) {
                            float fl = (float)kp[c0 + j + l], fh = (float)kp[c0 + j + 8 + l];
                            ta = fmaf(q0[c0 + j + l], fl, fmaf(q0[c0 + j + 8 + l], fh, ta));
                            tb = fmaf(q1[c0 + j + l], fl, fmaf(q1[c0 + j + 8 + l], fh, tb));
                        }
                        a[l] = fmaf(ta, ks[bl], a[l]);
                        b[l] = fmaf(tb, ks[bl], b[l]);
                    }
                }
                d[0][kk] = hsum8_pairs(a) * scale;
                d[1][kk] = hsum8_pairs(b) * scale;
            }
            sc0[t] = d[0][0]; sc0[t + 1] = d[0][1];
            sc1[t] = d[1][0]; sc1[t + 1] = d[1][1];
            mx0 = maxf_ps(mx0, (d[0][0] > d[0][1]) ? d[0][0] : d[0][1]);
            mx1 = maxf_ps(mx1, (d[1][0] > d[1][1]) ? d[1][0] : d[1][1]);
        }
        for (; t < kv_len; t++) {
            float s0 = dot_q8_blk32(hd, q0, kc + (size_t)t * hd, ksc + (size_t)t * nb) * scale;
            float s1 = dot_q8_blk32(hd, q1, kc + (size_t)t * hd, ksc + (size_t)t * nb) * scale;
            sc0[t] = s0; if (s0 > mx0) mx0 = s0;
            sc1[t] = s1; if (s1 > mx1) mx1 = s1;
        }
        softmax_ref(kv_len, sc0, mx0);
        softmax_ref(kv_len, sc1, mx1);
    } else {
        for (; t < kv_len; t++) {
            float s = dot_q8_blk32(hd, q0, kc + (size_t)t * hd, ksc + (size_t)t * nb) * scale;
            sc0[t] = s;
            if (s > mx0) mx0 = s;
        }
        softmax_ref(kv_len, sc0, mx0);
    }
    for (int32_t dd = 0; dd < hd; dd++) {
        const int32_t bl = dd >> 5;
        float a = 0.0f, b = 0.0f;
        for (int32_t k = 0; k < kv_len; k++) {
            const float vs = vsc[(size_t)k * nb + bl];
            const float v = (float)vc[(size_t)k * hd + dd];
            a = fmaf(sc0[k] * vs, v, a);
            if (q1) b = fmaf(sc1[k] * vs, v, b);
        }
        o0[dd] = a;
        if (q1) o1[dd] = b;
    }
}

/* ------------------------------------------------------------------ engine */

typedef struct {
    DpufModelConfig cfg;
    DpufLayerWeights* layers;
    DpufWeightDesc tok, lm;
    const float* out_norm;
    float *cos_tab, *sin_tab;
    float *k_cache, *v_cache; /* [L][n_kv][max_seq][hd] */
    int8_t *k_q8, *v_q8;      /* kv_type 1: [L][n_kv][max_seq][hd] and block scales */
    float *k_sc, *v_sc;       /* [L][n_kv][max_seq][hd/32] */
    float *h, *hn, *q, *k, *v, *att, *gate, *up, *ffn;
    int8_t* pq;
    float* pxs;
    int32_t* pxm;
    float *sc0, *sc1;
    float deadzone;
    int32_t nt;
} OrcEngine;

ORC_EXPORT void* orc_engine_create(const DpufModelConfig* cfg, const DpufLayerWeights* layers,
                                   const DpufWeightDesc* tok, const DpufWeightDesc* lm, const float* out_norm) {
    if (!cfg || !layers || !tok || !lm || !out_norm) return NULL;
    OrcEngine* e = (OrcEngine*)calloc(1, sizeof(OrcEngine));
    e->cfg = *cfg;
    e->layers = (DpufLayerWeights*)malloc((size_t)cfg->num_layers * sizeof(DpufLayerWeights));
    memcpy(e->layers, layers, (size_t)cfg->num_layers * sizeof(DpufLayerWeights));
    e->tok = *tok;
    e->lm = *lm;
    e->out_norm = out_norm;
    const char* dz = getenv("DPUF_SWIGLU_DEADZONE");
    e->deadzone = dz ? (float)atof(dz) : 0.005f;
    e->nt = cfg->n_threads <= 0 ? 8 : (cfg->n_threads > 32 ? 32 : cfg->n_threads);
    int32_t H = cfg->hidden_size, I = cfg->intermediate_size, hd = cfg->head_dim;
    int32_t qd = cfg->num_q_heads * hd, kvd = cfg->num_kv_heads * hd, S = cfg->max_seq_len;
    int32_t mx = H > I ? H : I;
    if (qd > mx) mx = qd;
    size_t B = ORC_MAX_BATCH;
    e->cos_tab = (float*)malloc((size_t)S * (hd / 2) * sizeof(float));
    e->sin_tab = (float*)malloc((size_t)S * (hd / 2) * sizeof(float));
    orc_rope_tables(cfg, e->cos_tab, e->sin_tab);
    size_t kv = (size_t)cfg->num_layers * (size_t)S * (size_t)kvd;
    e->k_cache = (float*)calloc(kv, sizeof(float));
    e->v_cache = (float*)calloc(kv, sizeof(float));
    if (cfg->kv_type == DPUF_KV_Q8) {
        e->k_q8 = (int8_t*)calloc(kv, 1);
        e->v_q8 = (int8_t*)calloc(kv, 1);
        e->k_sc = (float*)calloc(kv / 32, sizeof(float));
        e->v_sc = (float*)calloc(kv / 32, sizeof(float));
    }
    e->h = (float*)malloc(B * H * sizeof(float));
    e->hn = (float*)malloc(B * H * sizeof(float));
    e->q = (float*)malloc(B * qd * sizeof(float));
    e->k = (float*)malloc(B * kvd * sizeof(float));
    e->v = (float*)malloc(B * kvd * sizeof(float));
    e->att = (float*)malloc(B * (size_t)(qd > H ? qd : H) * sizeof(float));
    e->gate = (float*)malloc(B * I * sizeof(float));
    e->up = (float*)malloc(B * I * sizeof(float));
    e->ffn = (float*)malloc(B * I * sizeof(float));
    e->pq = (int8_t*)malloc((size_t)mx);
    e->pxs = (float*)malloc((size_t)(mx / 32) * sizeof(float));
    e->pxm = (int32_t*)malloc((size_t)(mx / 32) * sizeof(int32_t));
    e->sc0 = (float*)malloc((size_t)S * sizeof(float));
    e->sc1 = (float*)malloc((size_t)S * sizeof(float));
    return e;
}

ORC_EXPORT void orc_engine_destroy(void* handle) {
    OrcEngine* e = (OrcEngine*)handle;
    if (!e) return;
    free(e->layers); free(e->cos_tab); free(e->sin_tab); free(e->k_cache); free(e->v_cache);
    free(e->k_q8); free(e->v_q8); free(e->k_sc); free(e->v_sc);
    free(e->h); free(e->hn); free(e->q); free(e->k); free(e->v); free(e->att);
    free(e->gate); free(e->up); free(e->ffn); free(e->pq); free(e->pxs); free(e->pxm);
    free(e->sc0); free(e->sc1);
    free(e);
}

ORC_EXPORT void orc_engine_reset_cache(void* handle) {
    OrcEngine* e = (OrcEngine*)handle;
    size_t kv = (size_t)e->cfg.num_layers * (size_t)e->cfg.max_seq_len * (size_t)(e->cfg.num_kv_heads * e->cfg.head_dim);
    memset(e->k_cache, 0, kv * sizeof(float));
    memset(e->v_cache, 0, kv * sizeof(float));
    if (e->k_q8) {
        memset(e->k_q8, 0, kv);
        memset(e->v_q8, 0, kv);
        memset(e->k_sc, 0, kv / 32 * sizeof(float));
        memset(e->v_sc, 0, kv / 32 * sizeof(float));
    }
}

/* Tiles [t0, t1) of weight w on a prepped activation, by the weight's mode (12, 13 or 14; the
 * reference engine's run_weight_tile_range, dpuf_engine.c:1046-1089). */
static void tiles_range(const DpufWeightDesc* w, int32_t t0, int32_t t1, const int8_t* q, const float* xs,
                        const int32_t* xm, float* out) {
    if (w->mode == 13 || w->mode == 14)
        had_tiles(w->mode == 14, w->cols, w->tensor_base, w->tile_offsets, t0, t1, q, xs, xm, out);
    else
        matvec_tiles(w->cols, w->tensor_base, w->tile_offsets, t0, t1, q, xs, xm, out);
}

/* y[M][rows] = W x for each token (prep with this weight's signs, then matvec). */
static void linear(OrcEngine* e, const DpufWeightDesc* w, int32_t M, const float* x, float* y, int32_t t_end) {
    for (int32_t m = 0; m < M; m++) {
        orc_prep_mode12(w->cols, x + (size_t)m * (size_t)w->cols, w->sign_bits, e->pq, e->pxs, e->pxm);
        tiles_range(w, 0, t_end, e->pq, e->pxs, e->pxm, y + (size_t)m * (size_t)w->rows);
    }
}

/* Forward step with the reference semantics (dpuf_engine_forward_batch_ex,
 * dpuf_engine.c:1625-2147) for token inputs.  Environment knobs are read where the reference
 * reads them: DPUF_{PREFILL,GEN}_KEEP_TILES, DPUF_EARLY_TILES, DPUF_EARLY_MARGIN.
 * If zone_out is non-NULL it receives {used, exited, b1 bits, b2 bits} of the zone-A test. */
ORC_EXPORT int32_t orc_engine_forward(void* handle, int32_t M, const int32_t* ids, int32_t pos0,
                                      int32_t only_last, float* logits, int32_t* zone_out) {
    OrcEngine* e = (OrcEngine*)handle;
    if (!e || !ids || (!logits && only_last != 2)) return -1;
    if (M <= 0 || M > ORC_MAX_BATCH) return -2;
    if (pos0 < 0 || pos0 + M > e->cfg.max_seq_len) return -3;
    const DpufModelConfig* c = &e->cfg;
    const int32_t H = c->hidden_size, I = c->intermediate_size, hd = c->head_dim;
    const int32_t nq = c->num_q_heads, nkv = c->num_kv_heads, groups = nq / nkv;
    const int32_t qd = nq * hd, kvd = nkv * hd, half = hd >> 1, S = c->max_seq_len;
    const float eps = c->rms_eps, scale = 1.0f / sqrtf((float)hd);
    if (zone_out) memset(zone_out, 0, 4 * sizeof(int32_t));

    if (e->tok.mode == 13 || e->tok.mode == 14)
        orc_embed_had_asym_f32(e->tok.mode == 14, M, H, ids, e->tok.tensor_base, e->tok.tile_offsets,
                               e->tok.sign_bits, e->h);
    else
        orc_embed_mode12_f32(M, H, ids, e->tok.tensor_base, e->tok.tile_offsets, e->tok.sign_bits, e->h);

    for (int32_t l = 0; l < c->num_layers; l++) {
        const DpufLayerWeights* lw = &e->layers[l];
        for (int32_t m = 0; m < M; m++)
            orc_add_rmsnorm(H, e->h + (size_t)m * H, l > 0 ? e->hn + (size_t)m * H : NULL, lw->attn_norm, eps,
                            e->hn + (size_t)m * H);
        linear(e, &lw->w_q, M, e->hn, e->q, lw->w_q.n_tiles);
        linear(e, &lw->w_k, M, e->hn, e->k, lw->w_k.n_tiles);
        linear(e, &lw->w_v, M, e->hn, e->v, lw->w_v.n_tiles);
        for (int32_t m = 0; m < M; m++) {
            int32_t pos = pos0 + m;
            const float* cs = e->cos_tab + (size_t)pos * half;
            const float* sn = e->sin_tab + (size_t)pos * half;
            for (int32_t kh = 0; kh < nkv; kh++) {
                float* ks = e->k + (size_t)m * kvd + (size_t)kh * hd;
                float* vs = e->v + (size_t)m * kvd + (size_t)kh * hd;
                if (c->has_qk_norm && lw->attn_k_norm) orc_add_rmsnorm(hd, ks, NULL, lw->attn_k_norm, eps, ks);
                rope_apply(hd, ks, cs, sn);
                size_t off = ((size_t)l * nkv + kh) * (size_t)S * hd + (size_t)pos * hd;
                if (e->k_q8) {
                    orc_quantize_q8_blk32(hd, ks, e->k_q8 + off, e->k_sc + off / 32);
                    orc_quantize_q8_blk32(hd, vs, e->v_q8 + off, e->v_sc + off / 32);
                } else {
                    memcpy(e->k_cache + off, ks, (size_t)hd * sizeof(float));
                    memcpy(e->v_cache + off, vs, (size_t)hd * sizeof(float));
                }
            }
            for (int32_t qh = 0; qh < nq; qh++) {
                float* qv = e->q + (size_t)m * qd + (size_t)qh * hd;
                if (c->has_qk_norm && lw->attn_q_norm) orc_add_rmsnorm(hd, qv, NULL, lw->attn_q_norm, eps, qv);
                rope_apply(hd, qv, cs, sn);
            }
        }
        for (int32_t m = 0; m < M; m++) {
            int32_t kv_len = pos0 + m + 1;
            for (int32_t kh = 0; kh < nkv; kh++) {
                const float* kc = e->k_cache + ((size_t)l * nkv + kh) * (size_t)S * hd;
                const float* vc = e->v_cache + ((size_t)l * nkv + kh) * (size_t)S * hd;
                for (int32_t g = 0; g < groups; g += 2) {
                    int32_t qh = kh * groups + g;
                    const float* q0 = e->q + (size_t)m * qd + (size_t)qh * hd;
                    float* a0 = e->att + (size_t)m * qd + (size_t)qh * hd;
                    int pair = (g + 1 < groups);
                    if (e->k_q8) {
                        const size_t ho = ((size_t)l * nkv + kh) * (size_t)S * hd;
                        attn_pair_q8(hd, kv_len, scale, e->k_q8 + ho, e->k_sc + ho / 32, e->v_q8 + ho,
                                     e->v_sc + ho / 32, q0, pair ? q0 + hd : NULL, e->sc0, e->sc1, a0,
                                     pair ? a0 + hd : NULL);
                    } else {
                        attn_pair(hd, kv_len, scale, kc, vc, q0, pair ? q0 + hd : NULL, e->sc0, e->sc1, a0,
                                  pair ? a0 + hd : NULL);
                    }
                }
            }
        }
        linear(e, &lw->w_o, M, e->att, e->hn, lw->w_o.n_tiles);
        for (int32_t m = 0; m < M; m++)
            orc_add_rmsnorm(H, e->h + (size_t)m * H, e->hn + (size_t)m * H, lw->ffn_norm, eps, e->att + (size_t)m * H);
        linear(e, &lw->w_gate, M, e->att, e->gate, lw->w_gate.n_tiles);
        linear(e, &lw->w_up, M, e->att, e->up, lw->w_up.n_tiles);
        {
            int64_t total = (int64_t)M * I;
            int slab_fuse = (M >= 2 && ((M + 5) / 6) >= e->nt);
            for (int64_t idx = 0; idx < total; idx++) {
                /* the slab-fused path splits by whole rows; I % 8 == 0 makes them all vector */
                int vec = slab_fuse ? 1 : orc_swiglu_is_vector(idx, total, e->nt);
                e->ffn[idx] = vec ? swiglu_vec(e->gate[idx], e->up[idx], e->deadzone)
                                  : swiglu_scalar(e->gate[idx], e->up[idx], e->deadzone);
            }
        }
        int32_t down_tiles = lw->w_down.n_tiles;
        const char* kt = getenv(M > 1 ? "DPUF_PREFILL_KEEP_TILES" : "DPUF_GEN_KEEP_TILES");
        if (kt) {
            int32_t v = atoi(kt);
            if (v > 0 && v < down_tiles) down_tiles = v;
        }
        linear(e, &lw->w_down, M, e->ffn, e->hn, down_tiles);
        if (down_tiles < lw->w_down.n_tiles)
            for (int32_t m = 0; m < M; m++)
                for (int32_t r = down_tiles * 16; r < lw->w_down.rows; r++) e->hn[(size_t)m * H + r] = 0.0f;
    }

    if (only_last == 2) return 0;
    int32_t lm_start = only_last ? M - 1 : 0, lm_M = M - lm_start;
    for (int32_t j = 0; j < lm_M; j++) {
        int32_t m = lm_start + j;
        orc_add_rmsnorm(H, e->h + (size_t)m * H, c->num_layers > 0 ? e->hn + (size_t)m * H : NULL, e->out_norm, eps,
                        e->att + (size_t)j * H);
    }
    const DpufWeightDesc* w = &e->lm;
    const char* env_t = getenv("DPUF_EARLY_TILES");
    if (env_t && lm_M == 1 && w->n_tiles > 2048) {
        int32_t za = atoi(env_t);
        if (za < 256) za = 256;
        if (za > w->n_tiles) za = w->n_tiles;
        orc_prep_mode12(w->cols, e->att, w->sign_bits, e->pq, e->pxs, e->pxm);
        tiles_range(w, 0, za, e->pq, e->pxs, e->pxm, logits);
        int32_t n_za = za * 16;
        if (n_za > c->vocab_size) n_za = c->vocab_size;
        float b1 = -1e30f, b2 = -1e30f;
        for (int32_t i = 0; i < n_za; i++) {
            float v = logits[i];
            if (v > b1) { b2 = b1; b1 = v; }
            else if (v > b2) { b2 = v; }
        }
        const char* env_m = getenv("DPUF_EARLY_MARGIN");
        float thr = env_m ? (float)atof(env_m) : 1.25f;
        int exited = (thr > 0.0f && (b1 - b2) >= thr);
        if (zone_out) {
            zone_out[0] = 1;
            zone_out[1] = exited;
            memcpy(&zone_out[2], &b1, 4);
            memcpy(&zone_out[3], &b2, 4);
        }
        if (exited) {
            for (int32_t i = za * 16; i < c->vocab_size; i++) logits[i] = -1e9f;
        } else {
            tiles_range(w, za, w->n_tiles, e->pq, e->pxs, e->pxm, logits);
        }
    } else {
        linear(e, w, lm_M, e->att, logits, w->n_tiles);
    }
    return 0;
}

/* Debug accessors: the last forward's residual stream and KV cache. */
ORC_EXPORT const float* orc_engine_hidden(void* handle) { return ((OrcEngine*)handle)->h; }
ORC_EXPORT const float* orc_engine_k_cache(void* handle) { return ((OrcEngine*)handle)->k_cache; }
ORC_EXPORT const float* orc_engine_v_cache(void* handle) { return ((OrcEngine*)handle)->v_cache; }

/* First index of the maximum, strict '>' (sample_token greedy branch, dpuf-cli.c:1997-2005). */
ORC_EXPORT int32_t orc_argmax(const float* x, int32_t n) {
    int32_t best = 0;
    float bv = x[0];
    for (int32_t i = 1; i < n; i++)
        if (x[i] > bv) { bv = x[i]; best = i; }
    return best;
}

/* ---- host libm expf over a range of inputs (test infrastructure) ----
 * Counts the inputs bits0 .. bits0 + n - 1 (as float bit patterns) where got[i] differs bit
 * for bit from this host's expf; *first (optional) receives the first differing index or -1. */
int64_t orc_expf_mismatch(uint32_t bits0, int64_t n, const float* got, int64_t* first) {
    int64_t bad = 0, lo = -1;
    #pragma omp parallel for reduction(+:bad) schedule(static)
    for (int64_t i = 0; i < n; i++) {
        uint32_t b = bits0 + (uint32_t)i, gb, wb;
        float x, w;
        memcpy(&x, &b, 4);
        w = expf(x);
        memcpy(&wb, &w, 4);
        memcpy(&gb, &got[i], 4);
        if (gb != wb) {
            bad++;
            #pragma omp critical
            { if (lo < 0 || i < lo) lo = i; }
        }
    }
    if (first) *first = lo;
    return bad;
}
