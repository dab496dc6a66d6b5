/*
 * pack_mode12.c - host-side encoder for DPUF mode 12 ("Hadamard-4bit packed") weight blobs,
 * plus a fast seeded N(0, sigma) weight generator used to build random-init models.
 *
 * This is the data format on the input side of the GPU path: it produces the same bytes as
 * the reference packer's `encode_tensor_qr_hadamard4_packed` (dpuf_format.py:1563) so that a
 * model built here can be fed unchanged to both the reference CPU engine and the CUDA engine.
 *
 * Algorithm (dpuf_format.py:1433-1536, `_encode_qr_hadamard4_common` with packed_layout=True):
 *   per row: bf16 -> fp32, multiply by the per-column sign (+-1), orthonormal FWHT over each
 *   64-column chunk (butterfly strides 1,2,...,32, then x0.125), then per 32-column block:
 *     amax   = max |w|
 *     base   = amax / 7.5f + 1e-12f
 *     scale  = the fp16 candidate among fp16(base * {0.78, 0.85, 0.92, 1.00}) with the smallest
 *              float32 squared error sum (strict '<', first candidate wins ties; the sum uses
 *              numpy's 8-accumulator pairwise order, dpuf_format.py:1480-1489)
 *     q      = clip(rint(w / scale), -8, 7), stored as the nibble u = q + 8
 *   tile (16 rows) body: per 8-row group g: fp16 scales [n_blk][8], then the nibbles
 *   [n_blk][chunk c=0..3][row ri=0..7][k=0..3] where byte = u[8c+k] | u[8c+4+k] << 4
 *   (dpuf_format.py:1504-1530); tile = 16-byte header {crc32(body), n_rows, 0, 0, 0} + body,
 *   zero-padded to 64 bytes.
 * Blob (dpuf_format.py:1182-1251): 64-byte finder header "QRDP", tile offsets, ECC offsets,
 *   pad64, sign bits (aux), pad64, tiles, XOR parity of each group of `ecc_group` tiles.
 *
 * All float arithmetic is plain IEEE binary32 with no contraction (build with
 * -ffp-contract=off), matching numpy's float32 element-wise semantics.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DPUF_PACK_EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------- CRC-32 (IEEE 802.3) */
static uint32_t g_crc_tab[256];
static int g_crc_init = 0;

static void crc_init(void) {
    if (g_crc_init) return;
    for (uint32_t i = 0; i < 256; i++) {
        uint32_t c = i;
        for (int k = 0; k < 8; k++) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
        g_crc_tab[i] = c;
    }
    g_crc_init = 1;
}

DPUF_PACK_EXPORT uint32_t dpuf_pack_crc32(const uint8_t* p, uint64_t n) {
    crc_init();
    uint32_t c = 0xFFFFFFFFu;
    for (uint64_t i = 0; i < n; i++) c = g_crc_tab[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

/* ---------------------------------------------------------------- fp16 <-> fp32 */
/* Round-to-nearest-even float32 -> binary16, including subnormals, inf and nan. */
static uint16_t f32_to_f16_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ex = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (ex == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    int32_t e = (int32_t)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

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

DPUF_PACK_EXPORT void dpuf_pack_f32_to_f16(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = f32_to_f16_rne(in[i]);
}

DPUF_PACK_EXPORT void dpuf_pack_f16_to_f32(const uint16_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = f16_to_f32(in[i]);
}

static inline float bf16_to_f32(uint16_t u) {
    uint32_t x = (uint32_t)u << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* Round-to-nearest-even float32 -> bfloat16 (dpuf_format.py:74-79 adds 0x7FFF + lsb). */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    return (uint16_t)((x + (((x >> 16) & 1u) + 0x7FFFu)) >> 16);
}

/* ---------------------------------------------------------------- encoder core */
/* numpy float32 pairwise sum of exactly 32 terms: 8 strided accumulators, then a tree. */
static inline float np_sum32(const float* a) {
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    for (int i = 8; i < 32; i += 8)
        for (int j = 0; j < 8; j++) r[j] = r[j] + a[i + j];
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

static inline float clip_round(float v) {
    float q = rintf(v);
    if (q < -8.0f) q = -8.0f;
    if (q > 7.0f) q = 7.0f;
    return q;
}

/* Encodes one row: rotated fp32 values -> per-block fp16 scale and 32 nibbles (u = q + 8). */
static void encode_row(const uint16_t* w_bf16, int32_t cols, const float* signs,
                       float* rot, uint16_t* sc_out, uint8_t* u4_out) {
    for (int32_t c = 0; c < cols; c++) rot[c] = bf16_to_f32(w_bf16[c]) * signs[c];
    for (int32_t c0 = 0; c0 < cols; c0 += 64) {
        float* y = rot + c0;
        for (int h = 1; h < 64; h <<= 1) {
            for (int g = 0; g < 64; g += 2 * h) {
                for (int i = g; i < g + h; i++) {
                    float a = y[i], b = y[i + h];
                    y[i] = a + b;
                    y[i + h] = a - b;
                }
            }
        }
        for (int i = 0; i < 64; i++) y[i] = y[i] * 0.125f;
    }
    static const float mults[4] = {0.78f, 0.85f, 0.92f, 1.00f};
    const int32_t n_blk = cols >> 5;
    float sq[32];
    for (int32_t b = 0; b < n_blk; b++) {
        const float* wb = rot + (size_t)b * 32u;
        float amax = 0.0f;
        for (int k = 0; k < 32; k++) {
            float a = fabsf(wb[k]);
            if (a > amax) amax = a;
        }
        float base = amax / 7.5f;
        base = base + 1e-12f;
        uint16_t best = f32_to_f16_rne(base);
        float best_err = INFINITY;
        for (int mi = 0; mi < 4; mi++) {
            float prod = base * mults[mi];
            uint16_t cand = f32_to_f16_rne(prod);
            float cf = f16_to_f32(cand);
            float safe = (cf > 0.0f) ? cf : 1.0f;
            for (int k = 0; k < 32; k++) {
                float q = clip_round(wb[k] / safe);
                float qc = q * cf;
                float d = wb[k] - qc;
                sq[k] = d * d;
            }
            float err = np_sum32(sq);
            if (err < best_err) {
                best_err = err;
                best = cand;
            }
        }
        sc_out[b] = best;
        float sf = f16_to_f32(best);
        float safe = (sf > 0.0f) ? sf : 1.0f;
        for (int k = 0; k < 32; k++) {
            float q = clip_round(wb[k] / safe);
            u4_out[(size_t)b * 32u + (size_t)k] = (uint8_t)((int)q + 8);
        }
    }
}

static inline uint64_t pad64(uint64_t n) { return (64u - (n % 64u)) % 64u; }

static uint64_t tile_bytes(int32_t n_r, int32_t cols) {
    uint64_t n_8g = (uint64_t)((n_r + 7) / 8);
    uint64_t raw = 16u + n_8g * (uint64_t)(cols / 32) * 144u;
    return raw + pad64(raw);
}

/* Layout of a packed blob, shared by the size query and the encoder. */
typedef struct {
    int32_t n_tiles, n_ecc;
    uint64_t toff_pos, eoff_pos, aux_off, tiles_base_off, ecc_base_off, total;
} BlobLayout;

static void blob_layout(int32_t rows, int32_t cols, int32_t tile_rows, int32_t ecc_group, BlobLayout* L) {
    L->n_tiles = (rows + tile_rows - 1) / tile_rows;
    L->n_ecc = ecc_group > 0 ? (L->n_tiles + ecc_group - 1) / ecc_group : 0;
    uint64_t tiles_len = 0;
    for (int32_t t = 0; t < L->n_tiles; t++) {
        int32_t n_r = rows - t * tile_rows;
        if (n_r > tile_rows) n_r = tile_rows;
        tiles_len += tile_bytes(n_r, cols);
    }
    uint64_t ecc_len = 0;
    for (int32_t g = 0; g < L->n_ecc; g++) {
        int32_t g0 = g * ecc_group;
        int32_t g1 = g0 + ecc_group < L->n_tiles ? g0 + ecc_group : L->n_tiles;
        uint64_t mx = 0;
        for (int32_t t = g0; t < g1; t++) {
            int32_t n_r = rows - t * tile_rows;
            if (n_r > tile_rows) n_r = tile_rows;
            uint64_t tb = tile_bytes(n_r, cols);
            if (tb > mx) mx = tb;
        }
        ecc_len += (mx / 8u) * 8u;
    }
    L->toff_pos = 64;
    L->eoff_pos = 64 + (uint64_t)(L->n_tiles + 1) * 8u;
    uint64_t after_tables = L->eoff_pos + (uint64_t)(L->n_ecc + 1) * 8u;
    L->aux_off = after_tables + pad64(after_tables);
    uint64_t after_aux = L->aux_off + (uint64_t)(cols / 8);
    L->tiles_base_off = after_aux + pad64(after_aux);
    L->ecc_base_off = L->tiles_base_off + tiles_len;
    L->total = L->ecc_base_off + ecc_len;
}

DPUF_PACK_EXPORT int64_t dpuf_pack_mode12_size(int32_t rows, int32_t cols, int32_t tile_rows, int32_t ecc_group) {
    if (rows <= 0 || cols <= 0 || (cols % 64) != 0 || tile_rows != 16) return -1;
    BlobLayout L;
    blob_layout(rows, cols, tile_rows, ecc_group, &L);
    return (int64_t)L.total;
}

/*
 * Encodes a [rows][cols] bf16 matrix into a mode-12 blob.  `sign_bits` holds cols/8 bytes,
 * bit k of byte j set meaning column 8j+k is negated (numpy packbits, little bit order).
 * `out` must hold dpuf_pack_mode12_size() bytes.  Returns 0 on success, <0 on bad arguments.
 */
DPUF_PACK_EXPORT int32_t dpuf_pack_mode12(const uint16_t* w_bf16, int32_t rows, int32_t cols,
                                          const uint8_t* sign_bits, int32_t tile_rows,
                                          int32_t ecc_group, uint8_t* out, int32_t n_threads) {
    if (!w_bf16 || !sign_bits || !out) return -1;
    if (rows <= 0 || cols < 64 || (cols % 64) != 0 || tile_rows != 16 || ecc_group < 0) return -2;
    crc_init();
    BlobLayout L;
    blob_layout(rows, cols, tile_rows, ecc_group, &L);
    memset(out, 0, (size_t)L.total);
    const int32_t n_blk = cols / 32;

    float* signs = (float*)malloc((size_t)cols * sizeof(float));
    uint64_t* toffs = (uint64_t*)malloc((size_t)(L.n_tiles + 1) * sizeof(uint64_t));
    if (!signs || !toffs) { free(signs); free(toffs); return -3; }
    for (int32_t c = 0; c < cols; c++) signs[c] = ((sign_bits[c >> 3] >> (c & 7)) & 1u) ? -1.0f : 1.0f;
    uint64_t cur = 0;
    for (int32_t t = 0; t < L.n_tiles; t++) {
        int32_t n_r = rows - t * tile_rows;
        if (n_r > tile_rows) n_r = tile_rows;
        toffs[t] = cur;
        cur += tile_bytes(n_r, cols);
    }
    toffs[L.n_tiles] = cur;
    uint8_t* tiles = out + L.tiles_base_off;
    int failed = 0;

    if (n_threads <= 0) n_threads = 1;
    #pragma omp parallel num_threads(n_threads)
    {
        float* rot = (float*)malloc((size_t)cols * sizeof(float));
        uint16_t* sc = (uint16_t*)malloc((size_t)16 * (size_t)n_blk * sizeof(uint16_t));
        uint8_t* u4 = (uint8_t*)malloc((size_t)16 * (size_t)cols);
        if (!rot || !sc || !u4) {
            #pragma omp atomic write
            failed = 1;
        } else {
            #pragma omp for schedule(dynamic, 4)
            for (int32_t t = 0; t < L.n_tiles; t++) {
                int32_t r0 = t * tile_rows;
                int32_t n_r = rows - r0;
                if (n_r > tile_rows) n_r = tile_rows;
                int32_t n_8g = (n_r + 7) / 8;
                /* padded rows: scale 0, nibble 8 (dpuf_format.py:1510-1514) */
                for (int32_t i = 0; i < n_8g * 8; i++) {
                    if (i < n_r) {
                        encode_row(w_bf16 + (size_t)(r0 + i) * (size_t)cols, cols, signs, rot,
                                   sc + (size_t)i * (size_t)n_blk, u4 + (size_t)i * (size_t)cols);
                    } else {
                        memset(sc + (size_t)i * (size_t)n_blk, 0, (size_t)n_blk * 2u);
                        memset(u4 + (size_t)i * (size_t)cols, 8, (size_t)cols);
                    }
                }
                uint8_t* tp = tiles + toffs[t];
                uint8_t* body = tp + 16;
                uint8_t* bp = body;
                for (int32_t g = 0; g < n_8g; g++) {
                    for (int32_t b = 0; b < n_blk; b++)
                        for (int32_t ri = 0; ri < 8; ri++) {
                            uint16_t s = sc[(size_t)(g * 8 + ri) * (size_t)n_blk + (size_t)b];
                            bp[0] = (uint8_t)(s & 0xFFu);
                            bp[1] = (uint8_t)(s >> 8);
                            bp += 2;
                        }
                    for (int32_t b = 0; b < n_blk; b++)
                        for (int32_t c = 0; c < 4; c++)
                            for (int32_t ri = 0; ri < 8; ri++)
                                for (int32_t k = 0; k < 4; k++) {
                                    const uint8_t* ur = u4 + (size_t)(g * 8 + ri) * (size_t)cols + (size_t)b * 32u;
                                    *bp++ = (uint8_t)(ur[c * 8 + k] | (ur[c * 8 + 4 + k] << 4));
                                }
                }
                uint64_t body_len = (uint64_t)(bp - body);
                uint32_t crc = dpuf_pack_crc32(body, body_len);
                tp[0] = (uint8_t)crc; tp[1] = (uint8_t)(crc >> 8); tp[2] = (uint8_t)(crc >> 16); tp[3] = (uint8_t)(crc >> 24);
                tp[4] = (uint8_t)n_r; tp[5] = (uint8_t)(n_r >> 8);
            }
        }
        free(rot); free(sc); free(u4);
    }
    if (failed) { free(signs); free(toffs); return -3; }

    /* ECC: XOR of the (padded) tiles of each group, over whole uint64 words */
    uint8_t* ecc = out + L.ecc_base_off;
    uint64_t* eoffs = (uint64_t*)malloc((size_t)(L.n_ecc + 1) * sizeof(uint64_t));
    if (!eoffs) { free(signs); free(toffs); return -3; }
    uint64_t ecur = 0;
    for (int32_t g = 0; g < L.n_ecc; g++) {
        int32_t g0 = g * ecc_group;
        int32_t g1 = g0 + ecc_group < L.n_tiles ? g0 + ecc_group : L.n_tiles;
        uint64_t mx = 0;
        for (int32_t t = g0; t < g1; t++) {
            uint64_t tl = toffs[t + 1] - toffs[t];
            if (tl > mx) mx = tl;
        }
        uint64_t n_u64 = mx / 8u;
        eoffs[g] = ecur;
        uint8_t* dst = ecc + ecur;
        for (int32_t t = g0; t < g1; t++) {
            uint64_t tl = (toffs[t + 1] - toffs[t]) / 8u;
            const uint8_t* src = tiles + toffs[t];
            for (uint64_t w = 0; w < tl; w++) {
                uint64_t a, v;
                memcpy(&a, dst + w * 8u, 8);
                memcpy(&v, src + w * 8u, 8);
                a ^= v;
                memcpy(dst + w * 8u, &a, 8);
            }
        }
        ecur += n_u64 * 8u;
    }
    eoffs[L.n_ecc] = ecur;

    /* finder header "<B4sBHIIIIQQQ16x" (dpuf_format.py:936, dpuf-cli.c:75-88) */
    uint8_t* h = out;
    h[0] = 12;
    memcpy(h + 1, "QRDP", 4);
    h[5] = (uint8_t)tile_rows;
    uint16_t eg = (uint16_t)ecc_group;
    memcpy(h + 6, &eg, 2);
    uint32_t u32v;
    u32v = (uint32_t)rows; memcpy(h + 8, &u32v, 4);
    u32v = (uint32_t)cols; memcpy(h + 12, &u32v, 4);
    u32v = (uint32_t)L.n_tiles; memcpy(h + 16, &u32v, 4);
    u32v = (uint32_t)L.n_ecc; memcpy(h + 20, &u32v, 4);
    memcpy(h + 24, &L.aux_off, 8);
    memcpy(h + 32, &L.tiles_base_off, 8);
    memcpy(h + 40, &L.ecc_base_off, 8);
    memcpy(out + L.toff_pos, toffs, (size_t)(L.n_tiles + 1) * 8u);
    memcpy(out + L.eoff_pos, eoffs, (size_t)(L.n_ecc + 1) * 8u);
    memcpy(out + L.aux_off, sign_bits, (size_t)(cols / 8));
    free(signs); free(toffs); free(eoffs);
    return 0;
}

/* ---------------------------------------------------------------- seeded weight generator */
/*
 * Random-init weights for synthetic models: w = sigma * N(0,1), rounded to bf16 (RNE).
 * N(0,1) comes from a counter-based generator so the result is independent of the thread
 * count: element i of stream `stream` draws two uniforms from splitmix64(seed, stream, i)
 * and applies the Box-Muller transform in double precision, keeping the cosine branch.
 */
static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

DPUF_PACK_EXPORT void dpuf_gen_normal_bf16(uint64_t seed, uint64_t stream, int64_t n, float sigma,
                                           uint16_t* out, int32_t n_threads) {
    if (n_threads <= 0) n_threads = 1;
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
    #pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t i = 0; i < n; i++) {
        uint64_t a = splitmix64(key + 2u * (uint64_t)i);
        uint64_t b = splitmix64(key + 2u * (uint64_t)i + 1u);
        double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0, 1] */
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);         /* [0, 1) */
        double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        out[i] = f32_to_bf16((float)(z * (double)sigma));
    }
}
