/*
 * dpuf_kernels.h - drop-in C ABI of the DPUF B200 engine (libdpuf_cuda.so).
 *
 * The structs and entry points below keep the exact layout, names, argument meaning and
 * return codes of the reference header (dpuf_kernels.h in dulePan/dpuf) so that an existing
 * C host (the reference's dpuf-cli.c) or ctypes driver (dpuf_format.DPUFCTransformerEngine)
 * links against this library unchanged.  Each declaration cites the reference line it
 * replaces.  Only mode 12 (DPUF_MODE_QR_HAD4_PACKED) weights are accepted by this engine;
 * other modes make dpuf_engine_create return NULL.
 */
#ifndef DPUF_KERNELS_H
#define DPUF_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#if defined(_MSC_VER)
#define DPUF_EXPORT __declspec(dllexport)
#else
#define DPUF_EXPORT __attribute__((visibility("default")))
#endif

/* Weight codec ids (reference dpuf_kernels.h:29-37). */
enum {
    DPUF_MODE_QR_ZD4 = 8,
    DPUF_MODE_QR_SPLIT4 = 9,
    DPUF_MODE_QR_HAD4 = 10,
    DPUF_MODE_QR_Q8 = 11,
    DPUF_MODE_QR_HAD4_PACKED = 12,
    DPUF_MODE_QR_HAD4_ASYM = 13,
    DPUF_MODE_QR_HAD6 = 14
};

/* KV cache element types (reference dpuf_kernels.h:39-42). */
enum { DPUF_KV_F32 = 0, DPUF_KV_Q8 = 1 };

/* 16-byte header in front of every 16-row weight tile (reference dpuf_kernels.h:44-52). */
#pragma pack(push, 1)
typedef struct {
    uint32_t tile_crc32; /* CRC-32 of the tile body */
    uint16_t n_rows;     /* rows in this tile (16, fewer in the last tile) */
    uint16_t flags;
    uint32_t n_over8;
    uint32_t n_super16;
} DpufQrTileHdr;
#pragma pack(pop)

/* One quantised weight matrix, borrowed from the container (reference dpuf_kernels.h:54-63).
 * tensor_base + tile_offsets[t] is tile t; sign_bits holds cols/8 bytes of column signs. */
typedef struct {
    int32_t mode;
    int32_t rows;
    int32_t cols;
    int32_t n_tiles;
    const uint8_t* tensor_base;
    const uint64_t* tile_offsets;
    const float* col_scale;
    const uint8_t* sign_bits;
} DpufWeightDesc; /* 48 bytes */

/* Model hyper-parameters (reference dpuf_kernels.h:65-87).  n_threads selects the
 * reference thread count whose arithmetic is reproduced (it only decides where the
 * reference's SwiGLU switches to its scalar tail); default 8. */
typedef struct {
    int32_t hidden_size;
    int32_t intermediate_size;
    int32_t num_layers;
    int32_t num_q_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t vocab_size;
    int32_t max_seq_len;
    int32_t has_qk_norm;
    float rms_eps;
    float rope_theta;
    int32_t n_threads;
    int32_t use_llama3_rope;
    float rope_factor;
    float rope_low_freq;
    float rope_high_freq;
    int32_t rope_orig_max_pos;
    int32_t kv_type;            /* DPUF_KV_F32, or DPUF_KV_Q8: int8 rows with per-32 fp32 scales */
    int32_t has_mrope;
    int32_t mrope_section[3];
    int32_t mrope_interleaved;
} DpufModelConfig; /* 92 bytes */

/* Per-layer weights (reference dpuf_kernels.h:89-101). */
typedef struct {
    const float* attn_norm;
    const float* attn_q_norm;
    const float* attn_k_norm;
    const float* ffn_norm;
    DpufWeightDesc w_q;
    DpufWeightDesc w_k;
    DpufWeightDesc w_v;
    DpufWeightDesc w_o;
    DpufWeightDesc w_gate;
    DpufWeightDesc w_up;
    DpufWeightDesc w_down;
} DpufLayerWeights; /* 368 bytes */

#ifdef __cplusplus
extern "C" {
#endif

/* ---- standalone mode-12 ops (reference dpuf_kernels.h:267-277) ------------------------
 * Host pointers in, host pointers out; the call uploads, runs on the current CUDA device
 * and synchronises.  out is [M][rows] (matmul) or [n_tokens][cols] (embed). */
DPUF_EXPORT void dpuf_matmul_qr_hadamard4_packed_f32(
    int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
    const float* x_in, const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

DPUF_EXPORT void dpuf_embed_qr_hadamard4_packed_f32(
    int32_t n_tokens, int32_t cols, const int32_t* token_ids,
    const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

/* ---- standalone mode-13 / mode-14 ops (reference dpuf_kernels.h:279-314) -----------------
 * QR_HAD4_ASYM (4-bit) and QR_HAD6 (6-bit): asymmetric blk64 tiles (8 fp16 d, 8 fp16 m per
 * 64-block and 8-row group) over the same FWHT-64 activation prep; same calling convention as
 * the mode-12 matmul.  A bad descriptor (cols % 64, a tile whose rows fall outside [0, rows))
 * leaves out untouched and is reported by dpuf_cuda_last_error(). */
DPUF_EXPORT void dpuf_matmul_qr_had4_asym_f32(
    int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
    const float* x_in, const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

DPUF_EXPORT void dpuf_matmul_qr_had6_f32(
    int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
    const float* x_in, const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

/* Row lookup of modes 13 / 14 (reference dpuf_kernels.h:293-297 and 310-314): out is
 * [n_tokens][cols]; an id whose row is not in its tile is rejected (dpuf_cuda_last_error). */
DPUF_EXPORT void dpuf_embed_qr_had4_asym_f32(
    int32_t n_tokens, int32_t cols, const int32_t* token_ids,
    const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

DPUF_EXPORT void dpuf_embed_qr_had6_f32(
    int32_t n_tokens, int32_t cols, const int32_t* token_ids,
    const uint8_t* tensor_base, const uint64_t* tile_offsets,
    const uint8_t* sign_bits, float* out);

/* ---- persistent engine (reference dpuf_kernels.h:316-360) -------------------------------
 * create: copies every weight, norm and sign table to device memory (the caller's buffers
 *         need not outlive the call); returns NULL on bad arguments, unsupported weight
 *         modes, or device errors (reference dpuf_engine.c:1208-1354).
 * forward_*: 0 on success; -1 null argument, -2 n_tokens outside [1, 256], -3 position
 *         outside [0, max_seq_len) (reference dpuf_engine.c:1639-1641); this engine adds
 *         -4 for a CUDA error and -5 for an argument it does not support (embeds_in,
 *         deepstack_in, pos_t/h/w and M-RoPE are all supported); -3 also for a rotary
 *         position outside the RoPE table.  logits_out is host memory: [vocab] floats when
 *         only_last_logits == 1, [n_tokens][vocab] when 0, unused when 2. */
DPUF_EXPORT void* dpuf_engine_create(
    const DpufModelConfig* cfg,
    const DpufLayerWeights* layers,
    const DpufWeightDesc* w_tok_embd,
    const DpufWeightDesc* w_lm_head,
    const float* output_norm);
DPUF_EXPORT void dpuf_engine_destroy(void* handle);
DPUF_EXPORT void dpuf_engine_reset_cache(void* handle);
DPUF_EXPORT int32_t dpuf_engine_set_slot(void* handle, int32_t slot_id);
DPUF_EXPORT int32_t dpuf_engine_get_slot(void* handle);
DPUF_EXPORT void dpuf_engine_reset_slot(void* handle, int32_t slot_id);
DPUF_EXPORT size_t dpuf_engine_slot_memory(void* handle);
DPUF_EXPORT int32_t dpuf_engine_num_slots(void* handle);
DPUF_EXPORT int32_t dpuf_engine_freeze_prefix(void* handle, int32_t prefix_id, int32_t prefix_len);
DPUF_EXPORT int32_t dpuf_engine_apply_prefix(void* handle, int32_t slot_id, int32_t prefix_id);
DPUF_EXPORT int32_t dpuf_engine_get_prefix_len(void* handle, int32_t prefix_id);
DPUF_EXPORT int32_t dpuf_engine_forward_batch(
    void* handle, int32_t n_tokens, const int32_t* token_ids, int32_t pos0,
    int32_t only_last_logits, float* logits_out);
DPUF_EXPORT int32_t dpuf_engine_forward_batch_ex(
    void* handle, int32_t n_tokens, const int32_t* token_ids, int32_t pos0,
    const float* embeds_in, const int32_t* pos_t, const int32_t* pos_h, const int32_t* pos_w,
    const float* const* deepstack_in, int32_t only_last_logits, float* logits_out);
DPUF_EXPORT int32_t dpuf_engine_forward_token(
    void* handle, int32_t token_id, int32_t pos, float* logits_out);

#ifdef __cplusplus
}
#endif

#endif /* DPUF_KERNELS_H */
