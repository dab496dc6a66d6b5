/*
 * dpuf_cuda.h - entry points of libdpuf_cuda.so beyond the reference's C ABI.
 *
 * These have no counterpart in the reference (which is CPU-only); they expose what a GPU
 * host needs on top of dpuf_kernels.h: greedy decoding without shipping logits to the host,
 * device-resident weights for the standalone op, per-engine options and error text.
 */
#ifndef DPUF_CUDA_H
#define DPUF_CUDA_H

#include "dpuf_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Text of the last error seen by this thread's most recent failing call ("" if none). */
DPUF_EXPORT const char* dpuf_cuda_last_error(void);

/* Same step as dpuf_engine_forward_batch(..., only_last_logits = 1, ...) but the logits stay
 * on the device; *next_id receives the greedy token (first index of the maximum, as the
 * reference CLI's sample_token at temperature 0, dpuf-cli.c:1997-2005).  Returns the
 * forward_batch codes. */
DPUF_EXPORT int32_t dpuf_cuda_forward_greedy(void* handle, int32_t n_tokens, const int32_t* token_ids,
                                             int32_t pos0, int32_t* next_id);

/* n_steps greedy decode steps at batch 1 starting from token first_id at position pos0, with
 * each step's token chosen and fed back on the device (same kernels as forward_token; the
 * logits never leave the device).  ids_out[n_steps] receives the generated ids; *device_ms
 * (optional) the CUDA-event time of the steps on the engine's stream. */
DPUF_EXPORT int32_t dpuf_cuda_decode_greedy(void* handle, int32_t first_id, int32_t pos0, int32_t n_steps,
                                            int32_t* ids_out, float* device_ms);

/* One greedy decode step of n independent sequences (batched serving; the reference runs them
 * one after another): row i continues the sequence in slot slots[i] (distinct, allocated on
 * first use) at position pos[i] with input token ids[i].  Every row is computed as that
 * sequence's own batch-1 step (the M-row kernels, with the reference's one-row SwiGLU
 * vector/scalar split), so its logits and id equal dpuf_engine_forward_token's on that slot
 * (DPUF_GEN_KEEP_TILES applies; Zone A does not).  next_ids[n] (host) receive the greedy ids,
 * logits_out (optional, host) [n][vocab].  Env DPUF_CUDA_SLOTS (default 8, the reference's
 * count; at most 256) sets the number of slots at create.  Env DPUF_CUDA_KV_F16=1 at create
 * stores every slot's (and prefix's) K and V in fp16, halving the cache and its reads (the
 * reference's cache is fp32: results then agree within tolerance, not bit for bit; batch-1
 * steps use the per-step kernels).  Returns the forward codes. */
DPUF_EXPORT int32_t dpuf_cuda_decode_batch(void* handle, int32_t n, const int32_t* slots, const int32_t* ids,
                                           const int32_t* pos, int32_t* next_ids, float* logits_out);

/* Copies the last forward's logits row `row` (0-based among the rows produced) to host. */
DPUF_EXPORT int32_t dpuf_cuda_read_logits(void* handle, int32_t row, float* out);

/* Engine options (call before the first forward):
 *   "pdl" (0/1)        programmatic dependent launch between kernels (default 1)
 *   "graphs" (0/1)     capture each step shape in a CUDA graph (default 1)
 *   "persistent" (0/1) run batch-1 steps (forward_token, forward_batch with one token,
 *                      decode_greedy) as one persistent cooperative kernel when the engine
 *                      supports it (default 1; env DPUF_CUDA_PERSISTENT=0 turns it off)
 *   "wait_ms" (> 0)    how long any wait inside the persistent kernel may last before the call
 *                      gives up with -6 (default: env DPUF_CUDA_WAIT_MS at create, else 2000)
 *   "test_stall_unit"  failure-detection test hook: in the next persistent launch only, the CTA
 *                      computing q/k/v unit `value` (8 rows of layer 0, q rows first) withholds
 *                      its outputs of the first step, so the waits on them run out and the call
 *                      returns -6; the next call on the same engine starts from a reset
 *                      exchange area (one GPU) and is exact again */
DPUF_EXPORT int32_t dpuf_cuda_set_option(void* handle, const char* name, int64_t value);

/* 1 if batch-1 steps run as the persistent kernel, 0 if they run as per-step kernels, -1 for a
 * null handle.  *why (optional) receives the reason the persistent kernel cannot be used ("" if
 * it can; Zone-A steps always use the per-step kernels).  A persistent step that hits a device
 * wait limit returns -6 with the reason in dpuf_cuda_last_error(). */
DPUF_EXPORT int32_t dpuf_cuda_persistent_decode(void* handle, const char** why);

/* Phase trace of the persistent kernel's last step, recorded when the engine was created with
 * env DPUF_CUDA_TRACE_DECODE=1 (otherwise returns -1).  Per CTA, per_cta globaltimer stamps
 * (ns), as recorded by the CTA's thread 0: for each layer (20) the end of the norm1 residual,
 * sum of squares and prep; q/k/v; the attention steps (q/k/v words in, inputs ready, QK-norm
 * and RoPE, scores, softmax, PV, output prep; CTAs hosting no head stamp them all at once);
 * the o input's load; o; the norm2 residual, sum of squares and prep; the end of warp 0's
 * gate/up stages; gate/up; the down input's load; down.  Then per step (5): start, embedding,
 * final norm, LM head, argmax.  *n_ctas and *per_cta receive the shape; out (optional) receives
 * n_ctas * per_cta values when max_values is large enough (else -2). */
DPUF_EXPORT int32_t dpuf_cuda_decode_trace(void* handle, int32_t* n_ctas, int32_t* per_cta, uint64_t* out,
                                           int64_t max_values);

/* ---- tensor parallelism of batch-1 decode over processes, one GPU each ----
 * The reference has no multi-GPU mode.  Every rank creates an engine for the same model on its
 * own GPU (weights are replicated), then:
 *   1. dpuf_cuda_tp_handle(h, rank, world, blob) allocates this rank's exchange buffer and
 *      writes DPUF_CUDA_TP_BLOB_BYTES bytes describing it (its IPC handle and the model shape);
 *   2. the caller all-gathers the blobs in rank order (any host transport: the caller's
 *      process group, a file, a socket) - this also ensures every buffer exists before use;
 *   3. dpuf_cuda_tp_attach(h, blobs[world * DPUF_CUDA_TP_BLOB_BYTES]) maps the other ranks'
 *      buffers (NVLink peer access).  Every rank must be on a GPU of its own (checked by PCI bus
 *      id): the ranks' kernels wait on each other.
 * From then on each batch-1 step that runs as the persistent kernel splits every projection
 * and the LM head over all ranks' CTAs; each rank stores its outputs, tagged with the phase
 * that produced them, to every rank's buffer, and readers wait on those tags (no cross-GPU
 * barrier).
 * Attention, norms and everything else run in full on every rank, so every rank returns the
 * same ids and logits, bit-identical to one GPU.  All ranks must make the same calls with the
 * same arguments in the same order (steps with M > 1, or with Zone A, simply run in full on
 * every rank).  A rank whose wait times out sets every rank's error word; the group then
 * returns -6 for every persistent step until the engines are re-created.
 * Returns 0; -1 bad arguments or order, or mismatching blobs; -4 CUDA error; -5 the engine
 * cannot run the persistent kernel (dpuf_cuda_persistent_decode gives the reason). */
#define DPUF_CUDA_TP_BLOB_BYTES 256
DPUF_EXPORT int32_t dpuf_cuda_tp_handle(void* handle, int32_t rank, int32_t world, uint8_t* blob_out);
DPUF_EXPORT int32_t dpuf_cuda_tp_attach(void* handle, const uint8_t* blobs);

/* Zone-A decision of the last forward: {used, exited} and the top-2 values. */
DPUF_EXPORT int32_t dpuf_cuda_zone_info(void* handle, int32_t* used, int32_t* exited, float* b1, float* b2);

/* ---- device-resident standalone op (for measuring the kernel with weights in HBM) ---- */
/* Uploads one mode-12 matrix; returns an opaque handle or NULL. */
DPUF_EXPORT void* dpuf_cuda_w12_upload(const DpufWeightDesc* w);
DPUF_EXPORT void dpuf_cuda_w12_free(void* wh);
/* y[M][rows] = W x[M][cols]; x and y are DEVICE pointers; runs on `stream` (cudaStream_t,
 * NULL = default stream) without synchronising.  Scratch for the quantised activation is
 * owned by the weight handle.  Returns 0 or a negative error. */
DPUF_EXPORT int32_t dpuf_cuda_matmul_dev(void* wh, int32_t M, const float* x_dev, float* y_dev, void* stream);

/* LM head with the Zone-A early exit (the engine's step, dpuf_engine.c:2091-2139) on n_vec
 * hidden vectors x_dev[n_vec][cols] (DEVICE, already RMS-normalised), each as one batch-1
 * step: rows of tiles [0, Z) (Z = zone_tiles clamped to [256, n_tiles]), exit when margin > 0
 * and the top two logits of [0, min(16Z, V)) differ by >= margin, else the remaining tiles;
 * on exit logits [16Z, V) = -1e9.  ids_out[n_vec] (host) = first-index argmax,
 * exits_out[n_vec] (host) = 1 where the step exited; *ms_out (optional) = device time of all
 * steps.  Returns 0 or a negative error. */
DPUF_EXPORT int32_t dpuf_cuda_zone_head(void* wh, int32_t n_vec, const float* x_dev, int32_t zone_tiles,
                                        float margin, int32_t* ids_out, int32_t* exits_out, float* ms_out);

/* Kernel-only timing of the matmul (activation prep excluded): `iters` launches rotating over
 * n_handles uploaded weights, CUDA events on `stream`; *ms_out = mean ms per launch. */
DPUF_EXPORT int32_t dpuf_cuda_matmul_dev_timed(void** whs, int32_t n_handles, int32_t M, const float* x_dev,
                                               float* y_dev, int32_t iters, void* stream, float* ms_out);

/* The standalone matmul for callers that cannot allocate device memory: hosts that reserve
 * the GPU's memory for their own pool at start-up (a further cudaMalloc fails or escapes their
 * accounting) and latency-critical loops that cannot afford cudaMalloc/cudaFree's implicit
 * device synchronisation.  No counterpart in the reference (its matmul is CPU-only).
 * Everything is a DEVICE pointer the caller owns: x[M][cols] in, y[M][rows] out, the weight as
 * its container tiles, tile offsets relative to tiles_dev (the reference's tile_offsets) and
 * sign bits (tiles_dev 16-byte aligned, tile offsets multiples of 16 as every packed container
 * has them).  Allocates nothing: the quantised activation lives in a fixed device array of
 * 2^20 values (1.25 MiB, held by every GPU that loads the library until exit).
 * Returns 0; -1 bad arguments (also a shape the matmul kernels do not take); -2 M * cols > 2^20
 * (rejected, see dpuf_cuda_last_error); -4 CUDA error.  A tile offset that is not a multiple of
 * 16 is not detected (the offsets stay on the device) and gives undefined results.  Enqueues on
 * `stream` without synchronising.  Every call looks the array's address up on the current
 * device (no allocation); the first call on a device also sets the kernels up - make it before
 * any stream capture.  All calls share the array: calls that overlap on the GPU race and must be
 * serialised. */
DPUF_EXPORT int32_t dpuf_cuda_matmul_noalloc(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                             const float* x_dev, const uint8_t* tiles_dev,
                                             const uint64_t* tile_offsets_dev, const uint8_t* sign_bits_dev,
                                             float* y_dev, void* stream);

/* Measurement of the mode-13/14 matmul kernel (no reference counterpart): uploads n_copies
 * copies of the matrix (so that a rotation over them exceeds the L2 cache), preps the M <= 256
 * tokens of x_in once, then times `reps` launches of the matmul kernel over the copies in
 * turn; *ms_per_matmul receives the mean device time of one launch.  mode is 13 or 14.
 * Returns 0, -1 for bad arguments, -4 for a CUDA error. */
DPUF_EXPORT int32_t dpuf_cuda_had_asym_timed(int32_t mode, int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                             const float* x_in, const uint8_t* tensor_base,
                                             const uint64_t* tile_offsets, const uint8_t* sign_bits,
                                             int32_t n_copies, int32_t reps, float* ms_per_matmul);

/* Builds or loads the glibc expf exception table; returns its entry count (host only). */
DPUF_EXPORT int64_t dpuf_cuda_prepare_expf_table(void);

/* ---- token sampling of the engine's callers (host code) ---- */
/* Replaces the reference CLI's sample_token (dpuf-cli.c:1997-2027) with its generator
 * rand_f32 (dpuf-cli.c:1987-1995), whose state is a process global there and the caller's
 * `*rng` here (start it at dpuf_cuda_sample_seed(), the reference's initial state).
 * temp <= 0: first index of the maximum (rng untouched); temp > 0: fp32 glibc expf
 * probabilities of (l - max) * (1 / temp), one generator step, sequential double CDF.  Returns the
 * id, or -1 for NULL logits, V <= 0, or NULL rng with temp > 0. */
DPUF_EXPORT uint64_t dpuf_cuda_sample_seed(void);
DPUF_EXPORT int32_t dpuf_cuda_sample_token(const float* logits, int32_t V, float temp, uint64_t* rng);

#ifdef __cplusplus
}
#endif

#endif /* DPUF_CUDA_H */
