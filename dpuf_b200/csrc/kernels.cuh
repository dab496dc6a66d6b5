// kernels.cuh - launch interface of the engine's CUDA kernels (host side).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace dpuf {

// A GEMV/GEMM job: rows [16*t_begin, 16*t_end) of weight w applied to activation `act`.
struct LinJob {
  W12 w;
  Act act;
  float* out;      // [M][ldo]
  int ldo;
  int t_begin, t_end;
};
constexpr int kMaxJobs = 3;
struct LinJobs {
  LinJob j[kMaxJobs];
  int n;
  int tile_prefix[kMaxJobs + 1];  // cumulative tile counts (t_end - t_begin)
};

// Launch configuration shared by all engine launches: stream and whether to attach the
// programmatic-dependent-launch attribute (kernels then overlap their weight prefetch with
// the previous kernel's tail and wait for it before touching activations).
struct Launch {
  cudaStream_t stream;
  bool pdl;
};

// Raises the dynamic shared-memory limit of the kernels that may need more than 48 KB.  Called
// once per device before any launch (never inside stream capture).
cudaError_t configure_kernels();

// ---- kernels_mode12.cu
cudaError_t launch_prep(const Launch& L, const float* x, int ldx, int M, int cols, const uint8_t* signs, Act out);
cudaError_t launch_embed(const Launch& L, const W12& w, const int32_t* ids, int M, float* out);
// Modes 13 / 14 (ops_had_asym.cu): y[m * ldo + r] for the rows of tiles [t_begin, t_end) of w
// on a prepped activation (nothing when *skip is set at launch time; *err set when a bounded
// wait of the one-token kernel gives up); the row lookup of a mode-13/14 embedding.  Kernels
// configured at engine create (configure_had_engine_kernels).
cudaError_t configure_had_engine_kernels();
cudaError_t launch_had_w(cudaStream_t s, const W12& w, const Act& a, int M, float* y, int ldo, int t_begin,
                         int t_end, const int* skip, int* err);
cudaError_t launch_had_embed_w(cudaStream_t s, const W12& w, const int32_t* ids, int M, float* out);
// M == 1: HBM-streaming GEMV over a persistent grid (kernels_gemv.cu).  All jobs of one launch
// share K.  skip_flag: when non-null and nonzero at run time, CTAs exit.  split: scratch that
// lets a 16-row unit be shared by two or more CTAs (pairs: gemv_split_pairs_bytes(cols) bytes,
// acc: kGemvMaxCtas*16 floats, count: kGemvMaxCtas zero-initialised words, left at zero); with
// split == nullptr every CTA takes whole units.  One launch at a time may use a scratch.
struct GemvSplit {
  float2* pairs;
  float* acc;
  unsigned* count;
};
constexpr int kGemvMaxCtas = 600;
constexpr int kMaxTp = 8;  // tensor-parallel ranks of the persistent decode kernel
size_t gemv_split_pairs_bytes(int max_cols);
cudaError_t launch_gemv(const Launch& L, const LinJobs& jobs, const int* skip_flag, const GemvSplit* split);
// M == 1 with every consumer warp owning whole 8-row groups (kernels_gemv_wg.cu): one CTA per SM,
// per-warp cp.async.bulk rings.  launch_gemv uses it unless env DPUF_CUDA_GEMV=mma.  *err
// (optional, device) becomes 1 if a wait gives up.
cudaError_t configure_gemv_wg_kernel();
size_t gemv_wg_smem_bytes(int cols, int n_x);
cudaError_t launch_gemv_wg(const Launch& L, const LinJobs& jobs, const int* skip_flag, int* err);
// M > 1: exact integer-dot GEMM on CUDA cores (reference order per (token,row)).
cudaError_t launch_gemm_exact(const Launch& L, const LinJobs& jobs, int M);
// M > 1 on the tensor cores (kernels_gemm_tc.cu): per-block int8 MMA into TMEM, then the same
// fp32 chain; *err (device) becomes nonzero if an MMA wait gives up.
cudaError_t configure_gemm_tc_kernels();
cudaError_t launch_gemm_tc(const Launch& L, const LinJobs& jobs, int M, int* err);
// The expanded copy of a mode-12 matrix that lets launch_gemm_tc skip the in-kernel unpack:
// x8_bytes(w) device bytes, filled by launch_x8_expand (*bad set when a stored scale is not finite,
// in which case the copy must not be used).
size_t x8_bytes(const W12& w);
cudaError_t launch_x8_expand(cudaStream_t s, const W12& w, uint8_t* x8, int* bad);

// ---- kernels_layer.cu
struct PrepTarget {
  const uint8_t* signs;
  Act act;
};
// h[m] += res[m] (if res), out = rmsnorm(h[m]) * w, then prep of `out` for up to 3 sign sets.
// norm_out (optional) receives the normalised fp32 vector.
cudaError_t launch_norm_prep(const Launch& L, float* h, const float* res, const float* w, float eps, int M, int H,
                             const PrepTarget* targets, int n_targets, float* norm_out);
// Per (token, head): QK RMSNorm + NeoX RoPE; K/V of the new tokens stored to the cache.
// KV-cache kinds.  A cache holds, per layer and KV head, max_seq rows, one per position:
//   kKvF32  hd fp32 values (the reference's kv_type 0);
//   kKvF16  hd fp16 values (env DPUF_CUDA_KV_F16, not a reference format);
//   kKvQ8   the reference's kv_type 1 (quantize_vec_q8_blk32, dpuf_engine.c:751-781): hd int8
//           values followed by hd/32 fp32 block scales in the same row, so that one
//           contiguous read fetches a key or value with its scales.
enum KvKind { kKvF32 = 0, kKvF16 = 1, kKvQ8 = 2 };
DPUF_HD size_t kv_row_bytes(int kind, int hd) {
  return kind == kKvF32 ? (size_t)hd * 4 : kind == kKvF16 ? (size_t)hd * 2 : (size_t)hd + hd / 8;
}
struct KvCache {
  float* k;  // rows [n_kv][max_seq] of this layer (raw storage of the cache's kind)
  float* v;
  int max_seq;
  // Batched decode (rows are independent sequences): token m's position tok_pos[m] and its
  // slot's cache tok_k[m] / tok_v[m] ([L][n_kv][max_seq] rows) + layer_off bytes; null: the
  // single cache above at positions *pos0 + m.
  const int32_t* tok_pos;
  float* const* tok_k;
  float* const* tok_v;
  size_t layer_off;  // bytes
  int kind;          // KvKind
};
// tok_cos / tok_sin (optional, [M][hd/2]): each token's rotation rows instead of the tables'
// rows at its cache position (forward_batch_ex rotary positions, M-RoPE).
cudaError_t launch_qk_post(const Launch& L, float* q, float* k, const float* v, int M, int n_q, int n_kv, int hd,
                           const float* q_norm, const float* k_norm, float eps, const float* cos_tab,
                           const float* sin_tab, const int* pos0_dev, KvCache kv, const float* tok_cos = nullptr,
                           const float* tok_sin = nullptr);
// Exact causal attention for M tokens, output [M][n_q*hd]: gqa_attn_head_pair_f32's order
// (fp32 and fp16 caches) or gqa_attn_head_pair_q8's (Q8 cache).
cudaError_t launch_attention(const Launch& L, const float* q, int M, int n_q, int n_kv, int hd, const int* pos0_dev,
                             KvCache kv, float* out, const ExpfTable& et);
// SwiGLU with dead-zone over [M][I] and prep of the result for w_down.  per_row: every row is
// its own batch-1 step (the reference's vector/scalar split of one row), else the split of one
// M-token step.
cudaError_t launch_swiglu_prep(const Launch& L, const float* gate, const float* up, int M, int I, float deadzone,
                               int nt_ref, const uint8_t* signs, Act out, const ExpfTable& et, bool per_row = false);
// Zero rows [r0, H) of out[M][H] (down-projection tile pruning).
cudaError_t launch_zero_rows(const Launch& L, float* out, int M, int H, int r0);
// out[i] += add[i] for i < n (DeepStack injection into the down projection's output).
cudaError_t launch_add_rows(const Launch& L, float* out, const float* add, int n);

// ---- kernels_lmhead.cu
// Zone-A test over logits[0, n): top-2 (b1, b2); flag = margin > 0 && b1 - b2 >= margin.
cudaError_t launch_zone_test(const Launch& L, const float* logits, int n, float margin, int* flag, float* b12);
// If *flag: logits[from, V) = -1e9.
cudaError_t launch_zone_mask(const Launch& L, float* logits, int from, int V, const int* flag);
// Greedy argmax over V logits on kArgmaxBlocks CTAs (part: kArgmaxBlocks partials; counter: one
// zero-initialised word, left at zero).  launch_argmax writes the index to *out;
// launch_greedy_advance feeds it back as the next decode step's token (ids[0], *pos0 += 1,
// hist[(*step)++]).
constexpr int kArgmaxBlocks = 148;
cudaError_t launch_argmax(const Launch& L, const float* logits, int V, float2* part, unsigned* counter, int32_t* out);
// First-index argmax of each of M rows [M][V] into out[M].
cudaError_t launch_argmax_rows(const Launch& L, const float* logits, int V, int M, int32_t* out);
cudaError_t launch_greedy_advance(const Launch& L, const float* logits, int V, float2* part, unsigned* counter,
                                  int32_t* ids, int32_t* pos0, int32_t* hist, int32_t* step);

// ---- kernels_decode.cu: batch-1 decode as one persistent cooperative kernel
// Device pointers of one layer (weights in container layout with a uniform tile stride).
struct DecLayer {
  const uint8_t* tiles[7];   // tile 0 of q, k, v, o, gate, up, down
  long long stride[7];       // bytes from one tile to the next
  const uint8_t* signs[4];   // sign tables of the inputs of q/k/v, o, gate/up, down
  const float* attn_norm;
  const float* ffn_norm;
  const float* q_norm;       // null without QK-norm
  const float* k_norm;
};
static_assert(sizeof(DecLayer) % 16 == 0, "layer table rows are copied as int4");

struct DecodeArgs {
  const DecLayer* layers;  // [L], device
  int L, H, I, nq, nkv, hd, qd, kvd, V, S, kmax, tok_rows;
  const uint8_t* lm_tiles;
  long long lm_stride;
  const uint8_t* lm_signs;
  const uint8_t* tok_tiles;
  long long tok_stride;
  const uint8_t* tok_signs;
  const float* out_norm;
  float eps, deadzone;
  int nt_ref;     // the reference's thread count (SwiGLU vector/tail split)
  int keep_down;  // down-projection tiles computed (rows beyond are zero)
  const float* cos_tab;
  const float* sin_tab;
  float* kv_k;    // active slot, [L][n_kv][S][hd]
  float* kv_v;
  ExpfTable et;
  // Vectors other CTAs (and ranks) produce are exchanged as tagged words: value bits in the low
  // half, the generation of the producing layer in the high half (one 64-bit store, so a reader
  // sees the value and its tag together).  Readers wait on the tags of the words they need; no
  // grid barrier separates the phases.
  uint64_t *q, *k, *v, *o_out, *d_out;  // [qd], [kvd] x2, [H], [H]
  // prepped projection inputs, 20 tagged words per 64-column chunk (16 words of four int8 codes,
  // 2 block scales, 2 block sums): the o projection's (written by the attention CTAs of this
  // GPU) and the down projection's (written by the warp holding each chunk's last gate/up pair)
  uint64_t *oprep, *dprep;            // [qd/64 * 20], [I/64 * 20]
  uint64_t* s_raw;                    // [I] SwiGLU outputs (tagged), read by the chunk's prep
  uint64_t* part;  // argmax partials [2 (LM generation parity)][ctas of all ranks][value, index]
  float* logits;   // [V] plain values, read by the host after the launch
  unsigned gen0;   // generation of this launch's first layer (L + 1 per step: layers, LM head)
  int* err;        // 0 at launch; 1 = a ring wait, 3 = a wait for another CTA's outputs timed out
  int32_t* hist;   // [n_steps] greedy ids
  int first_id, pos0, n_steps, write_logits;
  int grid, n_slots;                  // CTAs (one per SM); ring slots of a CTA
  int max_inflight;                   // ring stages a CTA may have requested but not received
  unsigned long long wait_ns;         // limit of every device wait
  int stall_unit;  // test hook: the CTA owning this q/k/v unit withholds its first outputs (-1: none)
  unsigned long long* trace;  // optional per-CTA phase timestamps of the last step (null: off)
  int trace_per_cta;
  // Tensor parallelism over tp_world processes (one GPU each; 1 = off).  Every projection's
  // units are dealt over all ranks' CTAs (virtual CTA blockIdx.x * tp_world + tp_rank); the
  // tagged vectors, the down input's raw values, counters and prep, the logits and the error
  // word live in an exchange buffer that every rank maps, and producers store to every rank's
  // copy (peer address = local + tp_delta[r]).
  int tp_rank, tp_world;
  long long tp_delta[kMaxTp];
};
// Exchange generations of one decode step (one per layer, one for the LM head).
DPUF_HD int decode_phases(int L) { return L + 1; }
constexpr int kDecodeConsWarps = 11;  // consumer warps of a decode CTA (plus one producer warp)
constexpr int kDecodeSvUnits = 24;    // gate/up units per decode CTA (SwiGLU outputs kept in shared memory)
size_t decode_smem_bytes(const DecodeArgs& A);
int decode_ring_slots(const DecodeArgs& A, size_t smem_limit);
int decode_trace_events(int L);
cudaError_t configure_decode_kernel();
cudaError_t decode_max_dyn_smem(size_t* bytes);
cudaError_t decode_blocks_per_sm(const DecodeArgs& A, int* blocks);
cudaError_t launch_decode(cudaStream_t stream, const DecodeArgs& A);

}  // namespace dpuf

