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
size_t gemv_split_pairs_bytes(int max_cols);
cudaError_t launch_gemv(const Launch& L, const LinJobs& jobs, const int* skip_flag, const GemvSplit* split);
// M > 1: exact integer-dot GEMM on CUDA cores (reference order per (token,row)).
cudaError_t launch_gemm_exact(const Launch& L, const LinJobs& jobs, int M);

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
struct KvCache {
  float* k;  // [n_kv][max_seq][hd] for this layer
  float* v;
  int max_seq;
};
cudaError_t launch_qk_post(const Launch& L, float* q, float* k, const float* v, int M, int n_q, int n_kv, int hd,
                           const float* q_norm, const float* k_norm, float eps, const float* cos_tab,
                           const float* sin_tab, const int* pos0_dev, KvCache kv);
// Exact causal attention (gqa_attn_head_pair_f32 order) for M tokens, output [M][n_q*hd].
cudaError_t launch_attention(const Launch& L, const float* q, int M, int n_q, int n_kv, int hd, const int* pos0_dev,
                             KvCache kv, float* out, const ExpfTable& et);
// SwiGLU with dead-zone over [M][I] and prep of the result for w_down.
cudaError_t launch_swiglu_prep(const Launch& L, const float* gate, const float* up, int M, int I, float deadzone,
                               int nt_ref, const uint8_t* signs, Act out, const ExpfTable& et);
// Zero rows [r0, H) of out[M][H] (down-projection tile pruning).
cudaError_t launch_zero_rows(const Launch& L, float* out, int M, int H, int r0);

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
cudaError_t launch_greedy_advance(const Launch& L, const float* logits, int V, float2* part, unsigned* counter,
                                  int32_t* ids, int32_t* pos0, int32_t* hist, int32_t* step);

}  // namespace dpuf
