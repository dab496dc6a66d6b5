// ops_abi.cu - standalone mode-12 ops behind the reference's exported signatures
// (dpuf_kernels.h:267-277; dpuf_avx2.c:2678-2783) and device-resident weight handles.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>

#include "dpuf_cuda.h"
#include "dpuf_kernels.h"
#include "engine_internal.h"
#include "kernels.cuh"

namespace dpuf {
namespace {

struct W12Handle {
  int device = 0;
  W12 w{};
  unsigned char* mem = nullptr;
  int8_t* q8 = nullptr;
  float* xs = nullptr;
  int32_t* xm = nullptr;
  GemvSplit split{};  // GEMV scratch (units shared by CTAs)
  int* tc_err = nullptr;  // error word of the tensor-core GEMM (and [1]: the expansion's flag)
  uint8_t* x8 = nullptr;  // expanded copy for the tensor-core GEMM (w.x8), or null
};

constexpr int kOpChunk = kMaxBatch;  // tokens per launch of the standalone matmul

bool fail(const char* where, cudaError_t e) {
  set_error(std::string(where) + ": " + cudaGetErrorString(e));
  return false;
}

// Uploads tiles [0, n_tiles) of a mode-12 matrix; the span end comes from the last tile's row
// count because the ABI does not pass tile_offsets[n_tiles].
bool upload(W12Handle* h, int rows, int cols, int n_tiles, const uint8_t* base, const uint64_t* toff,
            const uint8_t* signs) {
  if (cols <= 0 || cols % 64 != 0 || n_tiles <= 0 || !base || !toff) {
    set_error("bad mode-12 descriptor");
    return false;
  }
  uint64_t lo = toff[0], hi = 0;
  const int n_blk = cols / 32;
  for (int t = 0; t < n_tiles; t++) {
    if (toff[t] % 16 != 0) {
      set_error("tile offsets must be multiples of 16 bytes");
      return false;
    }
    const uint8_t* tp = base + toff[t];
    const int n_r = tp[4] | (tp[5] << 8);
    lo = std::min<uint64_t>(lo, toff[t]);
    hi = std::max<uint64_t>(hi, toff[t] + 16 + (uint64_t)((n_r + 7) / 8) * n_blk * 144);
  }
  const size_t span = (size_t)(hi - lo);
  const size_t off_toff = (span + 255) & ~(size_t)255;
  const size_t off_sign = (off_toff + (size_t)n_tiles * 8 + 255) & ~(size_t)255;
  const size_t total = off_sign + (size_t)cols / 8;
  cudaError_t e;
  if ((e = cudaGetDevice(&h->device)) != cudaSuccess) return fail("cudaGetDevice", e);
  if ((e = configure_kernels()) != cudaSuccess) return fail("kernel attributes", e);
  if ((e = cudaMalloc(&h->mem, total)) != cudaSuccess) return fail("cudaMalloc", e);
  if ((e = cudaMemcpy(h->mem, base + lo, span, cudaMemcpyHostToDevice)) != cudaSuccess) return fail("upload", e);
  std::string toffs((size_t)n_tiles * 8, '\0');
  uint64_t* tp = (uint64_t*)&toffs[0];
  for (int t = 0; t < n_tiles; t++) tp[t] = toff[t] - lo;
  if ((e = cudaMemcpy(h->mem + off_toff, tp, (size_t)n_tiles * 8, cudaMemcpyHostToDevice)) != cudaSuccess)
    return fail("upload", e);
  if (signs && (e = cudaMemcpy(h->mem + off_sign, signs, (size_t)cols / 8, cudaMemcpyHostToDevice)) != cudaSuccess)
    return fail("upload", e);
  h->w = W12{h->mem, (const uint64_t*)(h->mem + off_toff), signs ? h->mem + off_sign : nullptr, rows, cols, n_tiles};
  return true;
}

bool alloc_act(W12Handle* h) {
  const size_t cols = h->w.cols;
  cudaError_t e;
  if ((e = cudaMalloc(&h->q8, kOpChunk * cols)) != cudaSuccess) return fail("cudaMalloc", e);
  if ((e = cudaMalloc(&h->xs, kOpChunk * (cols / 32) * 4)) != cudaSuccess) return fail("cudaMalloc", e);
  if ((e = cudaMalloc(&h->xm, kOpChunk * (cols / 32) * 4)) != cudaSuccess) return fail("cudaMalloc", e);
  if ((e = cudaMalloc(&h->split.pairs, gemv_split_pairs_bytes((int)cols))) != cudaSuccess ||
      (e = cudaMalloc(&h->split.acc, (size_t)kGemvMaxCtas * kTileRows * sizeof(float))) != cudaSuccess ||
      (e = cudaMalloc(&h->split.count, (size_t)kGemvMaxCtas * sizeof(unsigned))) != cudaSuccess ||
      (e = cudaMemset(h->split.count, 0, (size_t)kGemvMaxCtas * sizeof(unsigned))) != cudaSuccess ||
      (e = cudaMalloc(&h->tc_err, 16)) != cudaSuccess || (e = cudaMemset(h->tc_err, 0, 16)) != cudaSuccess)
    return fail("cudaMalloc", e);
  return true;
}

// M > 1 on the tensor cores unless env DPUF_CUDA_TC_GEMM=0 (the exact dp4a GEMM).
bool tc_gemm_enabled() {
  const char* v = getenv("DPUF_CUDA_TC_GEMM");
  return !v || atoi(v) != 0;
}

// The expanded copy of the matrix for the tensor-core GEMM, unless env DPUF_CUDA_TC_EXPAND=0.
// When the allocation fails, or a stored scale is not finite, the GEMM unpacks the tiles itself.
bool expand(W12Handle* h) {
  const char* v = getenv("DPUF_CUDA_TC_EXPAND");
  if (v && atoi(v) == 0) return true;
  if (cudaMalloc(&h->x8, x8_bytes(h->w)) != cudaSuccess) {
    cudaGetLastError();  // not fatal
    h->x8 = nullptr;
    return true;
  }
  int bad = 0;
  cudaError_t e;
  if ((e = cudaMemset(h->tc_err + 1, 0, 4)) != cudaSuccess || (e = launch_x8_expand(0, h->w, h->x8, h->tc_err + 1)) ||
      (e = cudaMemcpy(&bad, h->tc_err + 1, 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
    return fail("expanded weights", e);
  if (bad) {
    cudaFree(h->x8);
    h->x8 = nullptr;
  }
  h->w.x8 = h->x8;
  return true;
}

void free_handle(W12Handle* h) {
  if (!h) return;
  cudaFree(h->x8);
  cudaFree(h->mem);
  cudaFree(h->q8);
  cudaFree(h->xs);
  cudaFree(h->xm);
  cudaFree(h->split.pairs);
  cudaFree(h->split.acc);
  cudaFree(h->split.count);
  cudaFree(h->tc_err);
  delete h;
}

// y = W x for M tokens, device pointers, in chunks of kOpChunk tokens.
int32_t matmul_dev(W12Handle* h, int M, const float* x, float* y, cudaStream_t s) {
  const Launch L{s, false};
  const Act a{h->q8, h->xs, h->xm, h->w.cols};
  for (int m0 = 0; m0 < M; m0 += kOpChunk) {
    const int mc = std::min(kOpChunk, M - m0);
    cudaError_t e = launch_prep(L, x + (size_t)m0 * h->w.cols, h->w.cols, mc, h->w.cols, h->w.signs, a);
    if (e != cudaSuccess) return fail("prep", e), -4;
    LinJobs J = {};
    J.n = 1;
    J.j[0] = {h->w, a, y + (size_t)m0 * h->w.rows, h->w.rows, 0, h->w.n_tiles};
    J.tile_prefix[1] = h->w.n_tiles;
    e = mc == 1 ? launch_gemv(L, J, nullptr, &h->split)
                : (tc_gemm_enabled() ? launch_gemm_tc(L, J, mc, h->tc_err) : launch_gemm_exact(L, J, mc));
    if (e != cudaSuccess) return fail("matmul", e), -4;
  }
  return 0;
}

// Error word of the tensor-core GEMM after the stream has been synchronised.
int32_t matmul_status(W12Handle* h) {
  int v = 0;
  if (cudaMemcpy(&v, h->tc_err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -4;
  if (v) {
    set_error("tensor-core GEMM: an MMA wait timed out");
    return -6;
  }
  return 0;
}

}  // namespace
}  // namespace dpuf

using dpuf::W12Handle;

extern "C" {

DPUF_EXPORT void* dpuf_cuda_w12_upload(const DpufWeightDesc* w) {
  if (!w || w->mode != DPUF_MODE_QR_HAD4_PACKED) {
    dpuf::set_error("dpuf_cuda_w12_upload: mode-12 descriptor required");
    return nullptr;
  }
  W12Handle* h = new W12Handle();
  if (!dpuf::upload(h, w->rows, w->cols, w->n_tiles, w->tensor_base, w->tile_offsets, w->sign_bits) ||
      !dpuf::alloc_act(h) || !dpuf::expand(h)) {
    dpuf::free_handle(h);
    return nullptr;
  }
  return h;
}

DPUF_EXPORT void dpuf_cuda_w12_free(void* wh) { dpuf::free_handle((W12Handle*)wh); }

DPUF_EXPORT int32_t dpuf_cuda_matmul_dev(void* wh, int32_t M, const float* x_dev, float* y_dev, void* stream) {
  W12Handle* h = (W12Handle*)wh;
  if (!h || M <= 0 || !x_dev || !y_dev) return -1;
  return dpuf::matmul_dev(h, M, x_dev, y_dev, (cudaStream_t)stream);
}

// Kernel-only timing: preps x once per handle, then launches only the matmul kernel `iters`
// times, rotating over the handles (so the weights streamed exceed L2), bracketed by CUDA
// events on `stream`.  *ms_out = average milliseconds per launch.
DPUF_EXPORT int32_t dpuf_cuda_matmul_dev_timed(void** whs, int32_t n_handles, int32_t M, const float* x_dev,
                                               float* y_dev, int32_t iters, void* stream, float* ms_out) {
  if (!whs || n_handles <= 0 || M <= 0 || M > dpuf::kOpChunk || iters <= 0 || !ms_out) return -1;
  cudaStream_t s = (cudaStream_t)stream;
  const dpuf::Launch L{s, false};
  for (int i = 0; i < n_handles; i++) {
    W12Handle* h = (W12Handle*)whs[i];
    const dpuf::Act a{h->q8, h->xs, h->xm, h->w.cols};
    if (dpuf::launch_prep(L, x_dev, h->w.cols, M, h->w.cols, h->w.signs, a) != cudaSuccess) return -4;
  }
  auto launch = [&](int i) {
    W12Handle* h = (W12Handle*)whs[i % n_handles];
    const dpuf::Act a{h->q8, h->xs, h->xm, h->w.cols};
    dpuf::LinJobs J = {};
    J.n = 1;
    J.j[0] = {h->w, a, y_dev, h->w.rows, 0, h->w.n_tiles};
    J.tile_prefix[1] = h->w.n_tiles;
    return M == 1 ? dpuf::launch_gemv(L, J, nullptr, &h->split)
                  : (dpuf::tc_gemm_enabled() ? dpuf::launch_gemm_tc(L, J, M, h->tc_err)
                                             : dpuf::launch_gemm_exact(L, J, M));
  };
  for (int i = 0; i < 2 * n_handles; i++)
    if (launch(i) != cudaSuccess) return -4;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) || cudaEventCreate(&e1)) return -4;
  cudaEventRecord(e0, s);
  for (int i = 0; i < iters; i++)
    if (launch(i) != cudaSuccess) return -4;
  cudaEventRecord(e1, s);
  float ms = 0;
  const bool ok = cudaEventSynchronize(e1) == cudaSuccess && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (!ok) return -4;
  *ms_out = ms / iters;
  return 0;
}

// LM head with the Zone-A early exit on n_vec hidden vectors (already RMS-normalised), one at
// a time as batch-1 decode steps, with the engine's step kernels (dpuf_engine.c:2091-2139):
// prep, rows of tiles [0, Z), top-2 test over logits [0, min(16Z, V)), the remaining tiles
// unless the test exits, logits [16Z, V) := -1e9 on exit, first-index argmax.  Z is clamped to
// [256, n_tiles] as the engine does; margin <= 0 never exits.
DPUF_EXPORT int32_t dpuf_cuda_zone_head(void* wh, int32_t n_vec, const float* x_dev, int32_t zone_tiles,
                                        float margin, int32_t* ids_out, int32_t* exits_out, float* ms_out) {
  W12Handle* h = (W12Handle*)wh;
  if (!h || n_vec <= 0 || !x_dev || !ids_out || !exits_out) return -1;
  const int V = h->w.rows, cols = h->w.cols, nt = h->w.n_tiles;
  const int za = std::min(std::max(zone_tiles, 256), nt);
  float *logits = nullptr, *b12 = nullptr;
  int* flag = nullptr;
  float2* part = nullptr;
  unsigned* counter = nullptr;
  int32_t *ids_d = nullptr, *exits_d = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int32_t rc = 0;
  auto ck = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == 0) {
      dpuf::set_error(std::string(what) + ": " + cudaGetErrorString(e));
      rc = -4;
    }
    return rc == 0;
  };
  if (ck(cudaMalloc(&logits, (size_t)V * 4), "cudaMalloc") && ck(cudaMalloc(&b12, 16), "cudaMalloc") &&
      ck(cudaMalloc(&flag, 16), "cudaMalloc") && ck(cudaMalloc(&part, dpuf::kArgmaxBlocks * sizeof(float2)), "cudaMalloc") &&
      ck(cudaMalloc(&counter, 64), "cudaMalloc") && ck(cudaMemset(counter, 0, 64), "cudaMemset") &&
      ck(cudaMalloc(&ids_d, (size_t)n_vec * 4), "cudaMalloc") && ck(cudaMalloc(&exits_d, (size_t)n_vec * 4), "cudaMalloc") &&
      ck(cudaEventCreate(&e0), "event") && ck(cudaEventCreate(&e1), "event")) {
    const dpuf::Launch L{nullptr, false};
    const dpuf::Act a{h->q8, h->xs, h->xm, cols};
    ck(cudaEventRecord(e0, nullptr), "event");
    for (int i = 0; i < n_vec && rc == 0; i++) {
      dpuf::LinJobs J0 = {}, J1 = {};
      J0.n = J1.n = 1;
      J0.j[0] = {h->w, a, logits, V, 0, za};
      J0.tile_prefix[1] = za;
      J1.j[0] = {h->w, a, logits, V, za, nt};
      J1.tile_prefix[1] = nt - za;
      ck(dpuf::launch_prep(L, x_dev + (size_t)i * cols, cols, 1, cols, h->w.signs, a), "prep") &&
          ck(dpuf::launch_gemv(L, J0, nullptr, &h->split), "zone gemv") &&
          ck(dpuf::launch_zone_test(L, logits, std::min(za * dpuf::kTileRows, V), margin, flag, b12), "zone test") &&
          ck(za < nt ? dpuf::launch_gemv(L, J1, flag, &h->split) : cudaSuccess, "rest gemv") &&
          ck(dpuf::launch_zone_mask(L, logits, za * dpuf::kTileRows, V, flag), "zone mask") &&
          ck(dpuf::launch_argmax(L, logits, V, part, counter, ids_d + i), "argmax") &&
          ck(cudaMemcpyAsync(exits_d + i, flag, 4, cudaMemcpyDeviceToDevice, nullptr), "copy");
    }
    ck(cudaEventRecord(e1, nullptr), "event");
    float ms = 0.0f;
    if (ck(cudaEventSynchronize(e1), "sync") && ck(cudaEventElapsedTime(&ms, e0, e1), "event") && ms_out) *ms_out = ms;
    ck(cudaMemcpy(ids_out, ids_d, (size_t)n_vec * 4, cudaMemcpyDeviceToHost), "copy");
    ck(cudaMemcpy(exits_out, exits_d, (size_t)n_vec * 4, cudaMemcpyDeviceToHost), "copy");
  }
  cudaFree(logits); cudaFree(b12); cudaFree(flag); cudaFree(part); cudaFree(counter); cudaFree(ids_d); cudaFree(exits_d);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  return rc;
}

// Reference signature (dpuf_avx2.c:2678): host in, host out, synchronous.
DPUF_EXPORT void dpuf_matmul_qr_hadamard4_packed_f32(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                                     const float* x_in, const uint8_t* tensor_base,
                                                     const uint64_t* tile_offsets, const uint8_t* sign_bits,
                                                     float* out) {
  dpuf::set_error("");
  if (M <= 0 || !x_in || !out) return;
  W12Handle* h = new W12Handle();
  float *dx = nullptr, *dy = nullptr;
  if (dpuf::upload(h, rows, cols, n_tiles, tensor_base, tile_offsets, sign_bits) && dpuf::alloc_act(h) &&
      (M == 1 || dpuf::expand(h)) && cudaMalloc(&dx, (size_t)M * cols * 4) == cudaSuccess && cudaMalloc(&dy, (size_t)M * rows * 4) == cudaSuccess &&
      cudaMemcpy(dx, x_in, (size_t)M * cols * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
      dpuf::matmul_dev(h, M, dx, dy, nullptr) == 0) {
    cudaError_t e = cudaMemcpy(out, dy, (size_t)M * rows * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) dpuf::set_error(cudaGetErrorString(e));
    else if (M > 1) dpuf::matmul_status(h);
  }
  cudaFree(dx);
  cudaFree(dy);
  dpuf::free_handle(h);
}

// Reference signature (dpuf_avx2.c:2738): rows are looked up by id; only the tiles up to the
// largest id are uploaded.
DPUF_EXPORT void dpuf_embed_qr_hadamard4_packed_f32(int32_t n_tokens, int32_t cols, const int32_t* token_ids,
                                                    const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                                    const uint8_t* sign_bits, float* out) {
  dpuf::set_error("");
  if (n_tokens <= 0 || !token_ids || !out) return;
  int32_t max_id = 0;
  for (int i = 0; i < n_tokens; i++) {
    if (token_ids[i] < 0) {
      dpuf::set_error("negative token id");
      return;
    }
    max_id = std::max(max_id, token_ids[i]);
  }
  const int n_tiles = max_id / dpuf::kTileRows + 1;
  W12Handle* h = new W12Handle();
  int32_t* dids = nullptr;
  float* dy = nullptr;
  if (dpuf::upload(h, n_tiles * dpuf::kTileRows, cols, n_tiles, tensor_base, tile_offsets, sign_bits) &&
      cudaMalloc(&dids, (size_t)n_tokens * 4) == cudaSuccess &&
      cudaMalloc(&dy, (size_t)n_tokens * cols * 4) == cudaSuccess &&
      cudaMemcpy(dids, token_ids, (size_t)n_tokens * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
    const dpuf::Launch L{nullptr, false};
    for (int m0 = 0; m0 < n_tokens; m0 += 65535) {
      const int mc = std::min(65535, n_tokens - m0);
      if (dpuf::launch_embed(L, h->w, dids + m0, mc, dy + (size_t)m0 * cols) != cudaSuccess) break;
    }
    cudaError_t e = cudaMemcpy(out, dy, (size_t)n_tokens * cols * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) dpuf::set_error(cudaGetErrorString(e));
  }
  cudaFree(dids);
  cudaFree(dy);
  dpuf::free_handle(h);
}

}  // extern "C"
