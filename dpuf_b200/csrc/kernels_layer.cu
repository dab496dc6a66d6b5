// kernels_layer.cu - per-layer pointwise and row-reduction kernels with the reference's
// exact fp32 operation order: residual add + RMSNorm + mode-12 prep, QK RMSNorm + NeoX RoPE
// + KV-cache store, SwiGLU with dead-zone + prep of the down-projection input.
#include <algorithm>

#include "kernels.cuh"
#include "layer_dev.cuh"

namespace dpuf {

namespace {

template <typename K, typename... Args>
cudaError_t launch_k(const Launch& L, K kernel, dim3 grid, dim3 block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = L.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

struct PrepTargets {
  PrepTarget t[3];
  int n;
};

// ------------------------------------------------------------------ residual + RMSNorm + prep
// add_and_rms_norm_f32 (dpuf_engine.c:244-272): s = h + res (stored back to h); "AVX lane" j
// accumulates fma(s_i, s_i, .) over i = j, j+8, ... in order; ss = split tree; the n % 8 tail
// is added sequentially; inv = 1 / sqrt(ss / n + eps); out_i = (s_i * inv) * w_i.
// One CTA per token.  Eight threads run the eight sequential chains.
__global__ void __launch_bounds__(1024) norm_prep_kernel(float* __restrict__ h, const float* __restrict__ res,
                                                         const float* __restrict__ w, float eps, int H, PrepTargets T,
                                                         float* __restrict__ norm_out) {
  extern __shared__ __align__(16) float S[];  // [H]
  __shared__ float lanes[8];
  __shared__ float inv_s;
  cudaGridDependencySynchronize();
  const int m = blockIdx.x;
  float* hr = h + (size_t)m * H;
  const float* rr = res ? res + (size_t)m * H : nullptr;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float s = hr[i];
    if (rr) {
      s = __fadd_rn(s, rr[i]);
      hr[i] = s;
    }
    S[i] = s;
  }
  __syncthreads();
  if (threadIdx.x < 8) lanes[threadIdx.x] = sumsq_lane(S, H & ~7, threadIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) inv_s = rms_inv(lanes, S, H, eps);
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float o = __fmul_rn(__fmul_rn(S[i], inv), w[i]);
    S[i] = o;
    if (norm_out) norm_out[(size_t)m * H + i] = o;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int k = 0; k < T.n; k++) {
    const Act& a = T.t[k].act;
    for (int c = warp; c < H / 64; c += nw) {
      const int c0 = c * 64;
      prep_chunk_warp(S[c0 + lane], S[c0 + 32 + lane], T.t[k].signs, c0, lane, a.q8 + (size_t)m * a.ld,
                      a.xs + (size_t)m * (a.ld >> 5), a.xm + (size_t)m * (a.ld >> 5));
    }
  }
}

// ------------------------------------------------------------------ QK-norm + RoPE + KV store
// Per (token, head) (dpuf_engine.c:1788-1822 / 1840-1879): RMSNorm over head_dim with the
// head's norm gain (same lane/tree order as above), NeoX rotation with host cos/sin tables
// (apply_rope_neox_f32, dpuf_engine.c:274-295: x1*c - x2*s and x2*c + x1*s as fused
// multiply-subtract/add of the rounded cross product), then K and V rows are written to the
// cache at position pos0 + m: as fp32, fp16, or quantized Q8 rows.  One warp per head vector.
__global__ void qk_post_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v, int n_q,
                               int n_kv, int hd, const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                               float eps, const float* __restrict__ cos_tab, const float* __restrict__ sin_tab,
                               const int* __restrict__ pos0_dev, KvCache kv, const float* __restrict__ tok_cos,
                               const float* __restrict__ tok_sin) {
  extern __shared__ __align__(16) float sv[];  // [warps][hd]
  cudaGridDependencySynchronize();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.x;
  const int hidx = blockIdx.y * (blockDim.x >> 5) + warp;
  if (hidx >= n_q + n_kv) return;
  const int pos = kv.tok_pos ? kv.tok_pos[m] : *pos0_dev + m;
  char* const kbase = (char*)(kv.tok_k ? kv.tok_k[m] : kv.k) + (kv.tok_k ? kv.layer_off : 0);
  char* const vbase = (char*)(kv.tok_v ? kv.tok_v[m] : kv.v) + (kv.tok_v ? kv.layer_off : 0);
  const bool is_k = hidx < n_kv;
  const int head = is_k ? hidx : hidx - n_kv;
  float* vec = is_k ? k + ((size_t)m * n_kv + head) * hd : q + ((size_t)m * n_q + head) * hd;
  const float* nw = is_k ? k_norm : q_norm;
  float* s = sv + warp * hd;
  for (int i = lane; i < hd; i += 32) s[i] = vec[i];
  __syncwarp();
  const size_t rrow = tok_cos ? (size_t)m * (hd >> 1) : (size_t)pos * (hd >> 1);
  qk_norm_rope_warp(s, nw, eps, hd, (tok_cos ? tok_cos : cos_tab) + rrow, (tok_sin ? tok_sin : sin_tab) + rrow, lane);
  for (int i = lane; i < hd; i += 32) vec[i] = s[i];
  if (!is_k) return;
  // this head's cache row at pos (kv_row_bytes per row)
  const size_t row = ((size_t)head * kv.max_seq + pos) * kv_row_bytes(kv.kind, hd);
  const float* vr = v + ((size_t)m * n_kv + head) * hd;
  if (kv.kind == kKvQ8) {  // quantize_vec_q8_blk32 of K and V (dpuf_engine.c:1801-1802)
    q8_row_warp(s, kbase + row, hd, lane);
    q8_row_warp(vr, vbase + row, hd, lane);
    return;
  }
  for (int i = lane; i < hd; i += 32) {
    if (kv.kind == kKvF16) {
      ((__half*)(kbase + row))[i] = __float2half_rn(s[i]);
      ((__half*)(vbase + row))[i] = __float2half_rn(vr[i]);
    } else {
      ((float*)(kbase + row))[i] = s[i];
      ((float*)(vbase + row))[i] = vr[i];
    }
  }
}

// ------------------------------------------------------------------ SwiGLU + prep for w_down
// swiglu_one per element (layer_dev.cuh), then the prep of each 64-column chunk.
__global__ void swiglu_prep_kernel(const float* __restrict__ gate, const float* __restrict__ up, int M, int I,
                                   float dz, int nt, const uint8_t* __restrict__ signs, Act out, ExpfTable et,
                                   bool per_row) {
  cudaGridDependencySynchronize();
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int m = blockIdx.y;
  if (chunk * 64 >= I) return;
  const int c0 = chunk * 64;
  const long long total = per_row ? I : (long long)M * I;
  const bool slab = !per_row && (M >= 2) && ((M + 5) / 6 >= nt);
  const long long ia = (long long)m * I + c0 + lane, ib = ia + 32;
  const long long ea = per_row ? c0 + lane : ia, eb = ea + 32;  // element index within the split
  const float a = swiglu_one(gate[ia], up[ia], dz, swiglu_vector_elem(ea, total, nt, slab), et);
  const float b = swiglu_one(gate[ib], up[ib], dz, swiglu_vector_elem(eb, total, nt, slab), et);
  prep_chunk_warp(a, b, signs, c0, lane, out.q8 + (size_t)m * out.ld, out.xs + (size_t)m * (out.ld >> 5),
                  out.xm + (size_t)m * (out.ld >> 5));
}

__global__ void zero_rows_kernel(float* __restrict__ out, int H, int r0) {
  cudaGridDependencySynchronize();
  const int m = blockIdx.y;
  for (int i = r0 + blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) out[(size_t)m * H + i] = 0.0f;
}

}  // namespace

cudaError_t configure_layer_kernels() {
  return set_max_dyn_smem(norm_prep_kernel);
}

cudaError_t launch_norm_prep(const Launch& L, float* h, const float* res, const float* w, float eps, int M, int H,
                             const PrepTarget* targets, int n_targets, float* norm_out) {
  PrepTargets T = {};
  T.n = n_targets;
  for (int i = 0; i < n_targets && i < 3; i++) T.t[i] = targets[i];
  const int threads = H >= 4096 ? 1024 : (H >= 1024 ? 512 : 256);
  const size_t smem = (size_t)H * sizeof(float);
  if (smem > kMaxDynSmem) return cudaErrorInvalidValue;
  return launch_k(L, norm_prep_kernel, dim3(M), dim3(threads), smem, h, res, w, eps, H, T, norm_out);
}

cudaError_t launch_qk_post(const Launch& L, float* q, float* k, const float* v, int M, int n_q, int n_kv, int hd,
                           const float* q_norm, const float* k_norm, float eps, const float* cos_tab,
                           const float* sin_tab, const int* pos0_dev, KvCache kv, const float* tok_cos,
                           const float* tok_sin) {
  const int wpb = 4;
  const int heads = n_q + n_kv;
  return launch_k(L, qk_post_kernel, dim3(M, (heads + wpb - 1) / wpb), dim3(wpb * 32), (size_t)wpb * hd * 4, q, k, v,
                  n_q, n_kv, hd, q_norm, k_norm, eps, cos_tab, sin_tab, pos0_dev, kv, tok_cos, tok_sin);
}

cudaError_t launch_swiglu_prep(const Launch& L, const float* gate, const float* up, int M, int I, float deadzone,
                               int nt_ref, const uint8_t* signs, Act out, const ExpfTable& et, bool per_row) {
  const int chunks = I / 64, wpb = 8;
  return launch_k(L, swiglu_prep_kernel, dim3((chunks + wpb - 1) / wpb, M), dim3(wpb * 32), 0, gate, up, M, I,
                  deadzone, nt_ref, signs, out, et, per_row);
}

__global__ void add_rows_kernel(float* __restrict__ out, const float* __restrict__ add, int n) {
  cudaGridDependencySynchronize();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = __fadd_rn(out[i], add[i]);
}

cudaError_t launch_add_rows(const Launch& L, float* out, const float* add, int n) {
  return launch_k(L, add_rows_kernel, dim3(std::min((n + 255) / 256, 1184)), dim3(256), 0, out, add, n);
}

cudaError_t launch_zero_rows(const Launch& L, float* out, int M, int H, int r0) {
  if (r0 >= H) return cudaSuccess;
  const int n = H - r0;
  return launch_k(L, zero_rows_kernel, dim3((n + 255) / 256, M), dim3(256), 0, out, H, r0);
}

}  // namespace dpuf
