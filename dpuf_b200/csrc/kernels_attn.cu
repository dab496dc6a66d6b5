// kernels_attn.cu - exact causal GQA attention over the KV cache, one CTA per (token, KV
// head, two pairs of Q heads) - the keys and values a CTA stages serve four query heads, so a
// KV head's cache is read once per token for groups of up to four; the arithmetic is
// attn_pair_body (layer_dev.cuh), a restatement of gqa_attn_head_pair_f32
// (dpuf_engine.c:341-577), pair by pair.
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

struct CtaSync {
  DPUF_DEV void operator()() const { __syncthreads(); }
};

template <typename T>  // cache element: float, or __half for an fp16 cache
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* __restrict__ q, int n_q, int n_kv, int hd,
                                                                  const int* __restrict__ pos0_dev, KvCache kv,
                                                                  float* __restrict__ out, ExpfTable et) {
  extern __shared__ __align__(16) float sm[];
  __shared__ AttnShared sh;
  cudaGridDependencySynchronize();
  const int m = blockIdx.x, kvh = blockIdx.y;
  int ppc, n_buf;
  attn_step_plan(hd, kv.max_seq, &ppc, &n_buf, (int)sizeof(T));
  const int groups = n_q / n_kv;
  const int g0 = blockIdx.z * 2 * ppc;
  const int nh = min(2 * ppc, groups - g0);  // the last head of an odd group is a lone head
  const int qh0 = kvh * groups + g0;
  const int kv_len = (kv.tok_pos ? kv.tok_pos[m] : *pos0_dev + m) + 1;
  const T* kbase = kv.tok_k ? (const T*)((const char*)kv.tok_k[m] + kv.layer_off) : (const T*)kv.k;
  const T* vbase = kv.tok_v ? (const T*)((const char*)kv.tok_v[m] + kv.layer_off) : (const T*)kv.v;
  const int sc_stride = (kv.max_seq + 3) & ~3;
  float* qs = sm;                                 // [2 ppc][hd]
  float* sc = qs + 2 * ppc * hd;                  // [2 ppc][sc_stride]
  T* kt = (T*)(sc + (size_t)2 * ppc * sc_stride);  // [n_buf][kAttnKeyTile][hd + pad]
  for (int i = threadIdx.x; i < nh * hd; i += blockDim.x) qs[i] = q[((size_t)m * n_q + qh0) * hd + i];
  attn_pair_body(qs, nh, (nh & 1) != 0, hd, kv_len, kbase + (size_t)kvh * kv.max_seq * hd,
                 vbase + (size_t)kvh * kv.max_seq * hd, sc_stride, sc, kt, n_buf, 0, nullptr, nullptr, &sh,
                 out + ((size_t)m * n_q + qh0) * hd, et, (int)threadIdx.x, CtaSync{});
}

// The Q8 cache (kv_type 1): the same grid and scratch plan over Q8 tiles, arithmetic
// attn_q8_body (gqa_attn_head_pair_q8, dpuf_engine.c:621-749).
__global__ void __launch_bounds__(kAttnThreads) attention_q8_kernel(const float* __restrict__ q, int n_q, int n_kv,
                                                                     int hd, const int* __restrict__ pos0_dev,
                                                                     KvCache kv, float* __restrict__ out,
                                                                     ExpfTable et) {
  extern __shared__ __align__(16) float sm[];
  __shared__ AttnShared sh;
  cudaGridDependencySynchronize();
  const int m = blockIdx.x, kvh = blockIdx.y;
  int ppc, n_buf;
  attn_step_plan(hd, kv.max_seq, &ppc, &n_buf, 1);
  const int groups = n_q / n_kv;
  const int g0 = blockIdx.z * 2 * ppc;
  const int nh = min(2 * ppc, groups - g0);
  const int qh0 = kvh * groups + g0;
  const int kv_len = (kv.tok_pos ? kv.tok_pos[m] : *pos0_dev + m) + 1;
  const size_t head_bytes = (size_t)kv.max_seq * kv_row_bytes(kKvQ8, hd);
  const char* kbase = kv.tok_k ? (const char*)kv.tok_k[m] + kv.layer_off : (const char*)kv.k;
  const char* vbase = kv.tok_v ? (const char*)kv.tok_v[m] + kv.layer_off : (const char*)kv.v;
  const int sc_stride = (kv.max_seq + 3) & ~3;
  float* qs = sm;                                       // [2 ppc][hd]
  float* sc = qs + 2 * ppc * hd;                        // [2 ppc][sc_stride]
  char* kt = (char*)(sc + (size_t)2 * ppc * sc_stride);  // [n_buf][kAttnKeyTile] Q8 rows
  for (int i = threadIdx.x; i < nh * hd; i += blockDim.x) qs[i] = q[((size_t)m * n_q + qh0) * hd + i];
  attn_q8_body(qs, nh, (nh & 1) != 0, hd, kv_len, kbase + kvh * head_bytes, vbase + kvh * head_bytes, sc_stride, sc,
               kt, n_buf, &sh, out + ((size_t)m * n_q + qh0) * hd, et, (int)threadIdx.x, CtaSync{});
}

}  // namespace

cudaError_t configure_attn_kernels() {
  cudaError_t e = set_max_dyn_smem(attention_kernel<float>);
  if (e == cudaSuccess) e = set_max_dyn_smem(attention_kernel<__half>);
  return e != cudaSuccess ? e : set_max_dyn_smem(attention_q8_kernel);
}

cudaError_t launch_attention(const Launch& L, const float* q, int M, int n_q, int n_kv, int hd, const int* pos0_dev,
                             KvCache kv, float* out, const ExpfTable& et) {
  int ppc, n_buf;
  const int es = kv.kind == kKvQ8 ? 1 : kv.kind == kKvF16 ? 2 : 4;
  attn_step_plan(hd, kv.max_seq, &ppc, &n_buf, es);
  const int groups = n_q / n_kv;
  const size_t smem = attn_step_floats(hd, kv.max_seq, ppc, n_buf, es) * sizeof(float);
  if (smem > kMaxDynSmem) return cudaErrorInvalidValue;
  const dim3 grid(M, n_kv, (groups + 2 * ppc - 1) / (2 * ppc));
  if (kv.kind == kKvQ8)
    return launch_k(L, attention_q8_kernel, grid, dim3(kAttnThreads), smem, q, n_q, n_kv, hd, pos0_dev, kv, out, et);
  if (kv.kind == kKvF16)
    return launch_k(L, attention_kernel<__half>, grid, dim3(kAttnThreads), smem, q, n_q, n_kv, hd, pos0_dev, kv, out, et);
  return launch_k(L, attention_kernel<float>, grid, dim3(kAttnThreads), smem, q, n_q, n_kv, hd, pos0_dev, kv, out, et);
}

}  // namespace dpuf
