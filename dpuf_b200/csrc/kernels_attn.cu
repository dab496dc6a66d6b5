// kernels_attn.cu - exact causal GQA attention over the fp32 KV cache.
//
// Reproduces gqa_attn_head_pair_f32 (dpuf_engine.c:341-577) bit for bit, per (token, KV head,
// pair of Q heads):
//   scores  keys t < kv_len & ~3: eight lanes accumulate fma(q_i, k_i) over i = l, l+8, ...;
//           "pairs" tree (hsum4_256_ps); keys in the kv_len % 4 tail: "split" tree
//           (eng_hsum256_ps) - for a lone head the tail uses dot_f32_avx2's two accumulators
//           over 16-wide steps, summed lane-wise before the split tree; then * 1/sqrt(hd).
//   softmax e_k = exp_poly(s_k - max) for k < kv_len & ~7, lane sums over k = j mod 8 in
//           order, split tree, then the tail adds glibc expf(s_k - max) sequentially;
//           p_k = e_k * (1 / (sum + 1e-12)).
//   PV      per output dim: fma(p_k, v_kd, acc) over k ascending (pair path); the lone-head
//           path takes keys two at a time, k+1 first (dpuf_engine.c:541-548).
#include "kernels.cuh"

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

constexpr int kAttnThreads = 256;
constexpr int kKeyTile = 32;  // keys staged per pass (8 threads per key)

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* __restrict__ q, int n_q, int n_kv, int hd,
                                                                  const int* __restrict__ pos0_dev, KvCache kv,
                                                                  float* __restrict__ out, ExpfTable et) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[2][kAttnThreads / 32];
  __shared__ float lane_sum[2][8];
  __shared__ float inv_s[2], max_s[2];
  cudaGridDependencySynchronize();
  const int m = blockIdx.x, kvh = blockIdx.y, pr = blockIdx.z;
  const int groups = n_q / n_kv;
  const int g0 = pr * 2;
  const int nh = (g0 + 1 < groups) ? 2 : 1;  // pair path or lone head
  const int qh0 = kvh * groups + g0;
  const int pos = *pos0_dev + m;
  const int kv_len = pos + 1;
  const int kvs = hd + 8;                    // padded smem row of a staged key
  float* qs = sm;                            // [2][hd]
  float* sc = qs + 2 * hd;                   // [2][max_seq]
  float* kt = sc + 2 * kv.max_seq;           // [kKeyTile][hd + 8]
  const int tid = threadIdx.x, lane = tid & 31;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const float* kc = kv.k + (size_t)kvh * kv.max_seq * hd;
  const float* vc = kv.v + (size_t)kvh * kv.max_seq * hd;

  for (int i = tid; i < nh * hd; i += blockDim.x) qs[i] = q[((size_t)m * n_q + qh0) * hd + i];
  const int kv4 = kv_len & ~3, kv8 = kv_len & ~7;
  float lmax[2] = {-1e30f, -1e30f};
  // ---- scores
  for (int t0 = 0; t0 < kv_len; t0 += kKeyTile) {
    const int nk = min(kKeyTile, kv_len - t0);
    __syncthreads();
    for (int i = tid; i < nk * hd; i += blockDim.x) {
      const int r = i / hd, c = i % hd;
      kt[r * kvs + c] = kc[(size_t)(t0 + r) * hd + c];
    }
    __syncthreads();
    const int key = tid >> 3, l = tid & 7;
    const int t = t0 + key;
    const bool valid = key < nk;
    const float* kp = kt + key * kvs;
    for (int h = 0; h < nh; h++) {
      const float* qv = qs + h * hd;
      // Shuffle trees run on all lanes (keys of one warp may sit on both sides of kv4).
      float acc = 0.0f;
      if (valid)
        for (int i = l; i < hd; i += 8) acc = __fmaf_rn(qv[i], kp[i], acc);
      const float t_pairs = tree8_pairs(acc);
      float t_split;
      if (nh == 2) {
        t_split = tree8_split(acc);
      } else {
        // lone head, tail key: dot_f32_avx2 (dpuf_engine.c:325-339)
        float a0 = 0.0f, a1 = 0.0f;
        if (valid) {
          int i = 0;
          for (; i + 15 < hd; i += 16) {
            a0 = __fmaf_rn(qv[i + l], kp[i + l], a0);
            a1 = __fmaf_rn(qv[i + 8 + l], kp[i + 8 + l], a1);
          }
          for (; i + 7 < hd; i += 8) a0 = __fmaf_rn(qv[i + l], kp[i + l], a0);
        }
        t_split = tree8_split(__fadd_rn(a0, a1));
      }
      float s = __fmul_rn((t < kv4) ? t_pairs : t_split, scale);
      if (valid && l == 0) {
        sc[h * kv.max_seq + t] = s;
        lmax[h] = max_ps(lmax[h], s);
      }
    }
  }
  // ---- max
  for (int h = 0; h < nh; h++) {
    float v = warp_max(lmax[h]);
    if (lane == 0) red[h][tid >> 5] = v;
  }
  __syncthreads();
  if (tid < nh) {
    float v = -1e30f;
    for (int w = 0; w < kAttnThreads / 32; w++) v = max_ps(v, red[tid][w]);
    max_s[tid] = v;
  }
  __syncthreads();
  // ---- exp over the 8-aligned part
  for (int h = 0; h < nh; h++) {
    const float mx = max_s[h];
    for (int k = tid; k < kv8; k += blockDim.x) sc[h * kv.max_seq + k] = exp_poly(__fsub_rn(sc[h * kv.max_seq + k], mx));
  }
  __syncthreads();
  // ---- lane sums (8 sequential chains per head); the <= 7 tail exponentials (glibc expf) are
  // independent, so eight more threads per head evaluate them meanwhile
  if (tid < 8 * nh) {
    const int h = tid >> 3, l = tid & 7;
    const float* s = sc + h * kv.max_seq;
    float acc = 0.0f;
    for (int k = l; k < kv8; k += 8) acc = __fadd_rn(acc, s[k]);
    lane_sum[h][l] = acc;
  } else if (tid >= 64 && tid < 64 + 8 * nh) {
    const int h = (tid - 64) >> 3, k = kv8 + ((tid - 64) & 7);
    if (k < kv_len) {
      float* s = sc + h * kv.max_seq;
      s[k] = glibc_expf(__fsub_rn(s[k], max_s[h]), et);
    }
  }
  __syncthreads();
  // split tree of the lane sums, then the tail added in order
  if (tid < nh) {
    const float* s = sc + tid * kv.max_seq;
    float sp = tree8_split_arr(lane_sum[tid]);
    for (int k = kv8; k < kv_len; k++) sp = __fadd_rn(sp, s[k]);
    inv_s[tid] = __fdiv_rn(1.0f, __fadd_rn(sp, 1e-12f));
  }
  __syncthreads();
  for (int h = 0; h < nh; h++) {
    const float inv = inv_s[h];
    for (int k = tid; k < kv_len; k += blockDim.x) sc[h * kv.max_seq + k] = __fmul_rn(sc[h * kv.max_seq + k], inv);
  }
  __syncthreads();
  // ---- PV
  for (int o = tid; o < nh * hd; o += blockDim.x) {
    const int h = o / hd, d = o % hd;
    const float* p = sc + h * kv.max_seq;
    float acc = 0.0f;
    if (nh == 2) {
      int k = 0;
      for (; k + 3 < kv_len; k += 4) {
        const float v0 = vc[(size_t)k * hd + d], v1 = vc[(size_t)(k + 1) * hd + d];
        const float v2 = vc[(size_t)(k + 2) * hd + d], v3 = vc[(size_t)(k + 3) * hd + d];
        acc = __fmaf_rn(p[k], v0, acc);
        acc = __fmaf_rn(p[k + 1], v1, acc);
        acc = __fmaf_rn(p[k + 2], v2, acc);
        acc = __fmaf_rn(p[k + 3], v3, acc);
      }
      for (; k < kv_len; k++) acc = __fmaf_rn(p[k], vc[(size_t)k * hd + d], acc);
    } else if ((hd & 63) == 0) {
      int k = 0;
      for (; k + 1 < kv_len; k += 2) {
        const float t1 = __fmaf_rn(p[k + 1], vc[(size_t)(k + 1) * hd + d], acc);
        acc = __fmaf_rn(p[k], vc[(size_t)k * hd + d], t1);
      }
      if (k < kv_len) acc = __fmaf_rn(p[k], vc[(size_t)k * hd + d], acc);
    } else {
      const int hd8 = hd & ~7;
      for (int k = 0; k < kv_len; k++) {
        const float pv = p[k], vv = vc[(size_t)k * hd + d];
        acc = (d < hd8) ? __fmaf_rn(pv, vv, acc) : __fadd_rn(acc, __fmul_rn(pv, vv));
      }
    }
    out[((size_t)m * n_q + qh0 + h) * hd + d] = acc;
  }
}

}  // namespace

cudaError_t configure_attn_kernels() {
  return set_max_dyn_smem(attention_kernel);
}

cudaError_t launch_attention(const Launch& L, const float* q, int M, int n_q, int n_kv, int hd, const int* pos0_dev,
                             KvCache kv, float* out, const ExpfTable& et) {
  const int groups = n_q / n_kv;
  const size_t smem = ((size_t)2 * hd + 2 * (size_t)kv.max_seq + (size_t)kKeyTile * (hd + 8)) * sizeof(float);
  if (smem > kMaxDynSmem) return cudaErrorInvalidValue;
  return launch_k(L, attention_kernel, dim3(M, n_kv, (groups + 1) / 2), dim3(kAttnThreads), smem, q, n_q, n_kv, hd,
                  pos0_dev, kv, out, et);
}

}  // namespace dpuf
