// kernels_lmhead.cu - Zone-A early-exit test and masking, greedy argmax.
//
// Zone A (dpuf_engine.c:2091-2139): after the LM-head rows of tiles [0, Z) are computed,
// the reference scans logits[0, min(16Z, V)) sequentially keeping the top two values with
// strict '>' (a repeated maximum counts for the second place) and exits when
// margin > 0 && b1 - b2 >= margin; on exit logits[16Z, V) = -1e9, otherwise the remaining
// tiles are computed.  The sequential top-2 equals a tree merge of partial (b1, b2) pairs
// (b1 = max, b2 = max(min(b1a, b1b), b2a, b2b)), which is what the kernel reduces.
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

DPUF_DEV void top2_push(float v, float& b1, float& b2) {
  if (v > b1) { b2 = b1; b1 = v; }
  else if (v > b2) { b2 = v; }
}
DPUF_DEV void top2_merge(float& b1, float& b2, float o1, float o2) {
  const float lo = fminf(b1, o1);
  b1 = fmaxf(b1, o1);
  b2 = fmaxf(fmaxf(b2, o2), lo);
}

__global__ void __launch_bounds__(1024) zone_test_kernel(const float* __restrict__ logits, int n, float margin,
                                                         int* __restrict__ flag, float* __restrict__ b12) {
  __shared__ float s1[32], s2[32];
  cudaGridDependencySynchronize();
  float b1 = -1e30f, b2 = -1e30f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) top2_push(logits[i], b1, b2);
  for (int m = 16; m; m >>= 1) {
    const float o1 = __shfl_xor_sync(kFull, b1, m), o2 = __shfl_xor_sync(kFull, b2, m);
    top2_merge(b1, b2, o1, o2);
  }
  if ((threadIdx.x & 31) == 0) { s1[threadIdx.x >> 5] = b1; s2[threadIdx.x >> 5] = b2; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    b1 = threadIdx.x < nw ? s1[threadIdx.x] : -1e30f;
    b2 = threadIdx.x < nw ? s2[threadIdx.x] : -1e30f;
    for (int m = 16; m; m >>= 1) {
      const float o1 = __shfl_xor_sync(kFull, b1, m), o2 = __shfl_xor_sync(kFull, b2, m);
      top2_merge(b1, b2, o1, o2);
    }
    if (threadIdx.x == 0) {
      *flag = (margin > 0.0f && __fsub_rn(b1, b2) >= margin) ? 1 : 0;
      if (b12) { b12[0] = b1; b12[1] = b2; }
    }
  }
}

__global__ void zone_mask_kernel(float* __restrict__ logits, int from, int V, const int* __restrict__ flag) {
  cudaGridDependencySynchronize();
  if (!*flag) return;
  for (int i = from + blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) logits[i] = -1e9f;
}

// First index of the maximum (strict '>' scan, dpuf-cli.c:1997-2005), over kArgmaxBlocks CTAs:
// CTA c reduces the slice [c*V/n, (c+1)*V/n) to (value, index) with ties keeping the lower
// index, writes it to part[c], and the last CTA to finish (counted by an atomic, no waiting)
// reduces the partials in slice order - the same first-maximal index as a sequential scan.
// With `greedy`, the winner becomes the next decode step's token: ids[0] = winner, the
// position advances and the id is appended to the history (back-to-back decode steps).
DPUF_DEV void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

DPUF_DEV void block_argmax(float& bv, int& bi, float* sv, int* si) {
  for (int m = 16; m; m >>= 1) {
    const float ov = __shfl_xor_sync(kFull, bv, m);
    const int oi = __shfl_xor_sync(kFull, bi, m);
    better(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    bv = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
    for (int m = 16; m; m >>= 1) {
      const float ov = __shfl_xor_sync(kFull, bv, m);
      const int oi = __shfl_xor_sync(kFull, bi, m);
      better(bv, bi, ov, oi);
    }
  }
}

__global__ void __launch_bounds__(256) argmax_blocks_kernel(const float* __restrict__ logits, int V, float2* part,
                                                            unsigned* counter, int32_t* out, bool greedy,
                                                            int32_t* ids, int32_t* pos0, int32_t* hist,
                                                            int32_t* step) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ bool last;
  cudaGridDependencySynchronize();
  const int c = blockIdx.x, nb = gridDim.x;
  const int i0 = (int)((long long)V * c / nb), i1 = (int)((long long)V * (c + 1) / nb);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) better(bv, bi, logits[i], i);
  block_argmax(bv, bi, sv, si);
  if (threadIdx.x == 0) {
    part[c] = make_float2(bv, __int_as_float(bi));
    __threadfence();
    last = atomicAdd(counter, 1u) == (unsigned)(nb - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int k = threadIdx.x; k < nb; k += blockDim.x) {
    const float2 p = __ldcg(part + k);
    better(bv, bi, p.x, __float_as_int(p.y));
  }
  __syncthreads();
  block_argmax(bv, bi, sv, si);
  if (threadIdx.x == 0) {
    const int id = (bi == 0x7fffffff) ? 0 : bi;
    *counter = 0u;
    if (greedy) {
      ids[0] = id;
      hist[*step] = id;
      *step += 1;
      *pos0 += 1;
    } else {
      *out = id;
    }
  }
}

// First-index argmax of each of M rows of logits (one CTA per row): the greedy id of every
// sequence of a batched decode step.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float* __restrict__ logits, int V,
                                                          int32_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  cudaGridDependencySynchronize();
  const float* row = logits + (size_t)blockIdx.x * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) better(bv, bi, row[i], i);
  block_argmax(bv, bi, sv, si);
  if (threadIdx.x == 0) out[blockIdx.x] = (bi == 0x7fffffff) ? 0 : bi;
}

}  // namespace

cudaError_t launch_argmax_rows(const Launch& L, const float* logits, int V, int M, int32_t* out) {
  return launch_k(L, argmax_rows_kernel, dim3(M), dim3(256), 0, logits, V, out);
}

cudaError_t launch_greedy_advance(const Launch& L, const float* logits, int V, float2* part, unsigned* counter,
                                  int32_t* ids, int32_t* pos0, int32_t* hist, int32_t* step) {
  return launch_k(L, argmax_blocks_kernel, dim3(kArgmaxBlocks), dim3(256), 0, logits, V, part, counter,
                  (int32_t*)nullptr, true, ids, pos0, hist, step);
}

cudaError_t launch_zone_test(const Launch& L, const float* logits, int n, float margin, int* flag, float* b12) {
  return launch_k(L, zone_test_kernel, dim3(1), dim3(1024), 0, logits, n, margin, flag, b12);
}

cudaError_t launch_zone_mask(const Launch& L, float* logits, int from, int V, const int* flag) {
  if (from >= V) return cudaSuccess;
  return launch_k(L, zone_mask_kernel, dim3(min(148, (V - from + 255) / 256)), dim3(256), 0, logits, from, V, flag);
}

cudaError_t launch_argmax(const Launch& L, const float* logits, int V, float2* part, unsigned* counter, int32_t* out) {
  return launch_k(L, argmax_blocks_kernel, dim3(kArgmaxBlocks), dim3(256), 0, logits, V, part, counter, out, false,
                  (int32_t*)nullptr, (int32_t*)nullptr, (int32_t*)nullptr, (int32_t*)nullptr);
}

}  // namespace dpuf
