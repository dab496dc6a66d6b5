// kernels_mode12.cu - mode-12 ("Hadamard-4bit packed") activation prep, embedding lookup,
// and exact prefill GEMM on CUDA cores (the decode GEMV is in kernels_gemv.cu).
//
// Arithmetic per (token, row), identical to dpuf_matmul_qr_hadamard4_packed_tile_range
// (dpuf_avx2.c:2585-2676):
//   dot_b = sum_k u_k * q_k - xm_b          (exact integer; u = stored nibble 0..15)
//   acc   = fmaf((float)dot_b, ws_b * xs_b, acc)   for blocks b ascending, xs_b <= 0 skipped
// The integer dot uses dp4a on nibbles widened to bytes (u < 16 fits a signed byte).
#include "kernels.cuh"
#include "layer_dev.cuh"

namespace dpuf {

namespace {

DPUF_DEV int dot_nibbles(uint32_t w, int x_lo, int x_hi, int acc) {
  acc = __dp4a((int)(w & 0x0F0F0F0Fu), x_lo, acc);
  acc = __dp4a((int)((w >> 4) & 0x0F0F0F0Fu), x_hi, acc);
  return acc;
}

DPUF_DEV const uint8_t* tile_ptr(const W12& w, int t) { return w.tiles + w.toff[t]; }
DPUF_DEV int tile_nrows(const uint8_t* tp) { return (int)(tp[4] | (tp[5] << 8)); }

DPUF_DEV int find_job(const LinJobs& J, int g, int& t) {
  int j = 0;
  while (j + 1 < J.n && g >= J.tile_prefix[j + 1]) j++;
  t = J.j[j].t_begin + (g - J.tile_prefix[j]);
  return j;
}

// ------------------------------------------------------------------ prep
__global__ void prep_kernel(const float* __restrict__ x, int ldx, int cols, const uint8_t* __restrict__ signs,
                            Act out) {
  cudaGridDependencySynchronize();
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int m = blockIdx.y;
  if (chunk * 64 >= cols) return;
  const int c0 = chunk * 64;
  const float* xr = x + (size_t)m * ldx;
  prep_chunk_warp(xr[c0 + lane], xr[c0 + 32 + lane], signs, c0, lane, out.q8 + (size_t)m * out.ld,
                  out.xs + (size_t)m * (out.ld >> 5), out.xm + (size_t)m * (out.ld >> 5));
}

// ------------------------------------------------------------------ embedding
// Row r of the embedding: (u - 8) * ws per column, FWHT-64, then the column sign
// (dpuf_embed_qr_hadamard4_packed_f32, dpuf_avx2.c:2738-2783).  One warp per 64-column chunk.
__global__ void embed_kernel(W12 w, const int32_t* __restrict__ ids, float* __restrict__ out) {
  cudaGridDependencySynchronize();
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int m = blockIdx.y;
  const int cols = w.cols, n_blk = cols >> 5;
  if (chunk * 64 >= cols) return;
  const int r = ids[m];
  const int c0 = chunk * 64;
  float oa, ob;
  embed_chunk_warp(tile_ptr(w, r / kTileRows), n_blk, r % kTileRows, w.signs, c0, lane, oa, ob);
  float* o = out + (size_t)m * cols;
  o[c0 + lane] = oa;
  o[c0 + 32 + lane] = ob;
}

// ------------------------------------------------------------------ exact prefill GEMM (M > 1)
// CTA = (16-row tile, 16-token tile).  Blocks are processed in chunks of 32: phase 1 computes
// the exact dots for every (token, row, block) of the chunk into shared memory, phase 2 runs
// the per-(token,row) fp32 chains over the chunk's blocks in order (acc stays in registers).
constexpr int kGemmMT = 16;
constexpr int kGemmBC = 16;

__global__ void __launch_bounds__(256) gemm_exact_kernel(LinJobs J, int M) {
  __shared__ __align__(16) int8_t xq[kGemmMT][kGemmBC * 32];
  __shared__ float xs[kGemmMT][kGemmBC];
  __shared__ int xm[kGemmMT][kGemmBC];
  __shared__ int D[kGemmMT][kTileRows][kGemmBC + 1];
  __shared__ uint16_t sc[kTileRows][kGemmBC];
  int t;
  const int j = find_job(J, blockIdx.y, t);
  const LinJob& job = J.j[j];
  const int cols = job.w.cols, n_blk = cols >> 5;
  const uint8_t* tp = tile_ptr(job.w, t);
  const int m0 = blockIdx.x * kGemmMT;
  const int mt = min(kGemmMT, M - m0);
  cudaGridDependencySynchronize();
  const int n_r = tile_nrows(tp);
  const int n_8g = (n_r + 7) >> 3;
  const int ldq = job.act.ld, lds = job.act.ld >> 5;
  const int my_m = threadIdx.x >> 4, my_row = threadIdx.x & 15;
  float acc = 0.0f;
  for (int b0 = 0; b0 < n_blk; b0 += kGemmBC) {
    const int bc = min(kGemmBC, n_blk - b0);
    __syncthreads();
    for (int i = threadIdx.x; i < mt * bc * 2; i += blockDim.x) {  // 16-byte pieces
      const int m = i / (bc * 2), p = i % (bc * 2);
      ((int4*)&xq[m][0])[p] = ((const int4*)(job.act.q8 + (size_t)(m0 + m) * ldq + (size_t)b0 * 32))[p];
    }
    for (int i = threadIdx.x; i < mt * bc; i += blockDim.x) {
      const int m = i / bc, b = i % bc;
      xs[m][b] = job.act.xs[(size_t)(m0 + m) * lds + b0 + b];
      xm[m][b] = job.act.xm[(size_t)(m0 + m) * lds + b0 + b];
    }
    for (int i = threadIdx.x; i < n_8g * 8 * bc; i += blockDim.x) {
      const int row = i / bc, b = i % bc;
      sc[row][b] = *(const uint16_t*)(tp + 16 + (size_t)(row >> 3) * n_blk * 144 + (size_t)(b0 + b) * 16 + (row & 7) * 2);
    }
    __syncthreads();
    for (int it = threadIdx.x; it < n_8g * 8 * bc; it += blockDim.x) {
      const int ri = it & 7, rg = (it >> 3) % n_8g, b = it / (8 * n_8g);
      const uint8_t* qb = tp + 16 + (size_t)rg * n_blk * 144 + (size_t)n_blk * 16 + (size_t)(b0 + b) * 128 + ri * 4;
      uint32_t w[4];
#pragma unroll
      for (int c = 0; c < 4; c++) w[c] = *(const uint32_t*)(qb + c * 32);
      for (int m = 0; m < mt; m++) {
        const int* xw = (const int*)&xq[m][b * 32];
        int d = -xm[m][b];
#pragma unroll
        for (int c = 0; c < 4; c++) d = dot_nibbles(w[c], xw[2 * c], xw[2 * c + 1], d);
        D[m][rg * 8 + ri][b] = d;
      }
    }
    __syncthreads();
    if (my_m < mt && my_row < n_r) {
      for (int b = 0; b < bc; b++) {
        const float bs = xs[my_m][b];
        if (bs <= 0.0f) continue;
        const float s = __fmul_rn(f16bits_to_f32(sc[my_row][b]), bs);
        acc = __fmaf_rn((float)D[my_m][my_row][b], s, acc);
      }
    }
  }
  if (my_m < mt && my_row < n_r) job.out[(size_t)(m0 + my_m) * job.ldo + (size_t)t * kTileRows + my_row] = acc;
}

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

}  // namespace

cudaError_t configure_gemv_kernels();
cudaError_t configure_mode12_kernels() { return configure_gemv_kernels(); }

cudaError_t launch_prep(const Launch& L, const float* x, int ldx, int M, int cols, const uint8_t* signs, Act out) {
  const int chunks = cols / 64, wpb = 8;
  return launch_k(L, prep_kernel, dim3((chunks + wpb - 1) / wpb, M), dim3(wpb * 32), 0, x, ldx, cols, signs, out);
}

cudaError_t launch_embed(const Launch& L, const W12& w, const int32_t* ids, int M, float* out) {
  const int chunks = w.cols / 64, wpb = 8;
  return launch_k(L, embed_kernel, dim3((chunks + wpb - 1) / wpb, M), dim3(wpb * 32), 0, w, ids, out);
}

cudaError_t launch_gemm_exact(const Launch& L, const LinJobs& jobs, int M) {
  return launch_k(L, gemm_exact_kernel, dim3((M + kGemmMT - 1) / kGemmMT, jobs.tile_prefix[jobs.n]), dim3(256), 0,
                  jobs, M);
}

}  // namespace dpuf
