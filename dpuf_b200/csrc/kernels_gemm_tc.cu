// kernels_gemm_tc.cu - exact mode-12 GEMM for M > 1 (prefill) on the 5th-generation tensor
// cores (tcgen05, TMEM).
//
// Per (token t, row r) the reference computes (dpuf_matmul_qr_hadamard4_packed_tile_range,
// dpuf_avx2.c:2585-2676):
//   dot_b = sum_k u_{r,k} q_{t,k} - xm_{t,b}              exact integers (u = nibble 0..15)
//   acc   = fmaf((float)dot_b, ws_{r,b} * xs_{t,b}, acc)   blocks b ascending, xs <= 0 skipped
// The integer part is what a kind::i8 MMA computes exactly (u8 x s8 -> s32, |sum| < 2^17), one
// MMA per 32-column block so that every block's dot lands in its own TMEM columns; the fp32
// chain then runs on CUDA cores in the reference's order.
//
// CTA = 128 weight rows (8 container tiles of one job) x N tokens (8, 16 or 32).  Per stage of
// kStageBlocks blocks all 256 threads
//   1. unpack the tiles' nibbles to u8 in shared memory, K-major without swizzle (core
//      matrices of 8 rows x 16 bytes; the two 16-byte K halves LBO = 128 bytes apart, 8-row
//      groups SBO = 256 bytes apart) - A; copy the tokens' int8 codes the same way - B; the
//      rows' fp16 block scales and the tokens' block scales and sums;
//   2. thread 0 issues one tcgen05.mma per block (M=128, N, K=32) into TMEM columns
//      [j*N, j*N+N) and commits them to an mbarrier;
//   3. after the (bounded) wait, warp w reads TMEM lanes 32*(w%4).. (its rows), columns of its
//      half of the tokens (tcgen05.ld 32x32b) and runs the chains of its (row, token) pairs.
// Outputs are written after the last stage.  TMEM (256 columns) is allocated by warp 0 and
// freed before exit, also when a wait gives up (it then sets the error word).
#include <algorithm>

#include "kernels.cuh"

namespace dpuf {

namespace {

constexpr int kTcThreads = 256;
constexpr int kTcRows = 128;
constexpr int kStageBlocks = 8;
constexpr int kTmemCols = 256;  // kStageBlocks * 32 tokens at most
constexpr unsigned long long kTcWaitNs = 2000000000ull;

DPUF_DEV unsigned su32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

DPUF_DEV uint64_t smem_desc(const void* p, unsigned lbo, unsigned sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((su32(p) >> 4) & 0x3FFF);          // start address
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;         // leading (K) byte offset
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;         // stride (M/N) byte offset
  d |= (uint64_t)1 << 46;                             // descriptor version (sm100)
  return d;                                           // base offset 0, no swizzle
}

// kind::i8 instruction descriptor: D s32, A u8, B s8, both K-major, M = 128, N.
DPUF_HD uint32_t idesc_i8(int n) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

DPUF_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <int N>
DPUF_DEV void tmem_ld(uint32_t addr, uint32_t (&v)[N / 2]);
template <>
DPUF_DEV void tmem_ld<8>(uint32_t addr, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr));
}
template <>
DPUF_DEV void tmem_ld<16>(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr));
}
template <>
DPUF_DEV void tmem_ld<32>(uint32_t addr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr));
}

struct TcGroup {  // one CTA row group: 8 consecutive tiles of one job
  int job, t0;
};

struct TcArgs {
  LinJobs J;
  int M;            // tokens
  int n_groups;     // row groups over all jobs
  int group_prefix[kMaxJobs + 1];
  int* err;         // set to 1 when an MMA wait gives up
};

template <int N>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(TcArgs P) {
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t mma_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- this CTA's rows and tokens
  int jb = 0;
  while (jb + 1 < P.J.n && (int)blockIdx.x >= P.group_prefix[jb + 1]) jb++;
  const LinJob& job = P.J.j[jb];
  const int t_first = job.t_begin + ((int)blockIdx.x - P.group_prefix[jb]) * (kTcRows / kTileRows);
  const int n_tiles_here = min(kTcRows / kTileRows, job.t_end - t_first);
  const int tok0 = blockIdx.y * N;
  const int cols = job.w.cols, n_blk = cols >> 5;

  // ---- shared memory: A | B | ws | xs | xm per stage
  unsigned char* sA = sm;                                        // [kStageBlocks][128 x 32 B]
  unsigned char* sB = sA + kStageBlocks * kTcRows * 32;          // [kStageBlocks][N x 32 B]
  uint16_t* sW = (uint16_t*)(sB + kStageBlocks * N * 32);        // [128][kStageBlocks]
  float* sXs = (float*)(sW + kTcRows * kStageBlocks);            // [N][kStageBlocks]
  int* sXm = (int*)(sXs + N * kStageBlocks);                     // [N][kStageBlocks]

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_sh)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&mma_bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_sh = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;
  cudaGridDependencySynchronize();

  const Act& act = job.act;
  const int row = 32 * (warp & 3) + lane;  // TMEM lane = weight row of this thread's chains
  const int half = warp >> 2;              // which half of the N tokens
  constexpr int NH = N / 2;
  float acc[NH];
#pragma unroll
  for (int i = 0; i < NH; i++) acc[i] = 0.0f;
  const uint32_t idesc = idesc_i8(N);

  const int n_stages = (n_blk + kStageBlocks - 1) / kStageBlocks;
  for (int s = 0; s < n_stages; s++) {
    const int b0 = s * kStageBlocks, kb = min(kStageBlocks, n_blk - b0);
    // ---- 1. A: unpack nibble words (row, block, chunk) to 8 bytes each
    for (int i = tid; i < kTcRows * kStageBlocks * 4; i += kTcThreads) {
      const int c = i & 3, r = (i >> 2) & (kTcRows - 1), j = i >> 9;  // 4 chunks x 128 rows per block
      const int t = r >> 4, g = (r >> 3) & 1, ri = r & 7;
      uint2 v = make_uint2(0u, 0u);
      if (j < kb && t < n_tiles_here) {
        const int tt = t_first + t;
        const int n_r = min(kTileRows, job.w.rows - tt * kTileRows);
        if (g * 8 + ri < n_r) {
          const uint8_t* tp = job.w.tiles + job.w.toff[tt] + 16 + (size_t)g * n_blk * 144;
          const uint32_t w = *(const uint32_t*)(tp + (size_t)n_blk * 16 + (size_t)(b0 + j) * 128 + c * 32 + ri * 4);
          v = make_uint2(w & 0x0F0F0F0Fu, (w >> 4) & 0x0F0F0F0Fu);  // columns 8c..8c+3, 8c+4..8c+7
        }
      }
      *(uint2*)(sA + j * (kTcRows * 32) + (r >> 3) * 256 + (c >> 1) * 128 + (r & 7) * 16 + (c & 1) * 8) = v;
    }
    // ---- B: the tokens' codes, 16 bytes at a time
    for (int i = tid; i < N * kStageBlocks * 2; i += kTcThreads) {
      const int h = i & 1, n = (i >> 1) % N, j = (i >> 1) / N;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (j < kb && tok0 + n < P.M)
        v = *(const uint4*)(act.q8 + (size_t)(tok0 + n) * act.ld + (size_t)(b0 + j) * 32 + h * 16);
      *(uint4*)(sB + j * (N * 32) + (n >> 3) * 256 + h * 128 + (n & 7) * 16) = v;
    }
    // ---- row scales, token scales and sums
    for (int i = tid; i < kTcRows * kStageBlocks; i += kTcThreads) {
      const int r = i / kStageBlocks, j = i % kStageBlocks;
      const int t = r >> 4, g = (r >> 3) & 1, ri = r & 7;
      uint16_t w = 0;
      if (j < kb && t < n_tiles_here) {
        const int tt = t_first + t;
        const int n_r = min(kTileRows, job.w.rows - tt * kTileRows);
        if (g * 8 + ri < n_r)
          w = *(const uint16_t*)(job.w.tiles + job.w.toff[tt] + 16 + (size_t)g * n_blk * 144 + (size_t)(b0 + j) * 16 +
                                 ri * 2);
      }
      sW[r * kStageBlocks + j] = w;
    }
    for (int i = tid; i < N * kStageBlocks; i += kTcThreads) {
      const int n = i / kStageBlocks, j = i % kStageBlocks;
      float xs = 0.0f;
      int xm = 0;
      if (j < kb && tok0 + n < P.M) {
        xs = act.xs[(size_t)(tok0 + n) * (act.ld >> 5) + b0 + j];
        xm = act.xm[(size_t)(tok0 + n) * (act.ld >> 5) + b0 + j];
      }
      sXs[i] = xs;
      sXm[i] = xm;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
    __syncthreads();

    // ---- 2. one MMA per block, committed to the mbarrier
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int j = 0; j < kb; j++) {
        const uint64_t da = smem_desc(sA + j * (kTcRows * 32), 128, 256);
        const uint64_t db = smem_desc(sB + j * (N * 32), 128, 256);
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem + j * N),
            "l"(da), "l"(db), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
            : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(&mma_bar))
                   : "memory");
    }
    // ---- 3. wait for the MMAs (bounded), then the chains
    if (lane == 0) {
      const unsigned par = (unsigned)(s & 1);
      const unsigned long long t0 = gtimer();
      for (;;) {
        unsigned ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(su32(&mma_bar)), "r"(par), "r"(20000u)
            : "memory");
        if (ok) break;
        if (abort_sh || gtimer() - t0 > kTcWaitNs) {
          abort_sh = 1;
          atomicCAS(P.err, 0, 1);
          break;
        }
      }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!abort_sh) {
      const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
      for (int j = 0; j < kb; j++) {
        uint32_t d[NH];
        tmem_ld<N>(tmem + lane_base + j * N + half * NH, d);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const float ws = f16bits_to_f32(sW[row * kStageBlocks + j]);
#pragma unroll
        for (int i = 0; i < NH; i++) {
          const int n = half * NH + i;
          const float xs = sXs[n * kStageBlocks + j];
          const float p = (float)((int)d[i] - sXm[n * kStageBlocks + j]);
          const float sc = __fmul_rn(ws, xs);
          acc[i] = xs > 0.0f ? __fmaf_rn(p, sc, acc[i]) : acc[i];
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // A, B and the TMEM columns are reused by the next stage
  }

  // ---- outputs
  const int t = row >> 4;
  if (t < n_tiles_here) {
    const int r_global = (t_first + t) * kTileRows + (row & 15);
    if (r_global < job.w.rows)
#pragma unroll
      for (int i = 0; i < NH; i++) {
        const int n = tok0 + half * NH + i;
        if (n < P.M) job.out[(size_t)n * job.ldo + r_global] = acc[i];
      }
  }
  cudaTriggerProgrammaticLaunchCompletion();
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

template <int N>
size_t tc_smem_bytes() {
  return (size_t)kStageBlocks * kTcRows * 32 + (size_t)kStageBlocks * N * 32 + (size_t)kTcRows * kStageBlocks * 2 +
         (size_t)N * kStageBlocks * 8;
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

// At least 96 KB of shared memory per CTA, so that at most two CTAs (2 x 256 TMEM columns)
// share an SM and an allocation never waits on a third.
constexpr size_t kTcMinSmem = 96 * 1024;

}  // namespace

cudaError_t configure_gemm_tc_kernels() {
  cudaError_t e;
  if ((e = set_max_dyn_smem(gemm_tc_kernel<8>)) != cudaSuccess) return e;
  if ((e = set_max_dyn_smem(gemm_tc_kernel<16>)) != cudaSuccess) return e;
  return set_max_dyn_smem(gemm_tc_kernel<32>);
}

cudaError_t launch_gemm_tc(const Launch& L, const LinJobs& jobs, int M, int* err) {
  TcArgs P = {};
  P.J = jobs;
  P.M = M;
  P.err = err;
  P.group_prefix[0] = 0;
  for (int i = 0; i < jobs.n; i++) {
    if (jobs.j[i].w.cols != jobs.j[0].w.cols) return cudaErrorInvalidValue;
    const int tiles = jobs.j[i].t_end - jobs.j[i].t_begin;
    P.group_prefix[i + 1] = P.group_prefix[i] + (tiles + 7) / 8;
  }
  P.n_groups = P.group_prefix[jobs.n];
  if (P.n_groups == 0 || M <= 0) return cudaSuccess;
  // token tile: the largest of 32 / 16 / 8 that still gives >= 148 CTAs (or 8)
  int N = 32;
  while (N > 8 && (long long)P.n_groups * ((M + N - 1) / N) < 148) N >>= 1;
  const dim3 grid((unsigned)P.n_groups, (unsigned)((M + N - 1) / N));
  if (N == 32)
    return launch_k(L, gemm_tc_kernel<32>, grid, dim3(kTcThreads), std::max(tc_smem_bytes<32>(), kTcMinSmem), P);
  if (N == 16)
    return launch_k(L, gemm_tc_kernel<16>, grid, dim3(kTcThreads), std::max(tc_smem_bytes<16>(), kTcMinSmem), P);
  return launch_k(L, gemm_tc_kernel<8>, grid, dim3(kTcThreads), std::max(tc_smem_bytes<8>(), kTcMinSmem), P);
}

}  // namespace dpuf
