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
// CTA = 128 weight rows (8 container tiles of one job) x N tokens (8, 16 or 32); a stage is
// kStageBlocks blocks.  Warp-specialised pipeline, every hand-off on mbarriers (no CTA barrier
// per stage):
//   warp 12      TMA: the raw bytes of each stage (nibbles and fp16 scales of 16 (tile, group)
//                pairs) by bulk copies into a 3-deep raw ring;
//   warps 0..3   unpack: the nibbles to u8 in shared memory, K-major without swizzle (core
//                matrices of 8 rows x 16 bytes; the two 16-byte K halves LBO = 128 bytes apart,
//                8-row groups SBO = 256 bytes apart) - A - and the row scales, into a 3-deep
//                stage ring; they copy the tokens' int8 codes the same way (B) and the tokens'
//                block scales and sums one stage ahead with cp.async;
//   warp 13      MMA: one tcgen05.mma per block (M=128, N, K=32) into TMEM columns [j*N, j*N+N)
//                of a 2-deep TMEM ring, committed to an mbarrier;
//   warps 4..11  chains: warp w reads TMEM lanes 32*(w%4).. (its rows), columns of its half of
//                the tokens (tcgen05.ld 32x32b, four blocks at a time) and runs the chains of
//                its (row, token) pairs; outputs after the last stage.
// TMEM (2 x 8 x N columns) is allocated by warp 12 and freed before exit.  Every wait is
// bounded: one that gives up sets the error word and the CTA's abort flag, after which every
// role stops waiting; bulk copies still in flight are waited for (bounded) before exit.
#include <algorithm>

#include "kernels.cuh"

namespace dpuf {

namespace {

constexpr int kUnpackWarps = 4;   // warps 0..3
constexpr int kChainWarps = 8;    // warps 4..11
constexpr int kChainWarp0 = kUnpackWarps;
constexpr int kTmaWarp = kUnpackWarps + kChainWarps;  // 12
constexpr int kMmaWarp = kTmaWarp + 1;                // 13
constexpr int kTcThreads = (kMmaWarp + 1) * 32;       // 448
constexpr int kUnpackThreads = kUnpackWarps * 32;
constexpr int kRawRing = 3, kStageRing = 3, kTmemRing = 2;
constexpr int kTcRows = 128;
constexpr int kStageBlocks = 8;
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

template <>
DPUF_DEV void tmem_ld<64>(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
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

DPUF_DEV bool try_parity(uint64_t* bar, unsigned par) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(su32(bar)), "r"(par)
               : "memory");
  return ok != 0;
}

// Bounded wait for a phase.  The global timer is slow to read (hundreds of cycles), so it is read
// only once the first try has failed, and then every 16 tries.
DPUF_DEV bool wait_parity(uint64_t* bar, unsigned par, volatile int* abort_flag, int* err) {
  if (try_parity(bar, par)) return true;
  const unsigned long long t0 = gtimer();
  for (int it = 1;; it++) {
    if (try_parity(bar, par)) return true;
    if ((it & 15) == 0 && (*abort_flag || gtimer() - t0 > kTcWaitNs)) {
      *abort_flag = 1;
      atomicCAS(err, 0, 1);
      return false;
    }
  }
}

DPUF_DEV void cp16_zfill(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
DPUF_DEV void cp4_zfill(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}

// Raw stage bytes of one (tile, group): nibbles of kStageBlocks blocks, then their scales.
constexpr int kRawTG = kStageBlocks * 128 + kStageBlocks * 16;
constexpr int kRawBytes = (kTcRows / 8) * kRawTG;  // 16 (tile, group) pairs

template <int N>
struct TcLayout {  // shared memory of one CTA
  static constexpr int kA = kStageBlocks * kTcRows * 32;  // A of a stage
  static constexpr int kB = kStageBlocks * N * 32;        // B of a stage
  static constexpr int kW = kTcRows * kStageBlocks * 2;   // row scales of a stage
  static constexpr int kX = kStageBlocks * N * 4;         // xs or xm of a stage
  static constexpr int raw = 0;                            // [kRawRing][kRawBytes]
  static constexpr int a = raw + kRawRing * kRawBytes;    // [kStageRing][kA]
  static constexpr int b = a + kStageRing * kA;            // [kStageRing][kB]
  static constexpr int w = b + kStageRing * kB;            // [kStageRing][kW]
  static constexpr int xs = w + kStageRing * kW;           // [kStageRing][kX]
  static constexpr int xm = xs + kStageRing * kX;          // [kStageRing][kX]
  static constexpr int bytes = xm + kStageRing * kX;
  static constexpr int tmem_cols = kTmemRing * kStageBlocks * N < 32 ? 32 : kTmemRing * kStageBlocks * N;
};
static_assert(TcLayout<32>::bytes <= 200 * 1024, "shared memory of the 32-token CTA");

template <int N>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(TcArgs P) {
  using Lay = TcLayout<N>;
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t raw_full[kRawRing], raw_empty[kRawRing];
  __shared__ __align__(8) uint64_t stg_full[kStageRing], stg_empty[kStageRing];
  __shared__ __align__(8) uint64_t d_full[kTmemRing], d_empty[kTmemRing];
  __shared__ const uint8_t* grp_base[kTcRows / 8];  // group data of each (tile, group), or null
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- this CTA's rows and tokens
  int jb = 0;
  while (jb + 1 < P.J.n && (int)blockIdx.x >= P.group_prefix[jb + 1]) jb++;
  const LinJob& job = P.J.j[jb];
  const int t_first = job.t_begin + ((int)blockIdx.x - P.group_prefix[jb]) * (kTcRows / kTileRows);
  const int n_tiles_here = min(kTcRows / kTileRows, job.t_end - t_first);
  const int tok0 = blockIdx.y * N;
  const int cols = job.w.cols, n_blk = cols >> 5;
  const int n_stages = (n_blk + kStageBlocks - 1) / kStageBlocks;

  if (warp == kTmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_sh)),
                 "r"(Lay::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid < kTcRows / 8) {  // (tile, group) bases; null where the group has no rows
    const int t = tid >> 1, g = tid & 1;
    const uint8_t* p = nullptr;
    if (t < n_tiles_here) {
      const int tt = t_first + t;
      if (g * 8 < min(kTileRows, job.w.rows - tt * kTileRows))
        p = job.w.tiles + job.w.toff[tt] + 16 + (size_t)g * n_blk * 144;
    }
    grp_base[tid] = p;
  }
  if (tid == 0) {
    for (int i = 0; i < kRawRing; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&raw_full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&raw_empty[i])), "r"(kUnpackWarps) : "memory");
    }
    for (int i = 0; i < kStageRing; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&stg_full[i])), "r"(kUnpackWarps) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&stg_empty[i])), "r"(kChainWarps) : "memory");
    }
    for (int i = 0; i < kTmemRing; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&d_full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&d_empty[i])), "r"(kChainWarps) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_sh = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;
  auto arrive = [](uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
  };
  // one lane waits for the warp, which then follows its verdict
  auto warp_wait = [&](uint64_t* bar, unsigned par) {
    bool ok = true;
    if (lane == 0) ok = wait_parity(bar, par, &abort_sh, P.err);
    return __shfl_sync(kFull, (int)ok, 0) != 0;
  };

  if (warp == kTmaWarp) {
    // ================================================================ TMA: raw ring
    int issued = 0;
    for (int s = 0; s < n_stages; s++) {
      const int slot = s % kRawRing, k = s / kRawRing;
      if (!warp_wait(&raw_empty[slot], (unsigned)((k & 1) ^ 1))) break;
      const int b0 = s * kStageBlocks, kb = min(kStageBlocks, n_blk - b0);
      unsigned bytes = 0;
      for (int tg = 0; tg < kTcRows / 8; tg++)
        if (grp_base[tg]) bytes += (unsigned)kb * 144;
      if (lane == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&raw_full[slot])), "r"(bytes)
                     : "memory");
      __syncwarp();
      const int tg = lane >> 1, part = lane & 1;
      const uint8_t* gb = grp_base[tg];
      if (gb) {
        unsigned char* dst = sm + Lay::raw + slot * kRawBytes + tg * kRawTG + (part ? kStageBlocks * 128 : 0);
        const uint8_t* src = part ? gb + (size_t)b0 * 16 : gb + (size_t)n_blk * 16 + (size_t)b0 * 128;
        const unsigned n = (unsigned)kb * (part ? 16 : 128);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
            "l"(src), "r"(n), "r"(su32(&raw_full[slot]))
            : "memory");
      }
      issued = s + 1;
    }
    // copies in flight must land before the CTA exits (after an abort nobody else waits)
    if (abort_sh && lane == 0) {
      const unsigned long long t0 = gtimer();
      for (int q = max(0, issued - kRawRing); q < issued; q++) {
        unsigned ok = 0;
        while (!ok && gtimer() - t0 < kTcWaitNs)
          asm volatile(
              "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
              : "=r"(ok)
              : "r"(su32(&raw_full[q % kRawRing])), "r"((unsigned)((q / kRawRing) & 1))
              : "memory");
      }
    }
  } else if (warp < kUnpackWarps) {
    // ================================================================ unpack warps
    const Act& act = job.act;
    const int xld = act.ld >> 5;
    // the tokens' codes, block scales and block sums of stage s into stage buffer s % ring (one
    // cp.async group of this thread)
    auto request_act = [&](int s) {
      const int p = s % kStageRing, b0 = s * kStageBlocks, kb = min(kStageBlocks, n_blk - b0);
      unsigned char* sB = sm + Lay::b + p * Lay::kB;
      float* sXs = (float*)(sm + Lay::xs + p * Lay::kX);
      int* sXm = (int*)(sm + Lay::xm + p * Lay::kX);
      for (int i = tid; i < N * kStageBlocks * 2; i += kUnpackThreads) {
        const int h = i & 1, n = (i >> 1) % N, j = (i >> 1) / N;
        const bool ok = j < kb && tok0 + n < P.M;
        const int8_t* src = ok ? act.q8 + (size_t)(tok0 + n) * act.ld + (size_t)(b0 + j) * 32 + h * 16 : act.q8;
        cp16_zfill(sB + j * (N * 32) + (n >> 3) * 256 + h * 128 + (n & 7) * 16, src, ok);
      }
      for (int i = tid; i < N * kStageBlocks; i += kUnpackThreads) {
        const int j = i / N, n = i % N;
        const bool ok = j < kb && tok0 + n < P.M;
        const size_t o = ok ? (size_t)(tok0 + n) * xld + b0 + j : 0;
        cp4_zfill(sXs + i, act.xs + o, ok);
        cp4_zfill(sXm + i, act.xm + o, ok);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    unsigned valid_tg = 0u;  // (tile, group) pairs with rows
    for (int tg = 0; tg < kTcRows / 8; tg++)
      if (grp_base[tg]) valid_tg |= 1u << tg;
    cudaGridDependencySynchronize();  // the activations come from the previous kernel
    bool ok = warp_wait(&stg_empty[0], 1u);
    if (ok) request_act(0);
    for (int s = 0; ok && s < n_stages; s++) {
      const int p = s % kStageRing, pk = s / kStageRing, rs = s % kRawRing, rk = s / kRawRing;
      // the next stage's activations first (their buffer was freed by the chains of stage s-2)
      bool next = s + 1 < n_stages;
      if (next) {
        const int q = (s + 1) % kStageRing, qk = (s + 1) / kStageRing;
        if (!warp_wait(&stg_empty[q], (unsigned)((qk & 1) ^ 1))) break;
        request_act(s + 1);
      }
      if (!warp_wait(&raw_full[rs], (unsigned)(rk & 1))) break;
      const int kb = min(kStageBlocks, n_blk - s * kStageBlocks);
      const unsigned char* rb = sm + Lay::raw + rs * kRawBytes;
      unsigned char* sA = sm + Lay::a + p * Lay::kA;
      // a warp unpacks one (tile group, block) at a time: lane L takes chunk c and row ri with
      // (c >> 1, ri, c & 1) = (L >> 4, (L >> 1) & 7, L & 1), so it reads raw word c * 32 + ri * 4
      // and writes its 8 u8 (columns 8c..8c+7 of row ri) at byte 8L of the block's 8-row core
      // matrices: every warp load and store covers distinct banks
      {
        const int c = ((lane >> 4) << 1) | (lane & 1), ri = (lane >> 1) & 7;
        const int src_off = c * 32 + ri * 4, dst_off = lane * 8;
        constexpr int kPer = (kTcRows / 8) * kStageBlocks / kUnpackWarps;  // blocks per warp and stage
        constexpr int kBatch = 16;                                         // loads in flight
        static_assert(kStageBlocks == 8 && kPer % kBatch == 0, "unpack batches");
#pragma unroll 1
        for (int k0 = 0; k0 < kPer; k0 += kBatch) {
          uint32_t w[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; u++) {
            const int blk = warp + kUnpackWarps * (k0 + u), tg = blk >> 3, j = blk & 7;
            w[u] = (j < kb && ((valid_tg >> tg) & 1u)) ? *(const uint32_t*)(rb + tg * kRawTG + j * 128 + src_off) : 0u;
          }
#pragma unroll
          for (int u = 0; u < kBatch; u++) {
            const int blk = warp + kUnpackWarps * (k0 + u), tg = blk >> 3, j = blk & 7;
            *(uint2*)(sA + j * (kTcRows * 32) + tg * 256 + dst_off) =
                make_uint2(w[u] & 0x0F0F0F0Fu, (w[u] >> 4) & 0x0F0F0F0Fu);
          }
        }
      }
      uint16_t* sW = (uint16_t*)(sm + Lay::w + p * Lay::kW);
      for (int i = tid; i < kTcRows * kStageBlocks; i += kUnpackThreads) {  // [row][block]
        const int r = i >> 3, j = i & 7;
        sW[i] = (j < kb && grp_base[r >> 3])
                    ? *(const uint16_t*)(rb + (r >> 3) * kRawTG + kStageBlocks * 128 + j * 16 + (r & 7) * 2)
                    : (uint16_t)0;
      }
      // this stage's activations landed (the next stage's may still be in flight)
      if (next)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      else
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
      __syncwarp();
      if (lane == 0) {
        arrive(&raw_empty[rs]);
        arrive(&stg_full[p]);
      }
      (void)pk;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // nothing of ours in flight at exit
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issuer
    const uint32_t idesc = idesc_i8(N);
    for (int s = 0; s < n_stages; s++) {
      const int p = s % kStageRing, pk = s / kStageRing, ds = s % kTmemRing, dk = s / kTmemRing;
      if (!warp_wait(&stg_full[p], (unsigned)(pk & 1))) break;
      if (!warp_wait(&d_empty[ds], (unsigned)((dk & 1) ^ 1))) break;
      if (lane == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int kb = min(kStageBlocks, n_blk - s * kStageBlocks);
        const unsigned char* sA = sm + Lay::a + p * Lay::kA;
        const unsigned char* sB = sm + Lay::b + p * Lay::kB;
        const uint64_t da0 = smem_desc(sA, 128, 256), db0 = smem_desc(sB, 128, 256);
        for (int j = 0; j < kb; j++) {
          // the start-address field (bits 0..13, 16-byte units) advances by one block's bytes
          const uint64_t da = da0 + (uint64_t)(j * (kTcRows * 32 / 16));
          const uint64_t db = db0 + (uint64_t)(j * (N * 32 / 16));
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
                  tmem + ds * (kStageBlocks * N) + j * N),
              "l"(da), "l"(db), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         su32(&d_full[ds]))
                     : "memory");
      }
      __syncwarp();
    }
  } else {
    // ================================================================ chain warps
    const int cw = warp - kChainWarp0;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane = weight row of this thread's chains
    const int half = cw >> 2;                // which half of the N tokens
    constexpr int NH = N / 2;
    constexpr int kHB = kStageBlocks / 2;    // blocks per TMEM load
    float acc[NH];
#pragma unroll
    for (int i = 0; i < NH; i++) acc[i] = 0.0f;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    for (int s = 0; s < n_stages; s++) {
      const int p = s % kStageRing, pk = s / kStageRing, ds = s % kTmemRing, dk = s / kTmemRing;
      // the stage's scales (written by the unpack warps; already complete when the MMAs are)
      if (!warp_wait(&stg_full[p], (unsigned)(pk & 1))) break;
      if (!warp_wait(&d_full[ds], (unsigned)(dk & 1))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int kb = min(kStageBlocks, n_blk - s * kStageBlocks);
      const uint16_t* wsp = (const uint16_t*)(sm + Lay::w + p * Lay::kW) + row * kStageBlocks;
      const float* sXs = (const float*)(sm + Lay::xs + p * Lay::kX) + half * NH;
      const int* sXm = (const int*)(sm + Lay::xm + p * Lay::kX) + half * NH;
#pragma unroll
      for (int hb = 0; hb < kStageBlocks / kHB; hb++) {
        uint32_t d[kHB][NH];
#pragma unroll
        for (int jj = 0; jj < kHB; jj++) {
          const int j = hb * kHB + jj;
          if (j < kb) tmem_ld<N>(tmem + lane_base + ds * (kStageBlocks * N) + j * N + half * NH, d[jj]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (hb == kStageBlocks / kHB - 1) {
          // every TMEM column of this stage is read: the MMA warp may reuse them
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) arrive(&d_empty[ds]);
        }
#pragma unroll
        for (int jj = 0; jj < kHB; jj++) {
          const int j = hb * kHB + jj;
          if (j < kb) {
            const float ws = f16bits_to_f32(wsp[j]);
            const float* xs = sXs + j * N;
            const int* xm = sXm + j * N;
#pragma unroll
            for (int i = 0; i < NH; i++) {
              const float pv = (float)((int)d[jj][i] - xm[i]);
              acc[i] = xs[i] > 0.0f ? __fmaf_rn(pv, __fmul_rn(ws, xs[i]), acc[i]) : acc[i];
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) arrive(&stg_empty[p]);  // the stage's scales are read; its A and B were read by the MMAs
    }
    // ---- outputs
    cudaGridDependencySynchronize();  // the previous kernel is done with the output buffer
    const int t = row >> 4;
    if (!abort_sh && t < n_tiles_here) {
      const int r_global = (t_first + t) * kTileRows + (row & 15);
      if (r_global < job.w.rows)
#pragma unroll
        for (int i = 0; i < NH; i++) {
          const int n = tok0 + half * NH + i;
          if (n < P.M) job.out[(size_t)n * job.ldo + r_global] = acc[i];
        }
    }
  }
  cudaTriggerProgrammaticLaunchCompletion();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == kTmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Lay::tmem_cols)
                 : "memory");
}

// ============================================================================================
// Expanded weights.  The unpack above is the kernel's critical path; with a second device copy
// of each matrix already in the shared-memory image the MMA reads, a stage is two bulk copies.
// Per 128-row group G (tiles 8G..8G+7) of a matrix with n_blk 32-column blocks:
//   [n_blk][4096]  s8 weights u - 8 of block b, K-major core matrices: 8-row group tg (rows
//                  8tg..8tg+7 of the group) at tg * 256, its two 16-column halves 128 bytes apart,
//                  a row's 16 bytes at 16 * (row & 7)
//   [n_blk][256]   the 128 rows' fp16 block scales of block b
// Rows that do not exist are zero.  With s8 weights the MMA yields
// sum (u - 8) q = sum u q - 8 sum q = dot_b exactly (xm = 8 sum q), so the chain needs no xm.
constexpr int kXA = kTcRows * 32, kXW = kTcRows * 2, kXBlk = kXA + kXW;

// One CTA per (block, group), one thread per row.  `bad` is set when a real row's scale is not
// finite (the chain below would then differ from the reference for blocks it skips).
__global__ void __launch_bounds__(kTcRows) x8_expand_kernel(W12 w, uint8_t* __restrict__ x8, int* bad) {
  const int b = blockIdx.x, G = blockIdx.y, r = threadIdx.x;
  const int n_blk = w.cols >> 5;
  uint8_t* grp = x8 + (size_t)G * n_blk * kXBlk;
  const int tg = r >> 3, ri = r & 7, t = G * 8 + (tg >> 1), g = tg & 1;
  const int n_r = t < w.n_tiles ? min(kTileRows, w.rows - t * kTileRows) : 0;
  uint2 q[4] = {};
  uint16_t sc = 0;
  if (g * 8 < n_r) {  // the group is stored (8 rows, padded)
    const uint8_t* gb = w.tiles + w.toff[t] + 16 + (size_t)g * n_blk * 144;
    const uint8_t* nib = gb + (size_t)n_blk * 16 + (size_t)b * 128;
#pragma unroll
    for (int c = 0; c < 4; c++) {  // chunk c: columns 8c + k (low nibble of byte k), 8c + 4 + k (high)
      const uint32_t v = *(const uint32_t*)(nib + c * 32 + ri * 4);
      q[c] = make_uint2(__vsub4(v & 0x0F0F0F0Fu, 0x08080808u), __vsub4((v >> 4) & 0x0F0F0F0Fu, 0x08080808u));
    }
    sc = *(const uint16_t*)(gb + (size_t)b * 16 + ri * 2);
    if (g * 8 + ri < n_r && (sc & 0x7C00u) == 0x7C00u) atomicOr(bad, 1);
  }
  uint8_t* a = grp + (size_t)b * kXA + tg * 256 + ri * 16;
#pragma unroll
  for (int c = 0; c < 4; c++) *(uint2*)(a + (c >> 1) * 128 + (c & 1) * 8) = q[c];
  *(uint16_t*)(grp + (size_t)n_blk * kXA + (size_t)b * kXW + r * 2) = sc;
}

// kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, M = 128, N.
DPUF_HD uint32_t idesc_s8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

constexpr int kXChainWarps = 8;                       // warps 0..7 (TMEM lanes 32 * (warp % 4)..)
constexpr int kXLoadWarps = 2;                        // warps 8..9: the tokens' codes and scales
constexpr int kXLoad0 = kXChainWarps;
constexpr int kXProdWarp = kXLoad0 + kXLoadWarps;     // 10: the weight stages (bulk copies)
constexpr int kXMmaWarp = kXProdWarp + 1;             // 11
constexpr int kXThreads = (kXMmaWarp + 1) * 32;       // 384
// cp.async groups of this thread still allowed in flight (an immediate operand)
DPUF_DEV void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
  }
}

// N tokens per CTA, SB blocks per stage, R stages in shared memory, TR stages in TMEM.
template <int N, int SB, int R, int TR>
struct XLayout {  // shared memory of one CTA
  static constexpr int kA = SB * kXA;      // weights of a stage
  static constexpr int kW = SB * kXW;      // row scales of a stage
  static constexpr int kB = SB * N * 32;   // the tokens' codes of a stage
  static constexpr int kX = SB * N * 4;    // the tokens' block scales of a stage
  static constexpr int a = 0;              // [R][kA]
  static constexpr int w = a + R * kA;
  static constexpr int b = w + R * kW;
  static constexpr int xs = b + R * kB;
  static constexpr int bytes = xs + R * kX;
  static constexpr int tmem_cols = TR * SB * N < 32 ? 32 : TR * SB * N;
  static_assert(R >= 2 && R <= 8, "ring depth (cp.async groups in flight)");
  static_assert((tmem_cols & (tmem_cols - 1)) == 0 && tmem_cols <= 512, "TMEM allocation");
};

// CTA = one 128-row group of one job x N tokens; CTA index = group * token tiles + token tile,
// so the token tiles of a group run side by side and share its weights through L2.  Roles:
//   warp 10     bulk copies of each stage's weights and row scales (R-deep ring);
//   warps 8..9  the tokens' codes (B, K-major core matrices) and block scales by cp.async into
//               the same ring; one mbarrier per stage completes when the weights' bytes and
//               every loader thread's copies (cp.async.mbarrier.arrive) have landed;
//   warp 11     one tcgen05.mma (M = 128, N, K = 32) per block into TMEM columns [j*N, j*N+N)
//               of a TR-deep TMEM ring, committed to an mbarrier;
//   warps 0..7  chains: warp w reads TMEM lanes 32*(w%4).. (its rows), columns of its half of
//               the tokens, and runs acc = fma((float)dot, ws * xs, acc) in block order.
// Every wait is bounded as in gemm_tc_kernel.  MINB: CTAs per SM the launch bounds allow.
template <int N, int SB, int R, int TR, int MINB>
__global__ void __launch_bounds__(kXThreads, MINB) gemm_x8_kernel(TcArgs P) {
  using Lay = XLayout<N, SB, R, TR>;
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t full[R], s_empty[R];
  __shared__ __align__(16) float xfix[kXChainWarps * (N / 2) * SB];  // see the chain warps
  __shared__ __align__(8) uint64_t d_full[TR], d_empty[TR];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- this CTA's rows and tokens
  const int n_tt = (P.M + N - 1) / N;
  const int grp = (int)blockIdx.x / n_tt, tok0 = ((int)blockIdx.x % n_tt) * N;
  int jb = 0;
  while (jb + 1 < P.J.n && grp >= P.group_prefix[jb + 1]) jb++;
  const LinJob& job = P.J.j[jb];
  const int t_first = job.t_begin + (grp - P.group_prefix[jb]) * (kTcRows / kTileRows);
  const int n_tiles_here = min(kTcRows / kTileRows, job.t_end - t_first);
  const int n_blk = job.w.cols >> 5;
  const int n_stages = (n_blk + SB - 1) / SB;
  const uint8_t* xg = job.w.x8 + (size_t)(t_first / 8) * n_blk * kXBlk;  // t_begin % 8 == 0 (host)

  if (warp == kXProdWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_sh)),
                 "r"(Lay::tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < R; i++) {
      // the producer's arrival (with the weight bytes) and one per loader thread
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&full[i])), "r"(1 + kXLoadWarps * 32)
                   : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&s_empty[i])), "r"(kXChainWarps) : "memory");
    }
    for (int i = 0; i < TR; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&d_full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&d_empty[i])), "r"(kXChainWarps) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_sh = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base_sh;
  auto arrive = [](uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
  };
  // every lane polls (no shuffle of one lane's verdict); the warp reconverges after
  auto warp_wait = [&](uint64_t* bar, unsigned par) {
    const bool ok = wait_parity(bar, par, &abort_sh, P.err);
    __syncwarp();
    return ok;
  };

  if (warp == kXProdWarp) {
    // ================================================================ weights: bulk copies
    int issued = 0;
    for (int s = 0; s < n_stages; s++) {
      const int slot = s % R, k = s / R;
      if (!warp_wait(&s_empty[slot], (unsigned)((k & 1) ^ 1))) break;
      const int b0 = s * SB, kb = min(SB, n_blk - b0);
      if (lane == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[slot])),
                     "r"((unsigned)(kb * kXBlk))
                     : "memory");
      __syncwarp();
      if (lane <= kb) {  // lanes 0..kb-1: a block's weights; lane kb: the stage's row scales
        const bool wts = lane < kb;
        unsigned char* dst = wts ? sm + Lay::a + slot * Lay::kA + lane * kXA : sm + Lay::w + slot * Lay::kW;
        const uint8_t* src = wts ? xg + (size_t)(b0 + lane) * kXA : xg + (size_t)n_blk * kXA + (size_t)b0 * kXW;
        const unsigned n = wts ? (unsigned)kXA : (unsigned)(kb * kXW);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
            "l"(src), "r"(n), "r"(su32(&full[slot]))
            : "memory");
      }
      issued = s + 1;
    }
    // copies in flight must land before the CTA exits (after an abort nobody else waits)
    if (abort_sh && lane == 0) {
      const unsigned long long t0 = gtimer();
      for (int q = max(0, issued - R); q < issued; q++) {
        unsigned ok = 0;
        while (!ok && gtimer() - t0 < kTcWaitNs)
          asm volatile(
              "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
              : "=r"(ok)
              : "r"(su32(&full[q % R])), "r"((unsigned)((q / R) & 1))
              : "memory");
      }
    }
  } else if (warp >= kXLoad0 && warp < kXLoad0 + kXLoadWarps) {
    // ================================================================ activations: cp.async
    constexpr int kLT = kXLoadWarps * 32;
    const int lt = tid - kXLoad0 * 32;
    const Act& act = job.act;
    const int xld = act.ld >> 5;
    // stage s into ring slot s % R; each loader thread's arrival on full[] is made when its
    // copies of the stage have landed (cp.async.mbarrier.arrive), so no loader ever waits for its
    // own copies and a stage is delivered as soon as its data is in
    cudaGridDependencySynchronize();  // the activations come from the previous kernel
    for (int s = 0; s < n_stages; s++) {
      const int p = s % R, b0 = s * SB, kb = min(SB, n_blk - b0);
      if (!warp_wait(&s_empty[p], (unsigned)(((s / R) & 1) ^ 1))) break;
      unsigned char* sB = sm + Lay::b + p * Lay::kB;
      float* sXs = (float*)(sm + Lay::xs + p * Lay::kX);
      for (int i = lt; i < N * SB * 2; i += kLT) {
        const int h = i & 1, n = (i >> 1) % N, j = (i >> 1) / N;
        const bool ok = j < kb && tok0 + n < P.M;
        const int8_t* src = ok ? act.q8 + (size_t)(tok0 + n) * act.ld + (size_t)(b0 + j) * 32 + h * 16 : act.q8;
        cp16_zfill(sB + j * (N * 32) + (n >> 3) * 256 + h * 128 + (n & 7) * 16, src, ok);
      }
      for (int i = lt; i < N * SB; i += kLT) {  // [block][token]
        const int j = i / N, n = i % N;
        const bool ok = j < kb && tok0 + n < P.M;
        cp4_zfill(sXs + i, ok ? act.xs + (size_t)(tok0 + n) * xld + b0 + j : act.xs, ok);
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(&full[p])) : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // nothing of ours in flight at exit
  } else if (warp == kXMmaWarp) {
    // ================================================================ MMA issuer
    const uint32_t idesc = idesc_s8(N);
    for (int s = 0; s < n_stages; s++) {
      const int p = s % R, pk = s / R, ds = s % TR, dk = s / TR;
      if (!warp_wait(&full[p], (unsigned)(pk & 1))) break;
      if (!warp_wait(&d_empty[ds], (unsigned)((dk & 1) ^ 1))) break;
      if (lane == 0) {
        // the loaders' cp.async writes of B (observed through full[]) before the tensor core reads
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int kb = min(SB, n_blk - s * SB);
        const uint64_t da0 = smem_desc(sm + Lay::a + p * Lay::kA, 128, 256);
        const uint64_t db0 = smem_desc(sm + Lay::b + p * Lay::kB, 128, 256);
        for (int j = 0; j < kb; j++) {
          const uint64_t da = da0 + (uint64_t)(j * (kXA / 16));
          const uint64_t db = db0 + (uint64_t)(j * (N * 32 / 16));
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem + ds * (SB * N) + j * N),
              "l"(da), "l"(db), "r"(idesc), "r"(0)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         su32(&d_full[ds]))
                     : "memory");
      }
      __syncwarp();
    }
  } else {
    // ================================================================ chain warps
    // From 16 tokens on, two tokens per packed fp32x2 multiply and fma (each element rounds as
    // the scalar op).  A block scale that is not > 0 is then taken as 0 once per stage: with the
    // row scale finite (the expanded copy is only made then) the fma returns acc exactly (acc is
    // never -0), as the reference's skip does.  At 8 tokens the chain is cheap next to the MMA
    // issue, and the scalar form with the skip per step is faster.
    constexpr bool kPacked = N >= 16;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane = weight row of this thread's chains
    const int half = warp >> 2;
    constexpr int NH = N / 2;
    constexpr int kRegs = MINB > 1 ? 32 : 64;  // TMEM values held per batch
    constexpr int HB = kRegs / NH < 1 ? 1 : (kRegs / NH > SB ? SB : kRegs / NH);
    static_assert(SB % HB == 0 && NH % 2 == 0, "TMEM batches, token pairs");
    float* xf = xfix + warp * (NH * SB);  // this warp's block scales of the stage, [block][token]
    uint64_t acc2[NH / 2];
#pragma unroll
    for (int i = 0; i < NH / 2; i++) acc2[i] = 0ull;  // +0.0f twice
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    for (int s = 0; s < n_stages; s++) {
      const int p = s % R, pk = s / R, ds = s % TR, dk = s / TR;
      if (!warp_wait(&full[p], (unsigned)(pk & 1))) break;  // the row and block scales
      const int kb = min(SB, n_blk - s * SB);
      const float* sXs = (const float*)(sm + Lay::xs + p * Lay::kX) + half * NH;  // block j: [j * N]
      if (kPacked) {
        for (int e = lane; e < NH * SB; e += 32) {
          const float v = sXs[(e / NH) * N + e % NH];
          xf[e] = v > 0.0f ? v : 0.0f;
        }
        __syncwarp();
      }
      if (!warp_wait(&d_full[ds], (unsigned)(dk & 1))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint16_t* wsp = (const uint16_t*)(sm + Lay::w + p * Lay::kW) + row;  // block j: [j * 128]
#pragma unroll
      for (int hb = 0; hb < SB / HB; hb++) {
        uint32_t d[HB][NH];
#pragma unroll
        for (int jj = 0; jj < HB; jj++) {
          const int j = hb * HB + jj;
          if (j < kb) tmem_ld<N>(tmem + lane_base + ds * (SB * N) + j * N + half * NH, d[jj]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (hb == SB / HB - 1) {
          // every TMEM column of this stage is read: the MMA warp may reuse them
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) arrive(&d_empty[ds]);
        }
#pragma unroll
        for (int jj = 0; jj < HB; jj++) {
          const int j = hb * HB + jj;
          if (j < kb && !kPacked) {
            const float ws = f16bits_to_f32(wsp[j * kTcRows]);
            const float* xs = sXs + j * N;
#pragma unroll
            for (int q = 0; q < NH / 2; q++) {  // acc2[q] holds tokens 2q, 2q + 1
              float a0, a1;
              asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc2[q]));
              const float x0 = xs[2 * q], x1 = xs[2 * q + 1];
              a0 = x0 > 0.0f ? __fmaf_rn(__int2float_rn((int)d[jj][2 * q]), __fmul_rn(ws, x0), a0) : a0;
              a1 = x1 > 0.0f ? __fmaf_rn(__int2float_rn((int)d[jj][2 * q + 1]), __fmul_rn(ws, x1), a1) : a1;
              asm("mov.b64 %0, {%1, %2};" : "=l"(acc2[q]) : "f"(a0), "f"(a1));
            }
          } else if (j < kb) {
            const float ws = f16bits_to_f32(wsp[j * kTcRows]);
            uint64_t ws2;
            asm("mov.b64 %0, {%1, %1};" : "=l"(ws2) : "f"(ws));
            const uint64_t* xs2 = (const uint64_t*)(xf + j * NH);
#pragma unroll
            for (int q = 0; q < NH / 2; q++) {
              uint64_t w2, pv2;
              asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(w2) : "l"(ws2), "l"(xs2[q]));
              asm("mov.b64 %0, {%1, %2};"
                  : "=l"(pv2)
                  : "f"(__int2float_rn((int)d[jj][2 * q])), "f"(__int2float_rn((int)d[jj][2 * q + 1])));
              asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc2[q]) : "l"(pv2), "l"(w2));
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) arrive(&s_empty[p]);  // scales read; A and B were read by the MMAs
    }
    float acc[NH];
#pragma unroll
    for (int q = 0; q < NH / 2; q++) asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[2 * q]), "=f"(acc[2 * q + 1]) : "l"(acc2[q]));
    // ---- outputs
    cudaGridDependencySynchronize();  // the previous kernel is done with the output buffer
    const int t = row >> 4;
    if (!abort_sh && t < n_tiles_here) {
      const int r_global = (t_first + t) * kTileRows + (row & 15);
      if (r_global < job.w.rows)
#pragma unroll
        for (int i = 0; i < NH; i++) {
          const int n = tok0 + half * NH + i;
          if (n < P.M) job.out[(size_t)n * job.ldo + r_global] = acc[i];
        }
    }
  }
  cudaTriggerProgrammaticLaunchCompletion();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == kXProdWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Lay::tmem_cols)
                 : "memory");
}

// Shared memory of a launch: a CTA that must hold its SM alone (MINB 1: its TMEM allocation
// may be the whole TMEM) asks for at least 116 KB.
template <int N, int SB, int R, int TR, int MINB>
size_t x8_smem_bytes() {
  static_assert(MINB == 1 || (2 * XLayout<N, SB, R, TR>::tmem_cols <= 512 &&
                              XLayout<N, SB, R, TR>::bytes + 2048 <= 113 * 1024),
                "two CTAs per SM: TMEM and shared memory");
  const size_t b = (size_t)XLayout<N, SB, R, TR>::bytes;
  return MINB > 1 ? b : std::max(b, (size_t)116 * 1024);
}

template <int N>
size_t tc_smem_bytes() {
  return (size_t)TcLayout<N>::bytes;
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

// Shared memory per CTA at least 116 KB, so that one CTA holds an SM (its TMEM allocation is
// up to 512 columns, the whole TMEM) and an allocation never waits on another CTA.
constexpr size_t kTcMinSmem = 116 * 1024;

// Shapes of the expanded-weight GEMM: (N tokens, SB blocks per stage, R shared-memory stages,
// TR TMEM stages, CTAs per SM), with the measured cost of one CTA: about 5 us plus us_per_blk
// for each 32-column block (B200, the MMA issue and the stage hand-offs dominate; the chain's
// share grows with N).
struct X8Variant {
  int n, minb;
  float us_per_blk;
  cudaError_t (*launch)(const Launch&, dim3, const TcArgs&);
  cudaError_t (*configure)();
};
template <int N, int SB, int R, int TR, int MINB>
cudaError_t x8_launch(const Launch& L, dim3 grid, const TcArgs& P) {
  return launch_k(L, gemm_x8_kernel<N, SB, R, TR, MINB>, grid, dim3(kXThreads), x8_smem_bytes<N, SB, R, TR, MINB>(),
                  P);
}
template <int N, int SB, int R, int TR, int MINB>
cudaError_t x8_configure() {
  return set_max_dyn_smem(gemm_x8_kernel<N, SB, R, TR, MINB>);
}
#define DPUF_X8(N, SB, R, TR, MINB, C) {N, MINB, C, x8_launch<N, SB, R, TR, MINB>, x8_configure<N, SB, R, TR, MINB>}
const X8Variant kX8Variants[] = {
    DPUF_X8(8, 8, 4, 4, 1, 0.105f),
    DPUF_X8(16, 8, 4, 4, 1, 0.126f),
    DPUF_X8(32, 8, 4, 2, 1, 0.174f),
    DPUF_X8(64, 4, 6, 2, 1, 0.30f),
};
#undef DPUF_X8
constexpr int kX8NumVariants = (int)(sizeof(kX8Variants) / sizeof(kX8Variants[0]));

// The variant with the least modelled time for M tokens over n_groups 128-row groups of n_blk
// blocks: waves of one CTA per SM times the per-CTA cost.  Env DPUF_CUDA_X8_VARIANT=i forces
// kX8Variants[i] (tuning).
int x8_choose(int M, int n_groups, int n_blk, int n_sms) {
  if (const char* v = getenv("DPUF_CUDA_X8_VARIANT")) {
    const int i = atoi(v);
    if (i >= 0 && i < kX8NumVariants) return i;
  }
  int best = 0;
  double best_t = 1e30;
  for (int i = 0; i < kX8NumVariants; i++) {
    const X8Variant& v = kX8Variants[i];
    if (i > 0 && kX8Variants[i - 1].n >= M) break;  // a narrower tile already covers M
    const long long ctas = (long long)n_groups * ((M + v.n - 1) / v.n);
    const long long slots = (long long)n_sms * v.minb;
    const double t = (double)((ctas + slots - 1) / slots) * (5.0 + n_blk * v.us_per_blk);
    if (t < best_t) best_t = t, best = i;
  }
  return best;
}
}  // namespace

cudaError_t configure_gemm_tc_kernels() {
  cudaError_t e;
  if ((e = set_max_dyn_smem(gemm_tc_kernel<8>)) != cudaSuccess) return e;
  if ((e = set_max_dyn_smem(gemm_tc_kernel<16>)) != cudaSuccess) return e;
  if ((e = set_max_dyn_smem(gemm_tc_kernel<32>)) != cudaSuccess) return e;
  for (const X8Variant& v : kX8Variants)
    if ((e = v.configure()) != cudaSuccess) return e;
  return cudaSuccess;
}

size_t x8_bytes(const W12& w) { return (size_t)((w.n_tiles + 7) / 8) * (size_t)(w.cols / 32) * kXBlk; }

cudaError_t launch_x8_expand(cudaStream_t s, const W12& w, uint8_t* x8, int* bad) {
  if (w.mode != 12 || w.cols % 32 != 0 || w.n_tiles <= 0) return cudaErrorInvalidValue;
  x8_expand_kernel<<<dim3((unsigned)(w.cols / 32), (unsigned)((w.n_tiles + 7) / 8)), kTcRows, 0, s>>>(w, x8, bad);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const Launch& L, const LinJobs& jobs, int M, int* err) {
  TcArgs P = {};
  P.J = jobs;
  P.M = M;
  P.err = err;
  P.group_prefix[0] = 0;
  bool x8 = true;  // every job has expanded weights and starts on a 128-row group
  for (int i = 0; i < jobs.n; i++) {
    if (jobs.j[i].w.cols != jobs.j[0].w.cols) return cudaErrorInvalidValue;
    const int tiles = jobs.j[i].t_end - jobs.j[i].t_begin;
    P.group_prefix[i + 1] = P.group_prefix[i] + (tiles + 7) / 8;
    x8 = x8 && jobs.j[i].w.x8 && jobs.j[i].t_begin % 8 == 0;
  }
  P.n_groups = P.group_prefix[jobs.n];
  if (P.n_groups == 0 || M <= 0) return cudaSuccess;
  if (x8) {
    static const int n_sms = [] {
      int dev = 0, n = 148;
      if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      return n;
    }();
    const X8Variant& v = kX8Variants[x8_choose(M, P.n_groups, jobs.j[0].w.cols / 32, n_sms)];
    return v.launch(L, dim3((unsigned)(P.n_groups * ((M + v.n - 1) / v.n))), P);
  }
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
