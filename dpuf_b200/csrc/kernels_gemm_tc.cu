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

DPUF_DEV bool wait_parity(uint64_t* bar, unsigned par, volatile int* abort_flag, int* err) {
  const unsigned long long t0 = gtimer();
  for (;;) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(su32(bar)), "r"(par), "r"(20000u)
        : "memory");
    if (ok) return true;
    if (*abort_flag || gtimer() - t0 > kTcWaitNs) {
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
