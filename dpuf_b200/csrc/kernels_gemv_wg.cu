// kernels_gemv_wg.cu - mode-12 GEMV for one token (M = 1): every consumer warp owns whole
// 8-row groups and computes their rows start to finish, so no warp waits for another.
//
// Per output row r (dpuf_matmul_qr_hadamard4_packed_tile_range M=1 path, dpuf_avx2.c:2601-2640):
//   dot_b = sum_k (u_k - 8) q_k                     exact integer (dp4a on the nibbles)
//   acc   = fmaf((float)dot_b, ws_b * xs_b, acc)     blocks b ascending, blocks with xs_b <= 0
//                                                    leave acc untouched
//
// Work.  A job list (up to three matrices with the same K) is a list of 8-row groups (two per
// 16-row container tile; the second group of a tile with at most 8 rows is empty).  One CTA per
// SM takes a contiguous range of groups; consumer warp w of the CTA takes the range's groups
// w, w + kWarps, ... and streams each group's K in stages of 32 blocks (512 bytes of fp16 row
// scales, then 4096 bytes of nibbles: exactly the container's bytes, in two cp.async.bulk
// copies).
//
// Ring.  Every warp has its own kSlots-deep ring of stages, one mbarrier each, and issues its own
// copies: lane 0 requests the first kSlots stages at start and refills a slot with the stage
// kSlots ahead as soon as the warp has finished with it, so the CTA keeps kWarps * kSlots *
// 4.6 KB of weights in flight, no thread polls other warps' slots and a slow warp never stalls
// the others.  The weights do not depend on the previous kernel, so the stream starts before
// griddepcontrol.wait (programmatic dependent launch).
//
// Lanes.  Lane (ri = lane % 8, q = lane / 8) computes row ri's dots of blocks 8q .. 8q+7 of a
// stage; its four nibble words per block are read starting at chunk q (rotated), so the four
// lane octets hit different banks.  The in-order chain then runs octet by octet: octet q
// continues row ri's accumulator over its eight blocks and hands it to octet q+1 with a
// shuffle - the reference's sequential chain, bit for bit.
#include <algorithm>

#include "kernels.cuh"

namespace dpuf {

namespace {

constexpr int kWarps = 12;                    // warps, each its own ring
constexpr int kSlots = 3;                     // ring slots per consumer warp
constexpr int kKB = 32;                       // blocks per stage
constexpr int kScBytes = kKB * 16;            // 512: fp16 scales [32][8]
constexpr int kSlotBytes = kScBytes + kKB * 128;  // 4608
constexpr int kThreads = kWarps * 32;         // 384
constexpr unsigned long long kWaitNs = 2000000000ull;

struct WgArgs {
  LinJobs J;
  int group_prefix[kMaxJobs + 1];  // cumulative groups (2 per tile) per job
  int x_slot[kMaxJobs];
  int n_x, n_groups, n_blk, n_st, cols;
  int x_stride;                    // bytes per staged activation: cols codes + n_blk * 8
  int* err;                        // optional: 1 when a wait gave up
};

DPUF_DEV unsigned su32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
DPUF_DEV void wg_mbar_init(uint64_t* b, unsigned c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c) : "memory");
}
DPUF_DEV void wg_mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
DPUF_DEV void wg_mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
DPUF_DEV bool wg_mbar_try(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(su32(b)), "r"(parity)
               : "memory");
  return ok != 0;
}
DPUF_DEV uint64_t wg_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
DPUF_DEV void wg_bulk(void* dst, const void* src, unsigned bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          su32(dst)),
      "l"(src), "r"(bytes), "r"(su32(bar)), "l"(pol)
      : "memory");
}
DPUF_DEV unsigned long long wg_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// u8 (weights, 0..15 or 16 * 0..15) x s8 (activation codes) dot of four byte pairs
DPUF_DEV int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Group gi of the job list: its first tile byte (group header excluded), rows, output.
struct GroupRef {
  const uint8_t* base;  // scales of block 0
  int n_r;              // rows in the group (0: empty)
  float* out;
  int xoff;             // offset of the job's staged activation
};
DPUF_DEV GroupRef group_ref(const WgArgs& A, int gi) {
  int j = 0;
  while (j + 1 < A.J.n && gi >= A.group_prefix[j + 1]) j++;
  const LinJob& job = A.J.j[j];
  const int local = gi - A.group_prefix[j];
  const int t = job.t_begin + (local >> 1), g = local & 1;
  GroupRef r;
  const int row0 = t * kTileRows + g * 8;
  r.n_r = max(0, min(8, job.w.rows - row0));
  r.base = job.w.tiles + job.w.toff[t] + 16 + (size_t)g * A.n_blk * 144;
  r.out = job.out + row0;
  r.xoff = A.x_slot[j] * A.x_stride;
  return r;
}

template <bool kFull>
DPUF_DEV void stage_chain(const unsigned char* slot, const int8_t* xq, const float* xs, const int* xm, int b0, int kb,
                          int ri, int q, int lane, float& acc) {
  const unsigned char* nib = slot + kScBytes;
  float pp[8], ss[8];
  bool on[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int bl = q * 8 + j;
    pp[j] = 0.0f;
    ss[j] = 0.0f;
    on[j] = false;
    if (kFull || bl < kb) {
      const int b = b0 + bl;
      int dlo = 0, dhi = 0;
#pragma unroll
      for (int c4 = 0; c4 < 4; c4++) {
        const int cc = (c4 + q) & 3;
        const uint32_t w = *(const uint32_t*)(nib + bl * 128 + cc * 32 + ri * 4);
        const int2 xv = *(const int2*)(xq + b * 32 + cc * 8);
        dlo = dp4a_us(w & 0x0F0F0F0Fu, xv.x, dlo);
        dhi = dp4a_us(w & 0xF0F0F0F0u, xv.y, dhi);
      }
      const float bsc = xs[b];
      const float ws = f16bits_to_f32(*(const uint16_t*)(slot + bl * 16 + ri * 2));
      pp[j] = (float)(dlo + (dhi >> 4) - xm[b]);
      ss[j] = __fmul_rn(ws, bsc);
      on[j] = bsc > 0.0f;
    }
  }
  // in-order chain: octet q continues the row's accumulator over its blocks, then passes it on
#pragma unroll
  for (int qq = 0; qq < 4; qq++) {
    if (q == qq) {
#pragma unroll
      for (int j = 0; j < 8; j++) acc = on[j] ? __fmaf_rn(pp[j], ss[j], acc) : acc;
    }
    acc = __shfl_sync(kFull, acc, ri + 8 * qq);
  }
  (void)lane;
}

// The copies of one stage (scales, then nibbles) of group `gr` into `dst`, completing on `bar`.
DPUF_DEV void issue_stage(const GroupRef& gr, int s, int n_blk, unsigned char* dst, uint64_t* bar, uint64_t pol) {
  const int kb = min(kKB, n_blk - s * kKB);
  if (gr.n_r == 0) {
    wg_mbar_arrive(bar);  // empty group: nothing to copy
    return;
  }
  wg_mbar_expect_tx(bar, (unsigned)kb * 144);
  wg_bulk(dst, gr.base + (size_t)s * kScBytes, (unsigned)kb * 16, bar, pol);
  wg_bulk(dst + kScBytes, gr.base + (size_t)n_blk * 16 + (size_t)s * (kKB * 128), (unsigned)kb * 128, bar, pol);
}

__global__ void __launch_bounds__(kThreads, 1) gemv_wg_kernel(WgArgs A, const int* skip_flag) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full[kWarps * kSlots];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g0 = (int)((long long)A.n_groups * blockIdx.x / gridDim.x);
  const int g1 = (int)((long long)A.n_groups * (blockIdx.x + 1) / gridDim.x);
  const int n_local = g1 - g0;
  unsigned char* ring = smem + (size_t)warp * kSlots * kSlotBytes;
  uint64_t* bars = full + warp * kSlots;
  int8_t* xall = (int8_t*)(smem + (size_t)kWarps * kSlots * kSlotBytes);
  const int n_st = A.n_st, n_blk = A.n_blk;
  // this warp's stages: groups k = warp, warp + kWarps, ... of the CTA's range, n_st each
  const int my_groups = warp < n_local ? (n_local - warp + kWarps - 1) / kWarps : 0;
  const int my_stages = my_groups * n_st;
  const uint64_t pol = wg_evict_first();
  if (lane == 0)
    for (int i = 0; i < kSlots; i++) wg_mbar_init(&bars[i], 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncwarp();
  const bool skip_mode = skip_flag != nullptr;
  // issue cursor (lane 0): stage `is` of this warp's group `ik`
  int ik = 0, is = 0, issued = 0;
  GroupRef icur{};
  auto issue_next = [&](int slot) {
    if (is == 0) icur = group_ref(A, g0 + warp + ik * kWarps);
    issue_stage(icur, is, n_blk, ring + (size_t)slot * kSlotBytes, &bars[slot], pol);
    if (++is == n_st) {
      is = 0;
      ik++;
    }
    issued++;
  };
  // the weights do not depend on the previous kernel: the first stages are requested before
  // waiting for it (programmatic dependent launch), unless a skip flag decides whether to run
  if (!skip_mode && lane == 0)
    for (int i = 0; i < kSlots && issued < my_stages; i++) issue_next(i);
  cudaGridDependencySynchronize();
  cudaTriggerProgrammaticLaunchCompletion();
  if (skip_mode) {
    if (*(volatile const int*)skip_flag) return;
    if (lane == 0)
      for (int i = 0; i < kSlots && issued < my_stages; i++) issue_next(i);
  }
  // stage each distinct activation: codes, block scales, block sums
  for (int jx = 0; jx < A.J.n; jx++) {
    bool first = true;
    for (int jj = 0; jj < jx; jj++) first = first && (A.x_slot[jj] != A.x_slot[jx]);
    if (!first) continue;
    const Act& a = A.J.j[jx].act;
    int8_t* xq = xall + A.x_slot[jx] * A.x_stride;
    float* xs = (float*)(xq + A.cols);
    int* xm = (int*)(xs + n_blk);
    for (int i = tid; i < A.cols / 16; i += kThreads) ((int4*)xq)[i] = ((const int4*)a.q8)[i];
    for (int i = tid; i < n_blk; i += kThreads) {
      xs[i] = a.xs[i];
      xm[i] = a.xm[i];
    }
  }
  __syncthreads();

  const int ri = lane & 7, q = lane >> 3;
  int slot = 0, consumed = 0;
  unsigned ph = 0;
  bool ok = true;
  for (int k = 0; k < my_groups; k++) {
    const GroupRef gr = group_ref(A, g0 + warp + k * kWarps);
    const int8_t* xq = xall + gr.xoff;
    const float* xs = (const float*)(xq + A.cols);
    const int* xm = (const int*)(xs + n_blk);
    float acc = 0.0f;
    for (int s = 0; s < n_st; s++) {
      if (ok && !wg_mbar_try(&bars[slot], ph)) {
        const unsigned long long t0 = wg_timer();
        while (!wg_mbar_try(&bars[slot], ph)) {
          if (wg_timer() - t0 > kWaitNs) {
            if (A.err) atomicExch(A.err, 1);
            ok = false;
            break;
          }
        }
      }
      ok = __all_sync(kFull, ok);
      if (ok && gr.n_r > 0) {
        const int b0 = s * kKB, kb = min(kKB, n_blk - b0);
        const unsigned char* st = ring + (size_t)slot * kSlotBytes;
        if (kb == kKB)
          stage_chain<true>(st, xq, xs, xm, b0, kb, ri, q, lane, acc);
        else
          stage_chain<false>(st, xq, xs, xm, b0, kb, ri, q, lane, acc);
      }
      __syncwarp();  // every lane is done with the slot: refill it
      if (ok) consumed++;
      if (lane == 0 && ok && issued < my_stages) issue_next(slot);
      if (++slot == kSlots) {
        slot = 0;
        ph ^= 1u;
      }
    }
    if (ok && q == 0 && ri < gr.n_r) gr.out[ri] = acc;
  }
  // copies still in flight (only after a wait gave up) must land before the CTA exits: stages
  // consumed .. issued-1, stage i in slot i % kSlots with parity (i / kSlots) & 1
  if (!ok && lane == 0) {
    const unsigned long long t0 = wg_timer();
    for (int i = consumed; i < issued; i++)
      while (!wg_mbar_try(&bars[i % kSlots], (unsigned)(i / kSlots) & 1u) && wg_timer() - t0 < kWaitNs) {
      }
  }
}

template <typename K, typename... Args>
cudaError_t launch_wg(const Launch& L, K kernel, dim3 grid, dim3 block, size_t smem, Args... args) {
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

int g_wg_sms[64] = {};

}  // namespace

cudaError_t configure_gemv_wg_kernel() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && dev >= 0 && dev < 64)
    e = cudaDeviceGetAttribute(&g_wg_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = set_max_dyn_smem(gemv_wg_kernel);
  return e;
}

size_t gemv_wg_smem_bytes(int cols, int n_x) {
  return (size_t)kWarps * kSlots * kSlotBytes + (size_t)n_x * (((size_t)cols + (size_t)(cols / 32) * 8 + 15) & ~(size_t)15);
}

cudaError_t launch_gemv_wg(const Launch& L, const LinJobs& jobs, const int* skip_flag, int* err) {
  WgArgs A;
  A.J = jobs;
  A.group_prefix[0] = 0;
  A.n_x = 0;
  A.cols = jobs.j[0].w.cols;
  for (int i = 0; i < jobs.n; i++) {
    if (jobs.j[i].w.cols != A.cols) return cudaErrorInvalidValue;  // one K per launch
    A.group_prefix[i + 1] = A.group_prefix[i] + 2 * (jobs.j[i].t_end - jobs.j[i].t_begin);
    int slot = -1;
    for (int k = 0; k < i; k++)
      if (jobs.j[k].act.q8 == jobs.j[i].act.q8) slot = A.x_slot[k];
    A.x_slot[i] = slot >= 0 ? slot : A.n_x++;
  }
  A.n_groups = A.group_prefix[jobs.n];
  if (A.n_groups == 0) return cudaSuccess;
  if (A.cols % 32) return cudaErrorInvalidValue;
  A.n_blk = A.cols / 32;
  A.n_st = (A.n_blk + kKB - 1) / kKB;
  A.x_stride = (A.cols + A.n_blk * 8 + 15) & ~15;
  A.err = err;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = (dev >= 0 && dev < 64 && g_wg_sms[dev] > 0) ? g_wg_sms[dev] : 148;
  const int grid = std::min(sms, A.n_groups);
  const size_t smem = gemv_wg_smem_bytes(A.cols, A.n_x);
  if (smem > (size_t)kMaxDynSmem) return cudaErrorInvalidValue;
  return launch_wg(L, gemv_wg_kernel, dim3((unsigned)grid), dim3(kThreads), smem, A, skip_flag);
}

}  // namespace dpuf
