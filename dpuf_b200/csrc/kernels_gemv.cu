// kernels_gemv.cu - HBM-streaming mode-12 GEMV for decode (M = 1).
//
// Per output row r (dpuf_matmul_qr_hadamard4_packed_tile_range M=1 path, dpuf_avx2.c:2601-2640):
//   dot_b = sum_k u_k q_k - xm_b                      exact integers (dp4a on nibbles)
//   acc   = fmaf((float)dot_b, ws_b * xs_b, acc)        blocks b ascending, xs_b <= 0 skipped
//
// Work list.  The weight is a list of units (16-row container tiles, possibly from up to three
// matrices with the same K); each unit is n_st stages of KB = 32 blocks (1024 columns).  The
// units are dealt to a persistent grid (up to four CTAs per SM) in contiguous ranges; the
// grid is the smallest one that reaches the minimal number of units per CTA, so the ranges
// are as even as whole units allow.  Only a GEMV with fewer units than SMs splits units.
// Streaming.  A CTA copies its items into an NS-stage shared-memory ring with 16-byte cp.async
// (thread t copies pieces t and t + 160 of each 8-row group), continuously across unit boundaries; the first
// NS-1 stages are requested before griddepcontrol.wait, so with programmatic dependent launch
// the stream starts while the previous kernel is still finishing.
// Compute, as a two-step pipeline over the stages of a CTA (one __syncthreads per stage):
//   MMA warps (4)  stage i, 8 blocks each: the integer block dots with warp-level int8 MMA
//                  (m16n8k32, exact int32).  A = the activation block (all 16 A rows equal),
//                  B = 8 weight rows' nibbles (0..15) of one block; lane (g, t) supplies weight
//                  row g, chunk t: its low nibbles as k = 4t..4t+3 and its high nibbles as
//                  k = 16+4t..16+4t+3, with A permuted the same way, so B needs one load and two
//                  masks.  Lane (g, t) keeps rows 2t, 2t+1 of the warp's g-th block and writes
//                  the pairs p = float(dot - xm), s = ws * xs (both 0 for a skipped block, which
//                  leaves the chain unchanged bit for bit).
//   chain warp (1) stage i-1: lane = row, acc = fma(p, s, acc) over the blocks in order.
// Units split between CTAs.  The in-order chain is kept exact: the part holding stage 0 (head)
// stores its accumulator after its last stage, every later part stores its pairs, and the last
// part to finish (an atomic arrival count; nobody waits) continues the chain from the head's
// accumulator through the stored pairs in block order and writes the rows.  Without scratch
// (split == nullptr) units are never split.
// Bank layout.  Within a stage the nibbles of group g start at g * (KB*128 + 32) bytes; the B
// load of one MMA (lane (g, t) reads word 8t + g of a block) covers 32 consecutive words.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "kernels.cuh"

namespace dpuf {

namespace {

constexpr int kKB = 32;  // blocks (of 32 columns) per stage
constexpr int kMmaWarps = 4;
constexpr int kChainWarp = kMmaWarps;
constexpr int kThreads = (kChainWarp + 1) * 32;  // 160
constexpr int kRT = 16;                         // rows per unit (one container tile)
constexpr int kNG = 2;                          // 8-row groups per unit
constexpr int kQG = kKB * 128 + 32;             // nibble bytes per group per stage (+ bank pad)
constexpr int kSG = kKB * 16 + 32;              // scale bytes per group per stage (+ bank pad)
constexpr int kStage = kNG * (kQG + kSG);       // 9344
constexpr int kNS = 4;                          // ring depth (four CTAs per SM)
constexpr int kPF = kNS - 1;                     // stages in flight ahead of the MMA warps
constexpr int kPsStride = 24;                   // pairs per block row (16 used; conflict-free stores)
constexpr int kPsBytes = 2 * kKB * kPsStride * 8;  // double-buffered (p, s) pairs
constexpr int kMaxUnitsPerCta = 96;
constexpr int kCopyThreads = kKB * 8 + kKB;     // 288: nibble pieces then scale pieces of a group
static_assert(kStage % 128 == 0, "stage alignment");
static_assert(2 * kThreads >= kCopyThreads, "every thread copies at most two pieces per group");

DPUF_DEV void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
DPUF_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
DPUF_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// D = A (16x32 int8, row-major) * B (32x8 int8, col-major), int32 accumulate from zero.
DPUF_DEV void mma_s8_16832(int& d0, int& d1, int& d2, int& d3, int a0, int a1, int a2, int a3, int b0, int b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

struct GemvArgs {
  LinJobs J;
  int unit_prefix[kMaxJobs + 1];  // cumulative units per job
  int x_slot[kMaxJobs];           // which staged activation each job uses
  int n_x;                        // distinct activations
  int n_units, n_st, n_blk, cols;
  long long items;                // n_units * n_st
  GemvSplit split;                // scratch for units split between CTAs (or all null)
  int whole_units;                // 1: CTA ranges cover whole units (no scratch)
};

DPUF_DEV long long range_begin(const GemvArgs& A, int c) {
  if (A.whole_units) return (long long)((long long)A.n_units * c / gridDim.x) * A.n_st;
  return A.items * c / gridDim.x;
}
// CTA whose range contains item i.
DPUF_DEV int owner_of(const GemvArgs& A, long long i) {
  int c = (int)(i * gridDim.x / A.items);
  while (c > 0 && range_begin(A, c) > i) c--;
  while (c + 1 < (int)gridDim.x && range_begin(A, c + 1) <= i) c++;
  return c;
}

__global__ void __launch_bounds__(kThreads, 4) gemv_stream_kernel(GemvArgs A, const int* skip_flag) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ const uint8_t* unit_base[kMaxUnitsPerCta];  // tile start of each unit of this CTA
  __shared__ int unit_rows[kMaxUnitsPerCta];
  unsigned char* ring = smem;
  float2* ps = (float2*)(smem + kNS * kStage);
  int8_t* xq_all = (int8_t*)(smem + kNS * kStage + kPsBytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const long long i0 = range_begin(A, c), i1 = range_begin(A, c + 1);
  if (i0 >= i1) {
    cudaGridDependencySynchronize();
    cudaTriggerProgrammaticLaunchCompletion();
    return;
  }
  const int n_st = A.n_st, n_blk = A.n_blk, cols = A.cols;
  const int u_first = (int)(i0 / n_st);
  const int s_first = (int)(i0 - (long long)u_first * n_st);  // stage of this CTA's first item
  const int n_items = (int)(i1 - i0);
  const int n_my_units = (s_first + n_items + n_st - 1) / n_st;
  const int x_stride = cols + n_blk * 8;
  __shared__ float* unit_out[kMaxUnitsPerCta];  // output rows of each unit
  __shared__ int unit_xoff[kMaxUnitsPerCta];    // offset of the unit's staged activation

  // per-unit tables of this CTA (weights metadata: independent of the previous kernel)
  for (int k = tid; k < n_my_units; k += kThreads) {
    const int u = u_first + k;
    int j = 0;
    while (j + 1 < A.J.n && u >= A.unit_prefix[j + 1]) j++;
    const LinJob& job = A.J.j[j];
    const int t = job.t_begin + (u - A.unit_prefix[j]);
    unit_base[k] = job.w.tiles + job.w.toff[t];
    unit_rows[k] = min(kTileRows, job.w.rows - t * kTileRows);
    unit_out[k] = job.out + (size_t)t * kTileRows;
    unit_xoff[k] = A.x_slot[j] * x_stride;
  }
  __syncthreads();

  // copy assignment: per group and item there are 288 16-byte pieces, 256 of nibbles (piece p
  // holds block p/8) and 32 of scales (one block each); thread t moves pieces t and t + 160
  int ik = 0, is = s_first, islot = 0;  // issue cursor: unit, stage, ring slot
  auto copy_piece = [&](int pc, const uint8_t* tb, unsigned char* stage) {
    const bool q = pc < kKB * 8;
    const int pi = q ? pc : pc - kKB * 8;
    if (is * kKB + (q ? (pi >> 3) : pi) >= n_blk) return;  // partial last stage
    const int src = q ? n_blk * 16 + is * (kKB * 128) + pi * 16 : is * (kKB * 16) + pi * 16;
    unsigned char* dst = stage + (q ? pi * 16 : kNG * kQG + pi * 16);
    cp_async16(dst, tb + src);
    if (unit_rows[ik] > 8) cp_async16(dst + (q ? kQG : kSG), tb + n_blk * 144 + src);
  };
  auto issue_next = [&]() {
    const uint8_t* tb = unit_base[ik] + 16;
    unsigned char* stage = ring + islot * kStage;
    copy_piece(tid, tb, stage);
    if (tid + kThreads < kCopyThreads) copy_piece(tid + kThreads, tb, stage);
    if (++is == n_st) { is = 0; ik++; }
    if (++islot == kNS) islot = 0;
  };

  const bool skip_mode = skip_flag != nullptr;
  if (!skip_mode) {
#pragma unroll 1
    for (int q = 0; q < kPF; q++) {
      if (q < n_items) issue_next();
      cp_async_commit();
    }
  }
  cudaGridDependencySynchronize();
  cudaTriggerProgrammaticLaunchCompletion();
  if (skip_mode) {
    if (*skip_flag) return;
#pragma unroll 1
    for (int q = 0; q < kPF; q++) {
      if (q < n_items) issue_next();
      cp_async_commit();
    }
  }
  // activations (each distinct one once): codes, block scales, block sums
  for (int jx = 0; jx < A.J.n; jx++) {
    bool first = true;
    for (int jj = 0; jj < jx; jj++) first = first && (A.x_slot[jj] != A.x_slot[jx]);
    if (!first) continue;
    const Act& a = A.J.j[jx].act;
    int8_t* xq = xq_all + A.x_slot[jx] * x_stride;
    float* xs = (float*)(xq + cols);
    int* xm = (int*)(xs + n_blk);
    for (int i = tid; i < cols / 16; i += kThreads) ((int4*)xq)[i] = ((const int4*)a.q8)[i];
    for (int i = tid; i < n_blk; i += kThreads) {
      xs[i] = a.xs[i];
      xm[i] = a.xm[i];
    }
  }

  // per-role cursors over this CTA's items: unit k, stage s, ring slot
  int mk = 0, ms = s_first, mslot = 0;  // MMA warps: item ii
  int ck = 0, cs = s_first;             // chain warp: item ii - 1
  bool c_head = true, c_split = false;
  int c_slot = 0;
  float acc = 0.0f;
  auto chain_unit_begin = [&]() {
    const long long ub = (long long)(u_first + ck) * n_st;
    c_head = ub >= i0;
    c_split = !A.whole_units && (ub < i0 || ub + n_st > i1);
    c_slot = c_split ? owner_of(A, ub) : 0;
    acc = 0.0f;
  };
  if (warp == kChainWarp) chain_unit_begin();

  for (int ii = 0; ii <= n_items; ii++) {
    cp_async_wait<kPF - 1>();
    __syncthreads();  // item ii landed; every role finished iteration ii-1
    if (ii + kPF < n_items) issue_next();  // refills the slot of item ii-1 (no longer read)
    cp_async_commit();
    if (warp < kMmaWarps) {
      // ---- item ii, blocks 8w..8w+7: integer dots by MMA for both 8-row groups; lane (g, t)
      // keeps block 8w+g, rows 2t and 2t+1 of each group, and turns them into (p, s) pairs
      if (ii < n_items) {
        const int b0 = ms * kKB, kb = min(kKB, n_blk - b0);
        const int8_t* xq = xq_all + unit_xoff[mk];
        const float* xs = (const float*)(xq + cols);
        const int* xm = (const int*)(xs + n_blk);
        const unsigned char* st = ring + mslot * kStage;
        const int g = lane >> 2, t = lane & 3;
        constexpr int per = kKB / kMmaWarps;  // 8 blocks per warp
        int keep[kNG][2];
#pragma unroll 4
        for (int j = 0; j < per; j++) {
          const int bb = warp * per + j;
          if (bb >= kb) break;  // partial last stage (warp-uniform): no activation bytes there
          const int2 xw = *(const int2*)(xq + (b0 + bb) * 32 + t * 8);  // x words 2t, 2t+1
#pragma unroll
          for (int grp = 0; grp < kNG; grp++) {
            const uint32_t w = *(const uint32_t*)(st + grp * kQG + bb * 128 + t * 32 + g * 4);
            int d0, d1, d2, d3;
            mma_s8_16832(d0, d1, d2, d3, xw.x, xw.x, xw.y, xw.y, (int)(w & 0x0F0F0F0Fu),
                         (int)((w >> 4) & 0x0F0F0F0Fu));
            if (g == j) {
              keep[grp][0] = d0;
              keep[grp][1] = d1;
            }
          }
        }
        const int bb = warp * per + g;
        if (bb < kb) {
          const int b = b0 + bb;
          const float bsc = xs[b];
          const int xmb = xm[b];
          float2* out = ps + (ii & 1) * kKB * kPsStride + bb * kPsStride + 2 * t;
#pragma unroll
          for (int grp = 0; grp < kNG; grp++) {
            float4 pr = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (bsc > 0.0f) {
              const uint32_t ws2 = *(const uint32_t*)(st + kNG * kQG + grp * kSG + bb * 16 + t * 4);
              pr.x = (float)(keep[grp][0] - xmb);
              pr.y = __fmul_rn(f16bits_to_f32((uint16_t)(ws2 & 0xFFFFu)), bsc);
              pr.z = (float)(keep[grp][1] - xmb);
              pr.w = __fmul_rn(f16bits_to_f32((uint16_t)(ws2 >> 16)), bsc);
            }
            *(float4*)(out + grp * 8) = pr;
          }
        }
        if (++ms == n_st) { ms = 0; mk++; }
        if (++mslot == kNS) mslot = 0;
      }
    } else if (ii >= 1) {
      // ---- chain warp: item ii-1 (unit ck, stage cs)
      const int kb = min(kKB, n_blk - cs * kKB);
      const float2* in_ps = ps + ((ii - 1) & 1) * kKB * kPsStride;
      if (c_head) {
        if (lane < kRT) {
          int b = 0;
          for (; b + 3 < kb; b += 4) {
            const float2 a0 = in_ps[(b + 0) * kPsStride + lane], a1 = in_ps[(b + 1) * kPsStride + lane];
            const float2 a2 = in_ps[(b + 2) * kPsStride + lane], a3 = in_ps[(b + 3) * kPsStride + lane];
            acc = __fmaf_rn(a0.x, a0.y, acc);
            acc = __fmaf_rn(a1.x, a1.y, acc);
            acc = __fmaf_rn(a2.x, a2.y, acc);
            acc = __fmaf_rn(a3.x, a3.y, acc);
          }
          for (; b < kb; b++) {
            const float2 a = in_ps[b * kPsStride + lane];
            acc = __fmaf_rn(a.x, a.y, acc);
          }
        }
      } else {
        // later part of a split unit: hand the pairs over
        float2* dst = A.split.pairs + ((size_t)c_slot * n_blk + cs * kKB) * kRT;
        for (int e = lane; e < kb * kRT; e += 32) dst[e] = in_ps[(e >> 4) * kPsStride + (e & 15)];
      }
      const bool unit_end = cs + 1 == n_st;
      if (unit_end || ii == n_items) {  // this CTA's part of the unit is done
        const int n_r = unit_rows[ck];
        float* out = unit_out[ck];
        if (!c_split) {
          if (lane < n_r) out[lane] = acc;
        } else {
          const long long ub = (long long)(u_first + ck) * n_st;
          if (c_head && lane < kRT) A.split.acc[c_slot * kRT + lane] = acc;
          __threadfence();
          __syncwarp();
          const int n_parts = owner_of(A, ub + n_st - 1) - c_slot + 1;
          unsigned prev = 0;
          if (lane == 0) prev = atomicAdd(A.split.count + c_slot, 1u);
          prev = __shfl_sync(kFull, prev, 0);
          if ((int)prev == n_parts - 1) {
            // last part to arrive: finish the chain from the head's accumulator
            __threadfence();
            const int head_end = (int)(range_begin(A, c_slot + 1) - ub);  // stages held by the head
            // the pairs come through the pair buffer this warp just consumed, 16 blocks at a time,
            // loaded with every request of a refill in flight before the in-order chain reads them
            float a = lane < kRT ? __ldcg(A.split.acc + c_slot * kRT + lane) : 0.0f;
            const float2* pr = A.split.pairs + (size_t)c_slot * n_blk * kRT;
            float2* stage_buf = ps + ((ii - 1) & 1) * kKB * kPsStride;
            constexpr int kFB = kKB / 2;  // blocks per refill
            for (int b0 = head_end * kKB; b0 < n_blk; b0 += kFB) {
              const int nb = min(kFB, n_blk - b0);
              float2 tmp[kFB * kRT / 32];
#pragma unroll
              for (int e = 0; e < kFB * kRT / 32; e++)
                if (lane + 32 * e < nb * kRT) tmp[e] = __ldcg(pr + (size_t)b0 * kRT + lane + 32 * e);
#pragma unroll
              for (int e = 0; e < kFB * kRT / 32; e++)
                if (lane + 32 * e < nb * kRT) stage_buf[lane + 32 * e] = tmp[e];
              __syncwarp();
              if (lane < kRT)
                for (int b = 0; b < nb; b++) {
                  const float2 q = stage_buf[b * kRT + lane];
                  a = __fmaf_rn(q.x, q.y, a);
                }
              __syncwarp();
            }
            if (lane < n_r) out[lane] = a;
            if (lane == 0) A.split.count[c_slot] = 0u;
          }
        }
      }
      if (unit_end) {
        cs = 0;
        ck++;
        if (ii < n_items) chain_unit_begin();
      } else {
        cs++;
      }
    }
  }
  cp_async_wait<0>();
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

int g_num_sms[64] = {};

}  // namespace

cudaError_t configure_gemv_kernels() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && dev >= 0 && dev < 64)
    e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = set_max_dyn_smem(gemv_stream_kernel);
  if (e == cudaSuccess) e = configure_gemv_wg_kernel();
  return e;
}

size_t gemv_split_pairs_bytes(int max_cols) {
  return (size_t)kGemvMaxCtas * (max_cols / 32) * kRT * sizeof(float2);
}

cudaError_t launch_gemv(const Launch& L, const LinJobs& jobs, const int* skip_flag, const GemvSplit* split) {
  static const bool use_mma = [] {
    const char* v = getenv("DPUF_CUDA_GEMV");
    return v && strcmp(v, "mma") == 0;
  }();
  if (!use_mma) {
    int n_x = 0;
    const void* seen[kMaxJobs];
    for (int i = 0; i < jobs.n; i++) {
      bool dup = false;
      for (int k = 0; k < n_x; k++) dup = dup || seen[k] == jobs.j[i].act.q8;
      if (!dup) seen[n_x++] = jobs.j[i].act.q8;
    }
    if (gemv_wg_smem_bytes(jobs.j[0].w.cols, n_x) <= (size_t)kMaxDynSmem)
      return launch_gemv_wg(L, jobs, skip_flag, nullptr);
  }
  GemvArgs A;
  A.J = jobs;
  A.unit_prefix[0] = 0;
  A.n_x = 0;
  A.cols = jobs.j[0].w.cols;
  for (int i = 0; i < jobs.n; i++) {
    if (jobs.j[i].w.cols != A.cols) return cudaErrorInvalidValue;  // one K per launch
    A.unit_prefix[i + 1] = A.unit_prefix[i] + (jobs.j[i].t_end - jobs.j[i].t_begin);
    int slot = -1;
    for (int k = 0; k < i; k++)
      if (jobs.j[k].act.q8 == jobs.j[i].act.q8) slot = A.x_slot[k];
    A.x_slot[i] = slot >= 0 ? slot : A.n_x++;
  }
  A.n_units = A.unit_prefix[jobs.n];
  if (A.n_units == 0) return cudaSuccess;
  A.n_blk = A.cols / 32;
  A.n_st = (A.n_blk + kKB - 1) / kKB;
  A.items = (long long)A.n_units * A.n_st;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = (dev >= 0 && dev < 64 && g_num_sms[dev] > 0) ? g_num_sms[dev] : 148;
  const bool can_split = split && split->pairs && split->acc && split->count;
  A.whole_units = can_split ? 0 : 1;
  A.split = can_split ? *split : GemvSplit{nullptr, nullptr, nullptr};
  // Whole units: the smallest grid (up to three CTAs per SM) reaching the minimal number of
  // units per CTA.  Units are split between CTAs only when there are fewer units than SMs.
  const int max_ctas = std::min(4 * sms, kGemvMaxCtas);
  long long grid;
  if (can_split && A.n_units < sms && A.n_st > 1) {
    grid = std::min<long long>(A.items, 2LL * sms);
  } else {
    A.whole_units = 1;
    A.split = GemvSplit{nullptr, nullptr, nullptr};
    const long long per = (A.n_units + max_ctas - 1) / max_ctas;
    grid = (A.n_units + per - 1) / per;
  }
  if ((A.n_units + grid - 1) / grid + 2 > kMaxUnitsPerCta) return cudaErrorInvalidValue;
  const size_t smem = (size_t)kNS * kStage + kPsBytes + (size_t)A.n_x * (A.cols + A.n_blk * 8);
  if (smem > kMaxDynSmem) return cudaErrorInvalidValue;
  return launch_k(L, gemv_stream_kernel, dim3((unsigned)grid), dim3(kThreads), smem, A, skip_flag);
}

}  // namespace dpuf
