// ops_had_asym.cu - standalone matmul and row lookup of the reference's modes 13 (QR_HAD4_ASYM,
// 4-bit) and 14 (QR_HAD6, 6-bit) behind its exported signatures (dpuf_kernels.h:279-313,
// dpuf_avx2.c:2785-3221): the mode-12 activation prep (launch_prep: sign flip, FWHT-64, int8
// per 32 with block scale and block sum x 8), then had_asym_kernel; had_embed_kernel.
//
// Tile layout (16-byte header, then per 8-row group): n64 x [8 fp16 d | 8 fp16 m] per 64-block,
// then per 32-block 128 bytes of nibbles ordered [chunk c][row r][e] - the low nibble weighs
// x[8c+e], the high nibble x[8c+4+e] - and, for mode 14, per 32-block 64 bytes of high bit pairs
// (byte c*16 + half*8 + (r%2)*4 + e holds, at bits 2*(r/2), the pair of the low (half 0) or high
// (half 1) nibble).  Weights are asymmetric: w = d * u + m with u unsigned.
#include <algorithm>
#include <string>
#include <vector>

#include "dpuf_cuda.h"
#include "dpuf_kernels.h"
#include "engine_internal.h"
#include "kernels.cuh"

namespace dpuf {
namespace {

constexpr int kHadChunk = 256;   // tokens per prep + matmul launch pair

// One warp computes one 8-row group (rg) of tile t for token blockIdx.y; lane = 4 r + c: row r,
// chunk c (8 of the 32 columns) of every 32-block.  The block dot d_b = sum u * q is exact
// (dp4a over the lane's 4 + 4 weights, a two-step shuffle sum over the row's four lanes), as the
// reference's maddubs/madd sums are (no saturation or wrap at these ranges).  Then, per row and
// 64-block g in order (had_asym_tile_range_impl):
//   fdot = fma(d_{2g}, xs_{2g}, d_{2g+1} * xs_{2g+1})
//   acc  = fma(fdot, d_row, acc);  acc = fma(m_row, xm_s, acc)
// with xm_s = fma(xsum_{2g}, xs_{2g}, xsum_{2g+1} * xs_{2g+1}) * 0.125: the reference's scalar
// "(xsum0 * xs0 + xsum1 * xs1) * 0.125f", which its build (gcc, gnu11, -mfma) contracts.
// kG 64-blocks per batch (all their loads issued before their dots and chain steps) and kWarps
// 8-row groups per CTA; used for several tokens (shallow batches in larger CTAs: the tiles are
// re-read from L2, and more resident warps hide that better); one token runs on
// had_gemv_stream_kernel below.
template <bool kHad6, int kG, int kWarps>
__global__ void __launch_bounds__(kWarps * 32) had_asym_kernel(const uint8_t* __restrict__ tiles,
                                                                  const uint64_t* __restrict__ toff, int rows,
                                                                  int cols, int t0, int n_tiles, Act a,
                                                                  float* __restrict__ out, const int* skip) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int t = t0 + (gw >> 1), rg = gw & 1;
  if (t >= n_tiles || (skip && *skip)) return;
  const uint8_t* tp = tiles + toff[t];
  const int n_r = tp[4] | (tp[5] << 8);
  if (rg * 8 >= n_r) return;
  const int m = blockIdx.y;
  const int n_64 = cols >> 6;
  const size_t grp_bytes = kHad6 ? 416 : 288;
  const uint8_t* grp = tp + 16 + (size_t)rg * n_64 * grp_bytes;
  const uint16_t* dm = (const uint16_t*)grp;
  const uint8_t* q4 = grp + (size_t)n_64 * 32;
  const uint8_t* q2 = q4 + (size_t)n_64 * 256;
  const int r = lane >> 2, c = lane & 3, sh = 2 * (r >> 1);
  const int8_t* xq = a.q8 + (size_t)m * a.ld;
  const float* xs = a.xs + (size_t)m * (a.ld >> 5);
  const int* xm = a.xm + (size_t)m * (a.ld >> 5);
  float acc = 0.0f;
  for (int g0 = 0; g0 < n_64; g0 += kG) {
    const int ng = min(kG, n_64 - g0);
    uint32_t lo[kG][2], hi[kG][2];
    int xa[kG][2], xb[kG][2];
    uint16_t dv[kG], mv[kG];
#pragma unroll
    for (int i = 0; i < kG; i++) {
      if (i >= ng) break;
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int b = 2 * (g0 + i) + k;
        const uint32_t w = __ldg((const uint32_t*)(q4 + (size_t)b * 128 + c * 32 + r * 4));
        lo[i][k] = w & 0x0F0F0F0Fu;
        hi[i][k] = (w >> 4) & 0x0F0F0F0Fu;
        if (kHad6) {
          const uint8_t* hp = q2 + (size_t)b * 64 + c * 16 + (r & 1) * 4;
          lo[i][k] |= ((__ldg((const uint32_t*)hp) >> sh) & 0x03030303u) << 4;
          hi[i][k] |= ((__ldg((const uint32_t*)(hp + 8)) >> sh) & 0x03030303u) << 4;
        }
        const int* xw = (const int*)(xq + b * 32 + c * 8);
        xa[i][k] = xw[0];
        xb[i][k] = xw[1];
      }
      dv[i] = __ldg(dm + (g0 + i) * 16 + r);
      mv[i] = __ldg(dm + (g0 + i) * 16 + 8 + r);
    }
#pragma unroll
    for (int i = 0; i < kG; i++) {
      if (i >= ng) break;
      int d[2];
#pragma unroll
      for (int k = 0; k < 2; k++) {
        int p = __dp4a((int)lo[i][k], xa[i][k], 0);
        p = __dp4a((int)hi[i][k], xb[i][k], p);
        p += __shfl_xor_sync(kFull, p, 1);
        p += __shfl_xor_sync(kFull, p, 2);
        d[k] = p;
      }
      const int b0 = 2 * (g0 + i), b1 = b0 + 1;
      const float xs0 = xs[b0], xs1 = xs[b1];
      const float fdot = __fmaf_rn(__int2float_rn(d[0]), xs0, __fmul_rn(__int2float_rn(d[1]), xs1));
      const float xms =
          __fmul_rn(__fmaf_rn(__int2float_rn(xm[b0]), xs0, __fmul_rn(__int2float_rn(xm[b1]), xs1)), 0.125f);
      acc = __fmaf_rn(fdot, f16bits_to_f32(dv[i]), acc);
      acc = __fmaf_rn(f16bits_to_f32(mv[i]), xms, acc);
    }
  }
  if (c == 0 && rg * 8 + r < n_r) out[(size_t)m * rows + t * 16 + rg * 8 + r] = acc;
}

// One token (a GEMV), streamed: one warp per 8-row group.  The group's bytes move by bulk
// copies (scales, nibbles and, for mode 14, high pairs: three contiguous parts per stage of
// kHS 64-blocks) into a kHRing-deep ring of the warp's own, so that each warp keeps kHRing
// stages of weight bytes in flight; the lanes then compute exactly as had_asym_kernel does,
// reading the stage from shared memory (same bits).  A wait that gives up sets *err.
constexpr int kHWarps = 4, kHRing = 3, kHS = 16;
constexpr unsigned long long kHWaitNs = 2000000000ull;
template <bool kHad6>
DPUF_HD constexpr int had_stage_bytes() {
  return kHS * (32 + 256 + (kHad6 ? 128 : 0));
}

DPUF_DEV unsigned hsu32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
DPUF_DEV bool had_try(uint64_t* bar, unsigned par) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(hsu32(bar)), "r"(par)
               : "memory");
  return ok != 0;
}
DPUF_DEV unsigned long long had_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
DPUF_DEV bool had_wait(uint64_t* bar, unsigned par) {  // bounded; the timer only after a failed try
  if (had_try(bar, par)) return true;
  const unsigned long long t0 = had_timer();
  for (int it = 1;; it++) {
    if (had_try(bar, par)) return true;
    if ((it & 15) == 0 && had_timer() - t0 > kHWaitNs) return false;
  }
}
DPUF_DEV void had_bulk(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   hsu32(dst)),
               "l"(src), "r"(bytes), "r"(hsu32(bar))
               : "memory");
}

template <bool kHad6>
__global__ void __launch_bounds__(kHWarps * 32, 4) had_gemv_stream_kernel(const uint8_t* __restrict__ tiles,
                                                                        const uint64_t* __restrict__ toff, int cols,
                                                                        int t0, int n_tiles, Act a,
                                                                        float* __restrict__ out, const int* skip,
                                                                        int* err) {
  constexpr int kSt = had_stage_bytes<kHad6>();
  constexpr int kB = kHad6 ? 4 : 8;  // 64-blocks whose loads are in flight together
  static_assert(kHS % kB == 0, "batches");
  extern __shared__ __align__(128) unsigned char hsm[];
  __shared__ __align__(8) uint64_t full[kHWarps][kHRing];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (skip && *skip) return;
  const int gw = blockIdx.x * kHWarps + warp;
  const int t = t0 + (gw >> 1), rg = gw & 1;
  if (t >= n_tiles) return;  // warp-uniform from here on
  const uint8_t* tp = tiles + toff[t];
  const int n_r = tp[4] | (tp[5] << 8);
  if (rg * 8 >= n_r) return;
  const int n_64 = cols >> 6;
  const uint8_t* grp = tp + 16 + (size_t)rg * n_64 * (kHad6 ? 416 : 288);
  const uint8_t* gdm = grp;
  const uint8_t* gq4 = grp + (size_t)n_64 * 32;
  const uint8_t* gq2 = gq4 + (size_t)n_64 * 256;
  unsigned char* ring = hsm + (size_t)warp * kHRing * kSt;
  uint64_t* bar = full[warp];
  const int n_st = (n_64 + kHS - 1) / kHS;
  auto issue = [&](int st) {  // lane 0: stage st into its slot
    const int slot = st % kHRing, g0 = st * kHS, kb = min(kHS, n_64 - g0);
    unsigned char* d = ring + slot * kSt;
    const unsigned bytes = (unsigned)kb * (32u + 256u + (kHad6 ? 128u : 0u));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(hsu32(&bar[slot])), "r"(bytes)
                 : "memory");
    had_bulk(d, gdm + (size_t)g0 * 32, (unsigned)kb * 32u, &bar[slot]);
    had_bulk(d + kHS * 32, gq4 + (size_t)g0 * 256, (unsigned)kb * 256u, &bar[slot]);
    if (kHad6) had_bulk(d + kHS * 288, gq2 + (size_t)g0 * 128, (unsigned)kb * 128u, &bar[slot]);
  };
  int issued = min(kHRing, n_st);
  if (lane == 0) {
    for (int i = 0; i < kHRing; i++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(hsu32(&bar[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int st = 0; st < issued; st++) issue(st);
  }
  __syncwarp();
  const int r = lane >> 2, c = lane & 3, sh = 2 * (r >> 1);
  float acc = 0.0f;
  int st = 0;
  for (; st < n_st; st++) {
    const int slot = st % kHRing;
    const bool ok = had_wait(&bar[slot], (unsigned)((st / kHRing) & 1));
    if (__any_sync(kFull, !ok)) break;
    const unsigned char* d = ring + slot * kSt;
    const uint16_t* sdm = (const uint16_t*)d;
    const uint8_t* sq4 = d + kHS * 32;
    const uint8_t* sq2 = d + kHS * 288;
    const int g0 = st * kHS, kb = min(kHS, n_64 - g0);
    // kB 64-blocks at a time: every load first, then the exact dots and per-block terms, then
    // the row chain in block order (the only serial part)
    for (int i0 = 0; i0 < kb; i0 += kB) {
      uint32_t lo[kB][2], hi[kB][2];
      int xa[kB][2], xb[kB][2];
      float2 xs[kB];
      int2 xm[kB];
      uint16_t dv[kB], mv[kB];
#pragma unroll
      for (int j = 0; j < kB; j++) {
        const int i = min(i0 + j, kb - 1), g = g0 + i;  // a batch past kb repeats the last block, unused
#pragma unroll
        for (int k = 0; k < 2; k++) {
          const uint32_t w = *(const uint32_t*)(sq4 + (2 * i + k) * 128 + c * 32 + r * 4);
          lo[j][k] = w & 0x0F0F0F0Fu;
          hi[j][k] = (w >> 4) & 0x0F0F0F0Fu;
          if (kHad6) {
            const uint8_t* hp = sq2 + (2 * i + k) * 64 + c * 16 + (r & 1) * 4;
            lo[j][k] |= ((*(const uint32_t*)hp >> sh) & 0x03030303u) << 4;
            hi[j][k] |= ((*(const uint32_t*)(hp + 8) >> sh) & 0x03030303u) << 4;
          }
          const int2 xw = *(const int2*)(a.q8 + (2 * g + k) * 32 + c * 8);
          xa[j][k] = xw.x;
          xb[j][k] = xw.y;
        }
        xs[j] = *(const float2*)(a.xs + 2 * g);
        xm[j] = *(const int2*)(a.xm + 2 * g);
        dv[j] = sdm[i * 16 + r];
        mv[j] = sdm[i * 16 + 8 + r];
      }
      float fdot[kB], xms[kB];
#pragma unroll
      for (int j = 0; j < kB; j++) {
        int dd[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
          int p = __dp4a((int)lo[j][k], xa[j][k], 0);
          p = __dp4a((int)hi[j][k], xb[j][k], p);
          p += __shfl_xor_sync(kFull, p, 1);
          p += __shfl_xor_sync(kFull, p, 2);
          dd[k] = p;
        }
        fdot[j] = __fmaf_rn(__int2float_rn(dd[0]), xs[j].x, __fmul_rn(__int2float_rn(dd[1]), xs[j].y));
        xms[j] = __fmul_rn(__fmaf_rn(__int2float_rn(xm[j].x), xs[j].x, __fmul_rn(__int2float_rn(xm[j].y), xs[j].y)),
                           0.125f);
      }
#pragma unroll
      for (int j = 0; j < kB; j++)
        if (i0 + j < kb) {
          acc = __fmaf_rn(fdot[j], f16bits_to_f32(dv[j]), acc);
          acc = __fmaf_rn(f16bits_to_f32(mv[j]), xms[j], acc);
        }
    }
    __syncwarp();  // every lane is done with the slot
    if (lane == 0 && st + kHRing < n_st) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic reads before the copy's writes
      issue(st + kHRing);
      issued = st + kHRing + 1;
    }
  }
  if (st < n_st) {  // a wait gave up: report it, and let the copies in flight land before exiting
    if (lane == 0) {
      atomicOr(err, 1);
      issued = min(n_st, st + kHRing);
      for (int q = st; q < issued; q++) had_wait(&bar[q % kHRing], (unsigned)((q / kHRing) & 1));
    }
    return;
  }
  if (c == 0 && rg * 8 + r < n_r) out[t * 16 + rg * 8 + r] = acc;
}

// Row lookup (embed_qr_had_asym_impl, dpuf_avx2.c:3146-3221): one warp per 64-column chunk of
// one token's row.  Lane l dequantises columns c0+l and c0+32+l, v = u * d + m (u * d is exact:
// u < 64, d an fp16), then the chunk's FWHT-64 (fwht64_warp, the mode-12 lookup's) and the
// column signs.  Row ids were checked against the tiles on the host.
template <bool kHad6>
__global__ void __launch_bounds__(256) had_embed_kernel(const uint8_t* __restrict__ tiles,
                                                        const uint64_t* __restrict__ toff, int cols,
                                                        const int32_t* __restrict__ ids,
                                                        const uint8_t* __restrict__ signs, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int ch = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (ch * 64 >= cols) return;
  const int tok = blockIdx.y;
  const int row = ids[tok], t = row >> 4, lr = row & 15, rg = lr >> 3, ri = lr & 7;
  const int n_64 = cols >> 6;
  const uint8_t* grp = tiles + toff[t] + 16 + (size_t)rg * n_64 * (kHad6 ? 416 : 288);
  const uint16_t* dm = (const uint16_t*)grp;
  const uint8_t* q4 = grp + (size_t)n_64 * 32;
  const uint8_t* q2 = q4 + (size_t)n_64 * 256;
  const float wd = f16bits_to_f32(dm[ch * 16 + ri]), wm = f16bits_to_f32(dm[ch * 16 + 8 + ri]);
  float v[2];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int b = 2 * ch + h, p = lane, c = p >> 3, e = p & 3, high = (p >> 2) & 1;
    const uint8_t byte = q4[(size_t)b * 128 + c * 32 + ri * 4 + e];
    int u = high ? (byte >> 4) : (byte & 15);
    if (kHad6) u |= ((q2[(size_t)b * 64 + c * 16 + high * 8 + (ri & 1) * 4 + e] >> (2 * (ri >> 1))) & 3) << 4;
    v[h] = __fadd_rn(__fmul_rn((float)u, wd), wm);
  }
  fwht64_warp(v[0], v[1], lane);
  const int ca = ch * 64 + lane, cb = ca + 32;
  if (signs) {
    if ((signs[ca >> 3] >> (ca & 7)) & 1) v[0] = -v[0];
    if ((signs[cb >> 3] >> (cb & 7)) & 1) v[1] = -v[1];
  }
  out[(size_t)tok * cols + ca] = v[0];
  out[(size_t)tok * cols + cb] = v[1];
}

// A mode-13/14 matrix in device memory: its tile span, tile offsets relative to it, signs.
struct HadMat {
  unsigned char* mem = nullptr;
  const uint64_t* toff = nullptr;
  const uint8_t* signs = nullptr;
  int rows = 0, cols = 0, n_tiles = 0, had6 = 0;
  int t0 = 0;                 // the launches cover tiles [t0, n_tiles)
  const int* skip = nullptr;  // device flag: when set at launch time, the launch does nothing
  int* err = nullptr;         // device word set when a bounded wait of the one-token kernel gives up
};

bool had_fail(const char* where, cudaError_t e) {
  set_error(std::string(where) + ": " + cudaGetErrorString(e));
  return false;
}

// Checks the descriptor (every tile's rows inside [0, rows), 16-byte aligned offsets) and
// uploads tiles [0, n_tiles); the span end comes from the last bytes each tile's groups use.
bool had_upload(HadMat& h, int had6, int rows, int cols, int n_tiles, const uint8_t* base, const uint64_t* toff,
                const uint8_t* signs) {
  if (rows <= 0 || cols <= 0 || cols % 64 != 0 || n_tiles <= 0 || !base || !toff) {
    set_error("bad mode-13/14 descriptor");
    return false;
  }
  const uint64_t grp = (uint64_t)(cols / 64) * (had6 ? 416 : 288);
  uint64_t lo = toff[0], hi = 0;
  for (int t = 0; t < n_tiles; t++) {
    const uint8_t* tp = base + toff[t];
    const int n_r = tp[4] | (tp[5] << 8);
    if (toff[t] % 16 != 0 || n_r < 1 || n_r > kTileRows || (int64_t)t * kTileRows + n_r > rows) {
      set_error("mode-13/14 tile outside the matrix (row count or alignment)");
      return false;
    }
    lo = std::min<uint64_t>(lo, toff[t]);
    hi = std::max<uint64_t>(hi, toff[t] + 16 + (uint64_t)((n_r + 7) / 8) * grp);
  }
  const size_t span = (size_t)(hi - lo);
  const size_t off_toff = (span + 255) & ~(size_t)255;
  const size_t off_sign = (off_toff + (size_t)n_tiles * 8 + 255) & ~(size_t)255;
  const size_t total = off_sign + (size_t)cols / 8;
  cudaError_t e;
  if ((e = cudaMalloc(&h.mem, total)) != cudaSuccess) return had_fail("cudaMalloc", e);
  if ((e = cudaMemcpy(h.mem, base + lo, span, cudaMemcpyHostToDevice)) != cudaSuccess) return had_fail("upload", e);
  std::string rel((size_t)n_tiles * 8, '\0');
  uint64_t* rp = (uint64_t*)&rel[0];
  for (int t = 0; t < n_tiles; t++) rp[t] = toff[t] - lo;
  if ((e = cudaMemcpy(h.mem + off_toff, rp, (size_t)n_tiles * 8, cudaMemcpyHostToDevice)) != cudaSuccess)
    return had_fail("upload", e);
  if (signs && (e = cudaMemcpy(h.mem + off_sign, signs, (size_t)cols / 8, cudaMemcpyHostToDevice)) != cudaSuccess)
    return had_fail("upload", e);
  h.toff = (const uint64_t*)(h.mem + off_toff);
  h.signs = signs ? h.mem + off_sign : nullptr;
  h.rows = rows;
  h.cols = cols;
  h.n_tiles = n_tiles;
  h.had6 = had6;
  return true;
}

template <int kG, int kWarps>
void launch_had_t(cudaStream_t s, const HadMat& h, const Act& a, int M, float* y) {
  const dim3 grid((2 * (h.n_tiles - h.t0) + kWarps - 1) / kWarps, M);
  if (h.had6)
    had_asym_kernel<true, kG, kWarps>
        <<<grid, kWarps * 32, 0, s>>>(h.mem, h.toff, h.rows, h.cols, h.t0, h.n_tiles, a, y, h.skip);
  else
    had_asym_kernel<false, kG, kWarps>
        <<<grid, kWarps * 32, 0, s>>>(h.mem, h.toff, h.rows, h.cols, h.t0, h.n_tiles, a, y, h.skip);
}

cudaError_t configure_had_kernels() {
  cudaError_t e = cudaFuncSetAttribute(had_gemv_stream_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kHWarps * kHRing * had_stage_bytes<false>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(had_gemv_stream_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kHWarps * kHRing * had_stage_bytes<true>());
  return e;
}

// The launches of the matmul; the one-token kernel's shared-memory attribute must be set
// (configure_had_kernels) on the current device first.
cudaError_t launch_had_configured(cudaStream_t s, const HadMat& h, const Act& a, int M, float* y) {
  if (h.n_tiles <= h.t0) return cudaSuccess;
  if (M == 1) {
    if (!h.err) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((2 * (h.n_tiles - h.t0) + kHWarps - 1) / kHWarps));
    if (h.had6)
      had_gemv_stream_kernel<true><<<grid, kHWarps * 32, kHWarps * kHRing * had_stage_bytes<true>(), s>>>(
          h.mem, h.toff, h.cols, h.t0, h.n_tiles, a, y, h.skip, h.err);
    else
      had_gemv_stream_kernel<false><<<grid, kHWarps * 32, kHWarps * kHRing * had_stage_bytes<false>(), s>>>(
          h.mem, h.toff, h.cols, h.t0, h.n_tiles, a, y, h.skip, h.err);
  } else {
    launch_had_t<2, 8>(s, h, a, M, y);
  }
  return cudaGetLastError();
}

cudaError_t launch_had(cudaStream_t s, const HadMat& h, const Act& a, int M, float* y) {
  static thread_local int configured = -1;  // per host thread: the device it was done for
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    if (cudaError_t e = configure_had_kernels()) return e;
    configured = dev;
  }
  return launch_had_configured(s, h, a, M, y);
}

// Activation buffers for kHadChunk tokens.
struct HadAct {
  Act a{};
  int* err = nullptr;  // the one-token kernel's error word
  bool alloc(int cols) {
    cudaError_t e;
    if ((e = cudaMalloc(&err, 4)) != cudaSuccess || (e = cudaMemset(err, 0, 4)) != cudaSuccess)
      return had_fail("cudaMalloc", e);
    if ((e = cudaMalloc(&a.q8, (size_t)kHadChunk * cols)) != cudaSuccess) return had_fail("cudaMalloc", e);
    if ((e = cudaMalloc(&a.xs, (size_t)kHadChunk * (cols / 32) * 4)) != cudaSuccess) return had_fail("cudaMalloc", e);
    if ((e = cudaMalloc(&a.xm, (size_t)kHadChunk * (cols / 32) * 4)) != cudaSuccess) return had_fail("cudaMalloc", e);
    a.ld = cols;
    return true;
  }
  // after the stream is synchronised: did a bounded wait give up?
  bool timed_out() {
    int v = 0;
    return cudaMemcpy(&v, err, 4, cudaMemcpyDeviceToHost) == cudaSuccess && v != 0;
  }
  ~HadAct() {
    cudaFree(err);
    cudaFree(a.q8);
    cudaFree(a.xs);
    cudaFree(a.xm);
  }
};

// y = W x for M tokens (device pointers), kHadChunk tokens per prep + matmul pair.
bool had_matmul_dev(HadMat h, HadAct& act, int M, const float* x, float* y, cudaStream_t s) {
  const Launch L{s, false};
  h.err = act.err;
  for (int m0 = 0; m0 < M; m0 += kHadChunk) {
    const int mc = std::min(kHadChunk, M - m0);
    cudaError_t e = launch_prep(L, x + (size_t)m0 * h.cols, h.cols, mc, h.cols, h.signs, act.a);
    if (e != cudaSuccess) return had_fail("prep", e);
    if ((e = launch_had(s, h, act.a, mc, y + (size_t)m0 * h.rows)) != cudaSuccess) return had_fail("matmul", e);
  }
  return true;
}

// Reference signature, host in / host out, synchronous.
void had_matmul_host(int had6, int32_t M, int32_t rows, int32_t cols, int32_t n_tiles, const float* x_in,
                     const uint8_t* base, const uint64_t* toff, const uint8_t* signs, float* out) {
  set_error("");
  if (M <= 0 || !x_in || !out) return;
  HadMat h;
  HadAct act;
  float *dx = nullptr, *dy = nullptr;
  if (had_upload(h, had6, rows, cols, n_tiles, base, toff, signs) && act.alloc(cols) &&
      cudaMalloc(&dx, (size_t)M * cols * 4) == cudaSuccess && cudaMalloc(&dy, (size_t)M * rows * 4) == cudaSuccess &&
      cudaMemcpy(dx, x_in, (size_t)M * cols * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
      had_matmul_dev(h, act, M, dx, dy, nullptr)) {
    const cudaError_t e = cudaMemcpy(out, dy, (size_t)M * rows * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) set_error(cudaGetErrorString(e));
    else if (act.timed_out()) set_error("mode-13/14 GEMV: a bounded wait for weight bytes gave up");
  }
  cudaFree(dx);
  cudaFree(dy);
  cudaFree(h.mem);
}

// Reference signature: rows are looked up by id; the tiles up to the largest id are uploaded,
// and an id whose row is not in its tile is rejected (the reference would read past it).
void had_embed_host(int had6, int32_t n_tokens, int32_t cols, const int32_t* ids, const uint8_t* base,
                    const uint64_t* toff, const uint8_t* signs, float* out) {
  set_error("");
  if (n_tokens <= 0 || !ids || !out || !base || !toff) return;
  int32_t max_id = 0;
  for (int i = 0; i < n_tokens; i++) {
    const int32_t r = ids[i];
    if (r < 0) {
      set_error("negative token id");
      return;
    }
    const uint8_t* tp = base + toff[r >> 4];
    if ((r & 15) >= (tp[4] | (tp[5] << 8))) {
      set_error("token id beyond its tile's rows");
      return;
    }
    max_id = std::max(max_id, r);
  }
  const int n_tiles = max_id / kTileRows + 1;
  HadMat h;
  int32_t* dids = nullptr;
  float* dy = nullptr;
  if (had_upload(h, had6, n_tiles * kTileRows, cols, n_tiles, base, toff, signs) &&
      cudaMalloc(&dids, (size_t)n_tokens * 4) == cudaSuccess &&
      cudaMalloc(&dy, (size_t)n_tokens * cols * 4) == cudaSuccess &&
      cudaMemcpy(dids, ids, (size_t)n_tokens * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
    for (int m0 = 0; m0 < n_tokens; m0 += 65535) {
      const int mc = std::min(65535, n_tokens - m0);
      const dim3 grid((cols / 64 + 7) / 8, mc);
      if (had6)
        had_embed_kernel<true><<<grid, 256>>>(h.mem, h.toff, cols, dids + m0, h.signs, dy + (size_t)m0 * cols);
      else
        had_embed_kernel<false><<<grid, 256>>>(h.mem, h.toff, cols, dids + m0, h.signs, dy + (size_t)m0 * cols);
    }
    const cudaError_t e = cudaMemcpy(out, dy, (size_t)n_tokens * cols * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) set_error(cudaGetErrorString(e));
  }
  cudaFree(dids);
  cudaFree(dy);
  cudaFree(h.mem);
}

}  // namespace

// ---- engine layers in modes 13 / 14 (the per-step path; the engine configures the kernels at
// create, so these launch without touching function attributes, e.g. during a graph capture)
cudaError_t configure_had_engine_kernels() { return configure_had_kernels(); }

cudaError_t launch_had_w(cudaStream_t s, const W12& w, const Act& a, int M, float* y, int ldo, int t_begin,
                         int t_end, const int* skip, int* err) {
  HadMat h;
  h.t0 = t_begin;
  h.skip = skip;
  h.err = err;
  h.mem = const_cast<unsigned char*>(w.tiles);
  h.toff = w.toff;
  h.signs = w.signs;
  h.rows = ldo;  // the kernels use it as the output row stride
  h.cols = w.cols;
  h.n_tiles = t_end;
  h.had6 = w.mode == 14 ? 1 : 0;
  return launch_had_configured(s, h, a, M, y);
}

cudaError_t launch_had_embed_w(cudaStream_t s, const W12& w, const int32_t* ids, int M, float* out) {
  const dim3 grid((w.cols / 64 + 7) / 8, M);
  if (w.mode == 14)
    had_embed_kernel<true><<<grid, 256, 0, s>>>(w.tiles, w.toff, w.cols, ids, w.signs, out);
  else
    had_embed_kernel<false><<<grid, 256, 0, s>>>(w.tiles, w.toff, w.cols, ids, w.signs, out);
  return cudaGetLastError();
}

}  // namespace dpuf

extern "C" {

DPUF_EXPORT void dpuf_embed_qr_had4_asym_f32(int32_t n_tokens, int32_t cols, const int32_t* token_ids,
                                             const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                             const uint8_t* sign_bits, float* out) {
  dpuf::had_embed_host(0, n_tokens, cols, token_ids, tensor_base, tile_offsets, sign_bits, out);
}

DPUF_EXPORT void dpuf_embed_qr_had6_f32(int32_t n_tokens, int32_t cols, const int32_t* token_ids,
                                        const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                        const uint8_t* sign_bits, float* out) {
  dpuf::had_embed_host(1, n_tokens, cols, token_ids, tensor_base, tile_offsets, sign_bits, out);
}

DPUF_EXPORT void dpuf_matmul_qr_had4_asym_f32(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                              const float* x_in, const uint8_t* tensor_base,
                                              const uint64_t* tile_offsets, const uint8_t* sign_bits, float* out) {
  dpuf::had_matmul_host(0, M, rows, cols, n_tiles, x_in, tensor_base, tile_offsets, sign_bits, out);
}

DPUF_EXPORT void dpuf_matmul_qr_had6_f32(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles, const float* x_in,
                                         const uint8_t* tensor_base, const uint64_t* tile_offsets,
                                         const uint8_t* sign_bits, float* out) {
  dpuf::had_matmul_host(1, M, rows, cols, n_tiles, x_in, tensor_base, tile_offsets, sign_bits, out);
}

DPUF_EXPORT int32_t dpuf_cuda_had_asym_timed(int32_t mode, int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                             const float* x_in, const uint8_t* tensor_base,
                                             const uint64_t* tile_offsets, const uint8_t* sign_bits,
                                             int32_t n_copies, int32_t reps, float* ms_per_matmul) {
  using namespace dpuf;
  set_error("");
  if ((mode != 13 && mode != 14) || M <= 0 || M > kHadChunk || !x_in || n_copies <= 0 || n_copies > 64 ||
      reps <= 0 || !ms_per_matmul) {
    set_error("bad arguments");
    return -1;
  }
  std::vector<HadMat> hs((size_t)n_copies);
  HadAct act;
  float *dx = nullptr, *dy = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int32_t rc = -4;
  bool ok = act.alloc(cols) && cudaMalloc(&dx, (size_t)M * cols * 4) == cudaSuccess &&
            cudaMalloc(&dy, (size_t)M * rows * 4) == cudaSuccess &&
            cudaMemcpy(dx, x_in, (size_t)M * cols * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
  for (int i = 0; ok && i < n_copies; i++) {
    ok = had_upload(hs[i], mode == 14, rows, cols, n_tiles, tensor_base, tile_offsets, sign_bits);
    hs[i].err = act.err;
  }
  if (ok) ok = launch_prep(Launch{nullptr, false}, dx, cols, M, cols, hs[0].signs, act.a) == cudaSuccess;
  for (int i = 0; ok && i < n_copies; i++) ok = launch_had(nullptr, hs[i], act.a, M, dy) == cudaSuccess;  // warm-up
  if (ok) {
    cudaEventRecord(e0);
    for (int k = 0; k < reps; k++) launch_had(nullptr, hs[k % n_copies], act.a, M, dy);
    cudaEventRecord(e1);
    float ms = 0.0f;
    if (cudaEventSynchronize(e1) == cudaSuccess && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess &&
        cudaGetLastError() == cudaSuccess) {
      *ms_per_matmul = ms / reps;
      rc = 0;
      if (act.timed_out()) {
        set_error("mode-13/14 GEMV: a bounded wait for weight bytes gave up");
        rc = -6;
      }
    }
  }
  if (ok && rc == -4) set_error("CUDA error in the timed mode-13/14 matmul");
  for (auto& h : hs) cudaFree(h.mem);
  cudaFree(dx);
  cudaFree(dy);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  return rc;
}

}  // extern "C"
