// common.cuh - shared device helpers of the DPUF B200 engine.
//
// Bit-exactness rules used throughout (the reference is x86 AVX2 fp32 code):
//   * every file is compiled with --fmad=false: a*b+c is never contracted; the reference's
//     fused multiply-adds are written as explicit __fmaf_rn;
//   * division and square root are IEEE round-to-nearest (__fdiv_rn, __fsqrt_rn);
//   * AVX2 8-lane reductions are reproduced lane by lane: "lane" j of a reduction owns
//     elements j, j+8, j+16, ... and the horizontal sums use the reference's two trees
//       split  ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))   eng_hsum256_ps (dpuf_engine.c:37-46)
//       pairs  ((l0+l1)+(l2+l3)) + ((l4+l5)+(l6+l7))   hsum4_256_ps   (dpuf_engine.c:318-323)
//     (float addition is commutative bit-for-bit, so a butterfly shuffle tree that combines
//     the same pairs in the same grouping gives identical bits).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define DPUF_DEV __device__ __forceinline__
#define DPUF_HD __host__ __device__ __forceinline__

namespace dpuf {

constexpr int kTileRows = 16;      // rows per container tile
constexpr int kMaxBatch = 256;     // DPUF_ENGINE_MAX_BATCH (dpuf_engine.c:35)
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxDynSmem = 200 * 1024;  // largest dynamic shared memory a launch here asks for

// One mode-12 weight matrix resident in device memory, container layout unchanged:
// tile t starts at tiles + toff[t]; 16-byte header; per 8-row group g:
//   fp16 scales [n_blk][8] then nibbles [n_blk][chunk c][row ri][k], byte = u(8c+k) | u(8c+4+k)<<4
struct W12 {
  const uint8_t* tiles;
  const uint64_t* toff;
  const uint8_t* signs;  // cols/8 bytes, bit k of byte j = column 8j+k negated
  int rows, cols, n_tiles;
  int mode = 12;         // 12 (QR_HAD4_PACKED); 13 / 14 (QR_HAD4_ASYM / QR_HAD6) on the per-step path
  const uint8_t* x8 = nullptr;  // expanded copy for the tensor-core GEMM (kernels_gemm_tc.cu), or null
};

// Activation after prep (dpuf_prep_had4_packed_slab plain layout, dpuf_avx2.c:2364-2449):
// q8 [M][cols] int8, xs [M][cols/32] block scale amax/127, xm [M][cols/32] = 8 * sum(q).
struct Act {
  int8_t* q8;
  float* xs;
  int32_t* xm;
  int ld;  // row stride (elements) of q8; xs/xm use ld/32
};

// glibc expf reproduction: dpuf_exp_d rounded to float, corrected by an exception table of
// the inputs where glibc's expf differs, held as an open-addressing hash: slot i holds
// (input bits, glibc output bits), empty slots hold kExpfEmpty; a key's probe sequence starts
// at expf_hash(key) & mask and is at most max_probe slots long.
constexpr uint32_t kExpfEmpty = 0xFFFFFFFFu;  // a NaN pattern: never an exception key
struct ExpfTable {
  const uint2* slots;
  uint32_t mask;
  int max_probe;
};
DPUF_HD uint32_t expf_hash(uint32_t key) { return (key * 2654435761u) ^ (key >> 15); }

// Raises a kernel's dynamic shared-memory limit to the device's opt-in maximum minus the
// kernel's static shared memory.
template <typename F>
inline cudaError_t set_max_dyn_smem(F* fn) {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes a;
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, (const void*)fn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)a.sharedSizeBytes);
  return e;
}

DPUF_DEV float f16bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---------------------------------------------------------------- reductions
DPUF_DEV float shfl_xor(float v, int m) { return __shfl_xor_sync(kFull, v, m); }

// Lanes 8q..8q+7 of a warp hold the 8 "AVX lanes" l0..l7 of one reduction each.
DPUF_DEV float tree8_split(float v) {
  v = v + shfl_xor(v, 4);  // l0+l4, l1+l5, ...
  v = v + shfl_xor(v, 1);  // (l0+l4)+(l1+l5), (l2+l6)+(l3+l7)
  v = v + shfl_xor(v, 2);
  return v;
}
DPUF_DEV float tree8_pairs(float v) {
  v = v + shfl_xor(v, 1);  // l0+l1, l2+l3, ...
  v = v + shfl_xor(v, 2);  // (l0+l1)+(l2+l3)
  v = v + shfl_xor(v, 4);
  return v;
}
DPUF_HD float tree8_split_arr(const float* l) {
  float a0 = l[0] + l[4], a1 = l[1] + l[5], a2 = l[2] + l[6], a3 = l[3] + l[7];
  return (a0 + a1) + (a2 + a3);
}

DPUF_DEV float warp_max(float v) {
#pragma unroll
  for (int m = 16; m; m >>= 1) v = fmaxf(v, shfl_xor(v, m));
  return v;
}
DPUF_DEV int warp_sum_i(int v) {
#pragma unroll
  for (int m = 16; m; m >>= 1) v += __shfl_xor_sync(kFull, v, m);
  return v;
}

// _mm_max_ps / _mm_min_ps semantics for non-NaN inputs.
DPUF_DEV float max_ps(float a, float b) { return (a > b) ? a : b; }
DPUF_DEV float min_ps(float a, float b) { return (a < b) ? a : b; }

// ---------------------------------------------------------------- the reference's exp
// eng_avx2_exp_ps (dpuf_engine.c:297-316), one lane: clamp to [-45, 45], Cody-Waite split
// of ln2, degree-5 polynomial by fma, scale by 2^n.
DPUF_DEV float exp_poly(float x) {
  x = max_ps(-45.0f, min_ps(x, 45.0f));
  float fx = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-fx, 0.693359375f, x);
  r = __fmaf_rn(-fx, -2.12194440e-4f, r);
  float p = 1.9875691500e-4f;
  p = __fmaf_rn(p, r, 1.3981999507e-3f);
  p = __fmaf_rn(p, r, 8.3334519073e-3f);
  p = __fmaf_rn(p, r, 4.1665795894e-2f);
  p = __fmaf_rn(p, r, 1.6666665459e-1f);
  p = __fmaf_rn(p, r, 5.0000001201e-1f);
  float r2 = __fmul_rn(r, r);
  float er = __fadd_rn(__fmaf_rn(p, r2, r), 1.0f);
  int n = __float2int_rn(fx);
  return __fmul_rn(er, __int_as_float((n + 127) << 23));
}

// ---------------------------------------------------------------- glibc-compatible expf
// exp(x) in double: k = rint(x/ln2), r = x - k*ln2 (two-part ln2, exact first product),
// Taylor polynomial to degree 13 by Horner/fma, times 2^k.  Identical bits on host and
// device (IEEE double, explicit fma); used only to build/apply the expf exception table.
DPUF_HD double dpuf_exp_d(double x) {
  if (!(x == x)) return x;
  if (x < -160.0) return 0.0;
  if (x > 100.0) return __builtin_huge_val();
  double k = rint(x * 0x1.71547652b82fep+0);
  double r = fma(-k, 0x1.62e42fefa38p-1, x);
  r = fma(-k, 0x1.ef35793c7673p-45, r);
  double p = 0x1.6124613a86d09p-33;
  p = fma(p, r, 0x1.1eed8eff8d898p-29);
  p = fma(p, r, 0x1.ae64567f544e4p-26);
  p = fma(p, r, 0x1.27e4fb7789f5cp-22);
  p = fma(p, r, 0x1.71de3a556c734p-19);
  p = fma(p, r, 0x1.a01a01a01a01ap-16);
  p = fma(p, r, 0x1.a01a01a01a01ap-13);
  p = fma(p, r, 0x1.6c16c16c16c17p-10);
  p = fma(p, r, 0x1.1111111111111p-7);
  p = fma(p, r, 0x1.5555555555555p-5);
  p = fma(p, r, 0x1.5555555555555p-3);
  p = fma(p, r, 0x1.0000000000000p-1);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return ldexp(p, (int)k);
}

DPUF_DEV float glibc_expf(float x, const ExpfTable& t) {
  const uint32_t key = __float_as_uint(x);
  uint32_t i = expf_hash(key) & t.mask;
  for (int p = 0; p < t.max_probe; p++) {
    const uint2 e = t.slots[i];
    if (e.x == key) return __uint_as_float(e.y);
    if (e.x == kExpfEmpty) break;
    i = (i + 1) & t.mask;
  }
  return __double2float_rn(dpuf_exp_d((double)x));
}

// ---------------------------------------------------------------- mode-12 activation prep
// One warp rotates and quantises one 64-column chunk.  Lane l holds columns c0+l (a) and
// c0+32+l (b), already sign-flipped.  Butterfly strides 1,2,4,8,16 across lanes, 32 within
// the lane, then x0.125 (fwht64_block_f32, dpuf_avx2.c:724-772; ascending strides).
DPUF_DEV void fwht64_warp(float& a, float& b, int lane) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
    float pa = shfl_xor(a, h), pb = shfl_xor(b, h);
    if (lane & h) { a = __fsub_rn(pa, a); b = __fsub_rn(pb, b); }
    else          { a = __fadd_rn(a, pa); b = __fadd_rn(b, pb); }
  }
  float s = __fadd_rn(a, b), d = __fsub_rn(a, b);
  a = __fmul_rn(s, 0.125f);
  b = __fmul_rn(d, 0.125f);
}

// Quantises one 32-column block held one value per lane (dpuf_avx2.c:2397-2431):
// amax <= 1e-4 -> zeros; else xs = amax/127, q = clamp(rint(v * (127/amax)), -127, 127),
// xm = 8 * sum(q).
DPUF_DEV void quant32_warp(float v, int lane, int8_t* q_out, float* xs_out, int32_t* xm_out) {
  float amax = warp_max(fabsf(v));
  int q = 0;
  float xs = 0.0f;
  if (amax > 1e-4f) {
    xs = __fdiv_rn(amax, 127.0f);
    float inv = (amax > 1e-12f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    q = __float2int_rn(__fmul_rn(v, inv));
    q = max(-127, min(127, q));
  }
  int s = warp_sum_i(q);
  q_out[lane] = (int8_t)q;
  if (lane == 0) {
    *xs_out = xs;
    *xm_out = s * 8;
  }
}

DPUF_DEV float apply_sign(float v, const uint8_t* signs, int col) {
  return ((signs[col >> 3] >> (col & 7)) & 1) ? -v : v;
}

// Full prep of one 64-chunk by a warp: sign, FWHT-64, two quantised 32-blocks.
DPUF_DEV void prep_chunk_warp(float a, float b, const uint8_t* signs, int c0, int lane, int8_t* q8, float* xs,
                              int32_t* xm) {
  if (signs) {
    a = apply_sign(a, signs, c0 + lane);
    b = apply_sign(b, signs, c0 + 32 + lane);
  }
  fwht64_warp(a, b, lane);
  int blk = c0 >> 5;
  quant32_warp(a, lane, q8 + c0, xs + blk, xm + blk);
  quant32_warp(b, lane, q8 + c0 + 32, xs + blk + 1, xm + blk + 1);
}

}  // namespace dpuf
