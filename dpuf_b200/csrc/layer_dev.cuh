// layer_dev.cuh - per-layer device math shared by the per-step kernels and the persistent
// decode kernel, so both paths produce the same bits.  Every function restates one piece of
// the reference's fp32 operation order (dpuf_engine.c, cited per function).
#pragma once
#include "common.cuh"

namespace dpuf {

// ------------------------------------------------------------------ RMSNorm
// add_and_rms_norm_f32 / rms_norm_f32 (dpuf_engine.c:225-272): "AVX lane" j accumulates
// fma(s_i, s_i, .) over i = j, j+8, ... < (n & ~7) in order.
DPUF_DEV float sumsq_lane(const float* S, int n8, int j) {
  float acc = 0.0f;
  int i = j;
  for (; i + 56 < n8; i += 64) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = S[i + 8 * u];
#pragma unroll
    for (int u = 0; u < 8; u++) acc = __fmaf_rn(v[u], v[u], acc);
  }
  for (; i < n8; i += 8) acc = __fmaf_rn(S[i], S[i], acc);
  return acc;
}

// The same chain (identical operation order), software-pipelined: the next 32 values are loaded
// while the current 32 go through the fma chain, whose latency then bounds the loop.
DPUF_DEV float sumsq_lane32(const float* S, int n8, int j) {
  float acc = 0.0f;
  int i = j;
  if (i + 248 < n8) {
    float v[32];
#pragma unroll
    for (int u = 0; u < 32; u++) v[u] = S[i + 8 * u];
    for (; i + 248 < n8; i += 256) {
      const bool more = i + 256 + 248 < n8;
      float nv[32];
#pragma unroll
      for (int u = 0; u < 32; u++) nv[u] = more ? S[i + 256 + 8 * u] : 0.0f;
#pragma unroll
      for (int u = 0; u < 32; u++) acc = __fmaf_rn(v[u], v[u], acc);
#pragma unroll
      for (int u = 0; u < 32; u++) v[u] = nv[u];
    }
  }
  for (; i < n8; i += 8) acc = __fmaf_rn(S[i], S[i], acc);
  return acc;
}

// inv = 1 / sqrt(ss / n + eps) with ss = split tree of the eight lane sums, then the n % 8
// tail added in order.
DPUF_DEV float rms_inv(const float* lanes, const float* S, int n, float eps) {
  float ss = tree8_split_arr(lanes);
  for (int i = n & ~7; i < n; i++) ss = __fadd_rn(ss, __fmul_rn(S[i], S[i]));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// ------------------------------------------------------------------ QK-norm + NeoX RoPE
// One warp, one head vector s[hd] in shared memory, in place (dpuf_engine.c:1788-1822):
// RMSNorm over hd with gain nw (when nw != null), then apply_rope_neox_f32
// (dpuf_engine.c:274-295): for j < half & ~7, x1*c - x2*s and x2*c + x1*s as fused
// multiply-subtract/add of the rounded cross product; the tail j uses separate products.
DPUF_DEV void qk_norm_rope_warp(float* s, const float* nw, float eps, int hd, const float* cp, const float* sp,
                                int lane) {
  if (nw) {
    const int hd8 = hd & ~7;
    float acc = 0.0f;
    if (lane < 8)
      for (int i = lane; i < hd8; i += 8) acc = __fmaf_rn(s[i], s[i], acc);
    float ss = tree8_split(acc);  // lanes 0..7 hold the tree result
    ss = __shfl_sync(kFull, ss, 0);
    for (int i = hd8; i < hd; i++) ss = __fadd_rn(ss, __fmul_rn(s[i], s[i]));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
    __syncwarp();
    for (int i = lane; i < hd; i += 32) s[i] = __fmul_rn(__fmul_rn(s[i], inv), nw[i]);
    __syncwarp();
  }
  const int half = hd >> 1, half8 = half & ~7;
  for (int j = lane; j < half; j += 32) {
    const float x1 = s[j], x2 = s[j + half], c = cp[j], sn = sp[j];
    float o1, o2;
    if (j < half8) {
      o1 = __fmaf_rn(x1, c, -__fmul_rn(x2, sn));
      o2 = __fmaf_rn(x2, c, __fmul_rn(x1, sn));
    } else {
      o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
      o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
    }
    s[j] = o1;
    s[j + half] = o2;
  }
  __syncwarp();
}

// ------------------------------------------------------------------ SwiGLU with dead zone
// swiglu_range_avx2 (dpuf_engine.c:967-997): the 8-wide formula
//   silu = g / (1 + exp_poly(clamp(0 - g, -40, 40))),  r = silu * u,  |r| < dz -> 0
// for elements in the vector part of a thread's range, and the scalar formula (libm expf)
// for the range's tail.  Ranges follow the reference's split of the flat [M*I] array over
// its nt threads (dpuf_engine.c:2007-2011), or whole 6-token slabs when the reference takes
// its slab-fused path (M >= 2 and ceil(M/6) >= nt, dpuf_engine.c:1983-2005).
DPUF_DEV bool swiglu_vector_elem(long long idx, long long total, int nt, bool slab) {
  if (slab) return true;
  if (total * nt < (1LL << 31)) {  // the same in 32-bit arithmetic (64-bit division is a long routine)
    const unsigned T = (unsigned)total, i = (unsigned)idx, n = (unsigned)nt;
    unsigned t = (i * n) / T;
    while (t > 0 && (T * t) / n > i) t--;
    while (t + 1 < n && (T * (t + 1)) / n <= i) t++;
    const unsigned s0 = (T * t) / n, s1 = (T * (t + 1)) / n;
    return (i - s0) < ((s1 - s0) & ~7u);
  }
  long long tid = (idx * nt) / total;
  while (tid > 0 && (total * tid) / nt > idx) tid--;
  while (tid + 1 < nt && (total * (tid + 1)) / nt <= idx) tid++;
  const long long s0 = (total * tid) / nt, s1 = (total * (tid + 1)) / nt;
  return (idx - s0) < ((s1 - s0) & ~7LL);
}

DPUF_DEV float swiglu_one(float g, float u, float dz, bool vec, const ExpfTable& et) {
  float r;
  if (vec) {
    const float ng = max_ps(-40.0f, min_ps(__fsub_rn(0.0f, g), 40.0f));
    const float silu = __fdiv_rn(g, __fadd_rn(1.0f, exp_poly(ng)));
    r = __fmul_rn(silu, u);
    if (dz > 0.0f && !(fabsf(r) >= dz)) r = 0.0f;
  } else {
    const float silu = (g >= 40.0f) ? g : ((g <= -40.0f) ? 0.0f : __fdiv_rn(g, __fadd_rn(1.0f, glibc_expf(-g, et))));
    r = __fmul_rn(silu, u);
    if (dz > 0.0f && fabsf(r) < dz) r = 0.0f;
  }
  return r;
}

// ------------------------------------------------------------------ embedding row chunk
// One warp: columns [c0, c0+64) of row r of a mode-12 matrix as the embedding lookup computes
// them (dpuf_embed_qr_hadamard4_packed_f32, dpuf_avx2.c:2738-2783): (u - 8) * ws, FWHT-64,
// then the column sign.  tp = the row's tile, lr = the row within the tile.  embed_load
// fetches what lane `lane` needs (so a warp can have several chunks' loads in flight),
// embed_finish computes the lane's two values (columns c0+lane and c0+32+lane).
struct EmbedRaw {
  uint16_t ws[2];
  uint8_t q[2];
  uint8_t sa, sb;  // sign bytes of the lane's two columns
};
DPUF_DEV EmbedRaw embed_load(const uint8_t* tp, int n_blk, int lr, const uint8_t* signs, int c0, int lane) {
  const int rg = lr >> 3, ri = lr & 7;
  const uint8_t* grp = tp + 16 + (size_t)rg * n_blk * 144;
  const uint8_t* qg = grp + (size_t)n_blk * 16;
  EmbedRaw r;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int b = (c0 >> 5) + h;
    r.ws[h] = *(const uint16_t*)(grp + (size_t)b * 16 + ri * 2);
    r.q[h] = qg[(size_t)b * 128 + (lane >> 3) * 32 + ri * 4 + (lane & 3)];
  }
  r.sa = signs ? signs[(c0 + lane) >> 3] : 0;
  r.sb = signs ? signs[(c0 + 32 + lane) >> 3] : 0;
  return r;
}
DPUF_DEV void embed_finish(const EmbedRaw& r, int c0, int lane, float& oa, float& ob) {
  float v[2];
  const int hi = (lane >> 2) & 1;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int u = hi ? (r.q[h] >> 4) : (r.q[h] & 15);
    v[h] = __fmul_rn((float)(u - 8), f16bits_to_f32(r.ws[h]));
  }
  fwht64_warp(v[0], v[1], lane);
  oa = ((r.sa >> ((c0 + lane) & 7)) & 1) ? -v[0] : v[0];
  ob = ((r.sb >> ((c0 + 32 + lane) & 7)) & 1) ? -v[1] : v[1];
}
DPUF_DEV void embed_chunk_warp(const uint8_t* tp, int n_blk, int lr, const uint8_t* signs, int c0, int lane,
                               float& oa, float& ob) {
  embed_finish(embed_load(tp, n_blk, lr, signs, c0, lane), c0, lane, oa, ob);
}

// Prep of one 64-chunk whose sign bytes were loaded ahead (sa, sb: the bytes holding the
// lane's columns c0+lane and c0+32+lane); same arithmetic as prep_chunk_warp.
DPUF_DEV void prep_chunk_warp_sb(float a, float b, uint8_t sa, uint8_t sb, int c0, int lane, int8_t* q8, float* xs,
                                 int32_t* xm) {
  if ((sa >> ((c0 + lane) & 7)) & 1) a = -a;
  if ((sb >> ((c0 + 32 + lane) & 7)) & 1) b = -b;
  fwht64_warp(a, b, lane);
  const int blk = c0 >> 5;
  quant32_warp(a, lane, q8 + c0, xs + blk, xm + blk);
  quant32_warp(b, lane, q8 + c0 + 32, xs + blk + 1, xm + blk + 1);
}

// ------------------------------------------------------------------ prep, 8 lanes per chunk
// The activation prep of one 64-column chunk (dpuf_prep_had4_packed_slab, dpuf_avx2.c:2364-2449)
// by a group of eight lanes, lane q of the group holding columns c0+8q .. c0+8q+7 in v[] (so a
// warp preps four chunks at once):
//   sign flip (bit r of sign byte sbyte negates v[r]),
//   FWHT-64 with ascending strides (fwht64_block_f32, dpuf_avx2.c:724-772): strides 1, 2, 4
//   inside the lane, 8, 16, 32 across lanes q^1, q^2, q^4; each butterfly gives (a+b, a-b) for
//   the pair (lower, upper), then x0.125 - the same operations on the same operands as the
//   one-chunk-per-warp form, so the same bits;
//   per 32-block (lanes 0-3 and 4-7 of the group): amax, xs = amax/127,
//   q = clamp(rint(v * (127/amax)), -127, 127), xm = 8 * sum(q); amax <= 1e-4 gives zeros.
// Every lane of the warp must call this (shuffles span the warp); `active` masks groups
// without a chunk (they compute on zeros and store nothing).
struct PrepOut {
  uint32_t lo, hi;  // this lane's eight codes (columns 8q .. 8q + 7 of the chunk)
  float xs;         // the lane's 32-block scale and sum (lanes 0 and 4 of the group publish)
  int xm;
};
DPUF_DEV PrepOut prep_chunk_g8_core(float (&v)[8], uint8_t sbyte, int lane) {
  const int q = lane & 7;
#pragma unroll
  for (int r = 0; r < 8; r++)
    if ((sbyte >> r) & 1) v[r] = -v[r];
#pragma unroll
  for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
    for (int r = 0; r < 8; r++)
      if (!(r & h)) {
        const float a = v[r], b = v[r + h];
        v[r] = __fadd_rn(a, b);
        v[r + h] = __fsub_rn(a, b);
      }
  }
#pragma unroll
  for (int m = 1; m < 8; m <<= 1) {
#pragma unroll
    for (int r = 0; r < 8; r++) {
      const float p = __shfl_xor_sync(kFull, v[r], m);
      v[r] = (q & m) ? __fsub_rn(p, v[r]) : __fadd_rn(v[r], p);
    }
  }
  float amax = 0.0f;
#pragma unroll
  for (int r = 0; r < 8; r++) {
    v[r] = __fmul_rn(v[r], 0.125f);
    amax = fmaxf(amax, fabsf(v[r]));
  }
  amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
  int qs[8];
  float xsv = 0.0f;
  int sum = 0;
  if (amax > 1e-4f) {
    xsv = __fdiv_rn(amax, 127.0f);
    const float inv = (amax > 1e-12f) ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
    for (int r = 0; r < 8; r++) {
      qs[r] = max(-127, min(127, __float2int_rn(__fmul_rn(v[r], inv))));
      sum += qs[r];
    }
  } else {
#pragma unroll
    for (int r = 0; r < 8; r++) qs[r] = 0;
  }
  sum += __shfl_xor_sync(kFull, sum, 1);
  sum += __shfl_xor_sync(kFull, sum, 2);
  PrepOut o;
  o.lo = 0;
  o.hi = 0;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    o.lo |= (uint32_t)(qs[r] & 0xFF) << (8 * r);
    o.hi |= (uint32_t)(qs[r + 4] & 0xFF) << (8 * r);
  }
  o.xs = xsv;
  o.xm = sum * 8;
  return o;
}
DPUF_DEV void prep_chunk_g8(float (&v)[8], uint8_t sbyte, bool active, int c0, int lane, int8_t* q8, float* xs,
                            int32_t* xm) {
  const int q = lane & 7;
  const PrepOut o = prep_chunk_g8_core(v, sbyte, lane);
  if (active) {
    *(uint2*)(q8 + c0 + 8 * q) = make_uint2(o.lo, o.hi);
    if ((q & 3) == 0) {
      const int blk = (c0 >> 5) + (q >> 2);
      xs[blk] = o.xs;
      xm[blk] = o.xm;
    }
  }
}

// ------------------------------------------------------------------ attention, one head pair
// gqa_attn_head_pair_f32 (dpuf_engine.c:341-577) for one (token, KV head, pair of Q heads),
// run by kAttnThreads threads (tid 0..255) that call sync() as a barrier among themselves:
//   scores  keys t < kv_len & ~3: eight lanes accumulate fma(q_i, k_i) over i = l, l+8, ...;
//           "pairs" tree (hsum4_256_ps); keys in the kv_len % 4 tail: "split" tree
//           (eng_hsum256_ps) - for a lone head the tail uses dot_f32_avx2's two accumulators
//           over 16-wide steps, summed lane-wise before the split tree; then * 1/sqrt(hd).
//   softmax e_k = exp_poly(s_k - max) for k < kv_len & ~7, lane sums over k = j mod 8 in
//           order, split tree, then the tail adds glibc expf(s_k - max) sequentially;
//           p_k = e_k * (1 / (sum + 1e-12)).
//   PV      per output dim: fma(p_k, v_kd, acc) over k ascending (pair path); the lone-head
//           path takes keys two at a time, k+1 first (dpuf_engine.c:541-548).
// Up to four query heads of one KV head run together (two pairs sharing the staged keys and
// values; every head keeps its pair's arithmetic); with last_lone the last head is the lone
// head of an odd group.  nh * hd <= 2 * kAttnThreads.
// qs [nh][hd] holds the (normed, rotated) query heads; kc/vc are this KV head's cache rows
// [max_seq][hd] (read through L2: other CTAs may have written them); sc [nh][sc_stride] and
// n_buf key/value tiles kt [n_buf][kAttnKeyTile][hd+8] are scratch; out receives nh * hd
// values.  Up to n_buf tiles are in flight (cp.async groups); the caller may have issued the
// first `pre` key tiles already (attn_issue_tile, one committed group each, nothing committed
// after them).  cur_k / cur_v (optional) are the key and value of position kv_len - 1, which
// then replace that row of its tile instead of being read from the cache.
constexpr int kAttnThreads = 256;
constexpr int kAttnKeyTile = 32;  // keys per tile (8 threads per key)
constexpr int kAttnMaxBuf = 3;    // tiles in flight at most
constexpr int kAttnMaxHeads = 4;  // query heads per call

struct AttnShared {
  float red[kAttnMaxHeads][kAttnThreads / 32];
  float lane_sum[kAttnMaxHeads][8];
  float inv_s[kAttnMaxHeads], max_s[kAttnMaxHeads];
};

// Key/value tiles hold the cache's element type T: fp32, or fp16 for an fp16 cache (values are
// widened to fp32 as they are used).  Rows are padded (8 floats, 16 halves) so that the score
// loop's eight threads per key and four keys per warp read distinct banks; a padded row stays a
// multiple of 16 bytes for the async copies.
template <typename T>
DPUF_HD constexpr int attn_row_pad() { return sizeof(T) == 4 ? 8 : 16; }
DPUF_DEV float kv_to_f(float x) { return x; }
DPUF_DEV float kv_to_f(__half x) { return __half2float(x); }
DPUF_DEV void kv_from_f(float& d, float x) { d = x; }
DPUF_DEV void kv_from_f(__half& d, float x) { d = __float2half_rn(x); }
// A tile's size in floats of scratch for elements of es bytes: 4 (fp32), 2 (fp16), or 1 for
// Q8 rows (hd int8 values + hd/32 fp32 scales, unpadded).
DPUF_HD size_t attn_tile_floats(int hd, int es = 4) {
  return es == 4   ? (size_t)kAttnKeyTile * (hd + 8)
         : es == 2 ? (size_t)kAttnKeyTile * (hd + 16) / 2
                   : (size_t)kAttnKeyTile * (hd + hd / 8) / 4;
}
// Scores of two heads over max_seq keys (the persistent kernel's pair).
DPUF_HD size_t attn_sc_floats(int max_seq) { return 2 * (((size_t)max_seq + 3) & ~(size_t)3); }
// Scratch of the per-step kernel with ppc pairs per CTA and n_buf tiles: qs [2 ppc][hd] |
// sc [2 ppc][max_seq padded to 4] | n_buf tiles (16-byte aligned for the async copies).
DPUF_HD size_t attn_step_floats(int hd, int max_seq, int ppc, int n_buf, int es = 4) {
  return (size_t)2 * ppc * hd + ppc * attn_sc_floats(max_seq) + n_buf * attn_tile_floats(hd, es);
}
// The per-step kernel's plan: two pairs per CTA (four query heads sharing the staged keys and
// values) when their outputs fit two per thread, and two tiles in flight, each dropped to one
// when the scratch would not fit the shared memory.
DPUF_HD void attn_step_plan(int hd, int max_seq, int* ppc, int* n_buf, int es = 4) {
  *ppc = 4 * hd <= 2 * kAttnThreads ? 2 : 1;
  *n_buf = 2;
  if (attn_step_floats(hd, max_seq, *ppc, *n_buf, es) * 4 > (size_t)kMaxDynSmem) *n_buf = 1;
  if (attn_step_floats(hd, max_seq, *ppc, *n_buf, es) * 4 > (size_t)kMaxDynSmem) *ppc = 1;
}
DPUF_HD size_t attn_scratch_floats(int hd, int max_seq, int es = 4) {
  int ppc, n_buf;
  attn_step_plan(hd, max_seq, &ppc, &n_buf, es);
  return attn_step_floats(hd, max_seq, ppc, n_buf, es);
}

// ------------------------------------------------------------------ async copies to shared
DPUF_DEV void cp_async16_cg(void* dst, const void* src) {  // L2 only: data other CTAs wrote
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
DPUF_DEV void cp_async8_ca(void* dst, const void* src) {  // read-only tables
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
DPUF_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
DPUF_DEV void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// Waits until at most n (0..2) of this thread's most recent groups are pending.
DPUF_DEV void cp_async_wait_pending(int n) {
  if (n <= 0)
    asm volatile("cp.async.wait_group 0;" ::: "memory");
  else if (n == 1)
    asm volatile("cp.async.wait_group 1;" ::: "memory");
  else
    asm volatile("cp.async.wait_group 2;" ::: "memory");
}

// Issues (and commits, as one group of this thread) the copy of tile `t` of a cache [.][hd]
// into buffer `buf` with a padded row stride of hd + 8: rows [32t, min(32t + 32, n_rows)) -
// n_rows excludes a row the caller supplies itself.  Every thread commits a group, with or
// without copies.
template <typename T>
DPUF_DEV void attn_issue_tile(T* buf, const T* src, int t, int n_rows, int hd, int tid) {
  constexpr int kPer = 16 / sizeof(T);  // elements per 16-byte piece
  const int t0 = t * kAttnKeyTile;
  const int nk = max(0, min(kAttnKeyTile, n_rows - t0));
  const int per_row = hd / kPer, n = nk * per_row;
  for (int i = tid; i < n; i += kAttnThreads) {
    const int r = i / per_row, c = (i - r * per_row) * kPer;
    cp_async16_cg(buf + r * (hd + attn_row_pad<T>()) + c, src + (size_t)(t0 + r) * hd + c);
  }
  cp_async_commit();
}

// Waits for tile t (tiles t+1 .. min(t + n_buf, n_t) - 1 may stay in flight), writes row
// `cur_row` from `cur` when the tile holds it, then sync().
template <typename T, typename Sync>
DPUF_DEV void attn_land_tile(T* buf, int t, int n_t, int n_buf, const float* cur, int cur_row, int hd, int tid,
                             Sync sync) {
  cp_async_wait_pending(min(n_buf - 1, n_t - 1 - t));
  const int t0 = t * kAttnKeyTile;
  if (cur && cur_row >= t0 && cur_row < t0 + kAttnKeyTile)
    for (int i = tid; i < hd; i += kAttnThreads) kv_from_f(buf[(cur_row - t0) * (hd + attn_row_pad<T>()) + i], cur[i]);
  sync();
}

// vec_softmax_avx2 (dpuf_engine.c:579-601) of the nh score rows sc[h][0, kv_len) in place;
// lmax holds each thread's running maximum per head.  The scores must be complete (the
// caller's last sync() came after them); no sync() follows the final normalisation.
template <typename Sync>
DPUF_DEV void attn_softmax(float* sc, int sc_stride, int nh, int kv_len, const float (&lmax)[kAttnMaxHeads],
                           AttnShared* sh, const ExpfTable& et, int tid, Sync sync) {
  const int lane = tid & 31, kv8 = kv_len & ~7;
  // ---- max
#pragma unroll
  for (int h = 0; h < kAttnMaxHeads; h++) {
    if (h >= nh) break;
    float v = warp_max(lmax[h]);
    if (lane == 0) sh->red[h][tid >> 5] = v;
  }
  sync();
  if (tid < nh) {
    float v = -1e30f;
    for (int w = 0; w < kAttnThreads / 32; w++) v = max_ps(v, sh->red[tid][w]);
    sh->max_s[tid] = v;
  }
  sync();
  // ---- exp over the 8-aligned part
  for (int h = 0; h < nh; h++) {
    const float mx = sh->max_s[h];
    for (int k = tid; k < kv8; k += kAttnThreads)
      sc[h * sc_stride + k] = exp_poly(__fsub_rn(sc[h * sc_stride + k], mx));
  }
  sync();
  // ---- lane sums (8 sequential chains per head); the <= 7 tail exponentials (glibc expf) are
  // independent, so eight more threads per head evaluate them meanwhile
  if (tid < 8 * nh) {
    const int h = tid >> 3, l = tid & 7;
    const float* sp = sc + h * sc_stride;
    float acc = 0.0f;
    for (int k = l; k < kv8; k += 8) acc = __fadd_rn(acc, sp[k]);
    sh->lane_sum[h][l] = acc;
  } else if (tid >= 64 && tid < 64 + 8 * nh) {
    const int h = (tid - 64) >> 3, k = kv8 + ((tid - 64) & 7);
    if (k < kv_len) {
      float* sp = sc + h * sc_stride;
      sp[k] = glibc_expf(__fsub_rn(sp[k], sh->max_s[h]), et);
    }
  }
  sync();
  // split tree of the lane sums, then the tail added in order
  if (tid < nh) {
    const float* sp = sc + tid * sc_stride;
    float su = tree8_split_arr(sh->lane_sum[tid]);
    for (int k = kv8; k < kv_len; k++) su = __fadd_rn(su, sp[k]);
    sh->inv_s[tid] = __fdiv_rn(1.0f, __fadd_rn(su, 1e-12f));
  }
  sync();
  for (int h = 0; h < nh; h++) {
    const float inv = sh->inv_s[h];
    for (int k = tid; k < kv_len; k += kAttnThreads) sc[h * sc_stride + k] = __fmul_rn(sc[h * sc_stride + k], inv);
  }
}

template <typename T, typename Sync>
DPUF_DEV void attn_pair_body(float* qs, int nh, bool last_lone, int hd, int kv_len, const T* kc, const T* vc,
                             int sc_stride, float* sc, T* kt, int n_buf, int pre, const float* cur_k,
                             const float* cur_v, AttnShared* sh, float* out, const ExpfTable& et, int tid, Sync sync,
                             bool out_to_qs = false) {
  const int kvs = hd + attn_row_pad<T>();  // padded smem row of a staged key
  const size_t tile = (size_t)kAttnKeyTile * kvs;  // elements
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int kv4 = kv_len & ~3;
  const int n_t = (kv_len + kAttnKeyTile - 1) / kAttnKeyTile;
  const int n_rows = cur_k ? kv_len - 1 : kv_len;  // rows read from the cache
  float lmax[kAttnMaxHeads] = {-1e30f, -1e30f, -1e30f, -1e30f};
  // ---- scores
  for (int t = pre; t < min(n_buf, n_t); t++) attn_issue_tile(kt + (size_t)t * tile, kc, t, n_rows, hd, tid);
  for (int t = 0; t < n_t; t++) {
    const int t0 = t * kAttnKeyTile;
    const int nk = min(kAttnKeyTile, kv_len - t0);
    T* buf = kt + (size_t)(t % n_buf) * tile;
    attn_land_tile(buf, t, n_t, n_buf, cur_k, kv_len - 1, hd, tid, sync);
    const int key = tid >> 3, l = tid & 7;
    const int tk = t0 + key;
    const bool valid = key < nk;
    const T* kp = buf + key * kvs;
#pragma unroll
    for (int h = 0; h < kAttnMaxHeads; h++) {
      if (h >= nh) break;
      const float* qv = qs + h * hd;
      // Shuffle trees run on all lanes (keys of one warp may sit on both sides of kv4).
      float acc = 0.0f;
      if (valid)
        for (int i = l; i < hd; i += 8) acc = __fmaf_rn(qv[i], kv_to_f(kp[i]), acc);
      const float t_pairs = tree8_pairs(acc);
      float t_split;
      if (!(last_lone && h == nh - 1)) {
        t_split = tree8_split(acc);
      } else {
        // lone head, tail key: dot_f32_avx2 (dpuf_engine.c:325-339)
        float a0 = 0.0f, a1 = 0.0f;
        if (valid) {
          int i = 0;
          for (; i + 15 < hd; i += 16) {
            a0 = __fmaf_rn(qv[i + l], kv_to_f(kp[i + l]), a0);
            a1 = __fmaf_rn(qv[i + 8 + l], kv_to_f(kp[i + 8 + l]), a1);
          }
          for (; i + 7 < hd; i += 8) a0 = __fmaf_rn(qv[i + l], kv_to_f(kp[i + l]), a0);
        }
        t_split = tree8_split(__fadd_rn(a0, a1));
      }
      float sv = __fmul_rn((tk < kv4) ? t_pairs : t_split, scale);
      if (valid && l == 0) {
        sc[h * sc_stride + tk] = sv;
        lmax[h] = max_ps(lmax[h], sv);
      }
    }
    sync();  // the buffer is free again
    if (t + n_buf < n_t) attn_issue_tile(buf, kc, t + n_buf, n_rows, hd, tid);
  }
  // the first value tiles load while the softmax runs
  for (int t = 0; t < min(n_buf, n_t); t++) attn_issue_tile(kt + (size_t)t * tile, vc, t, n_rows, hd, tid);
  attn_softmax(sc, sc_stride, nh, kv_len, lmax, sh, et, tid, sync);
  // ---- PV: thread o owns outputs o and o + kAttnThreads, each a sequential chain over the
  // keys in the reference's order
  float acc[2] = {0.0f, 0.0f};
  const int hd8 = hd & ~7;
  for (int t = 0; t < n_t; t++) {
    const int t0 = t * kAttnKeyTile;
    const int nk = min(kAttnKeyTile, kv_len - t0);
    T* buf = kt + (size_t)(t % n_buf) * tile;
    attn_land_tile(buf, t, n_t, n_buf, cur_v, kv_len - 1, hd, tid, sync);
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int o = tid + j * kAttnThreads;
      if (o >= nh * hd) break;
      const int h = o / hd, d = o % hd;
      const float* pp = sc + h * sc_stride + t0;
      const T* vt = buf + d;
      float a = acc[j];
      if (!(last_lone && h == nh - 1)) {
        for (int k = 0; k < nk; k++) a = __fmaf_rn(pp[k], kv_to_f(vt[k * kvs]), a);
      } else if ((hd & 63) == 0) {
        // keys two at a time, k+1 first (tiles hold an even number of keys but the last)
        int k = 0;
        for (; k + 1 < nk; k += 2) {
          const float t1 = __fmaf_rn(pp[k + 1], kv_to_f(vt[(k + 1) * kvs]), a);
          a = __fmaf_rn(pp[k], kv_to_f(vt[k * kvs]), t1);
        }
        if (k < nk) a = __fmaf_rn(pp[k], kv_to_f(vt[k * kvs]), a);
      } else {
        for (int k = 0; k < nk; k++) {
          const float pv = pp[k], vv = kv_to_f(vt[k * kvs]);
          a = (d < hd8) ? __fmaf_rn(pv, vv, a) : __fadd_rn(a, __fmul_rn(pv, vv));
        }
      }
      acc[j] = a;
    }
    sync();  // the buffer is free again
    if (t + n_buf < n_t) attn_issue_tile(buf, vc, t + n_buf, n_rows, hd, tid);
  }
  // (with out_to_qs the outputs also replace the queries, which are no longer read)
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int o = tid + j * kAttnThreads;
    if (o < nh * hd) {
      out[o] = acc[j];
      if (out_to_qs) qs[o] = acc[j];
    }
  }
}

// ------------------------------------------------------------------ Q8 KV cache (kv_type 1)
// _mm256_cvtps_epi32 (round to nearest even), the saturating packs and max(-127) of
// quantize_vec_q8_blk32: a NaN or out-of-range product converts to INT32_MIN, i.e. -127.
DPUF_DEV int q8_cvt(float y) {
  if (!(y == y) || y >= 2147483648.0f || y < -2147483648.0f) return -127;
  return max(-127, min(127, __float2int_rn(y)));
}

// One warp quantizes the hd values x (lane-strided: element i is read by lane i % 32) into a
// Q8 cache row: hd int8 values, then hd/32 fp32 scales (quantize_vec_q8_blk32,
// dpuf_engine.c:751-781).  Per 32-block: amax by the reference's max tree (lanes j, j+8 and
// j+16, j+24 first, then the 4-wide and 2-wide folds), scale = amax / 127,
// q = cvt(x * (127 / amax)), or 0 when amax <= 1e-12.  hd % 32 == 0.
DPUF_DEV void q8_row_warp(const float* x, char* row, int hd, int lane) {
  float* scales = (float*)(row + hd);
  for (int c0 = 0; c0 < hd; c0 += 32) {
    const float v = x[c0 + lane];
    float m = fabsf(v);
    m = max_ps(m, __shfl_down_sync(kFull, m, 8));   // lanes 0-7, 16-23: max(|x_l|, |x_l+8|)
    m = max_ps(m, __shfl_down_sync(kFull, m, 16));  // lanes 0-7: the 8-lane vector
    m = max_ps(m, __shfl_down_sync(kFull, m, 4));   // lanes 0-3: 128-bit halves folded
    m = max_ps(m, __shfl_down_sync(kFull, m, 2));   // movehl fold
    m = max_ps(m, __shfl_down_sync(kFull, m, 1));   // max_ss
    const float amax = __shfl_sync(kFull, m, 0);
    const float inv = (amax > 1e-12f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    row[c0 + lane] = (char)q8_cvt(__fmul_rn(v, inv));
    if (lane == 0) scales[c0 >> 5] = __fdiv_rn(amax, 127.0f);
  }
}

// Issues (and commits, as one group of this thread) the copy of Q8 tile `t` - rows
// [32t, min(32t + 32, n_rows)) of rb bytes, contiguous in the cache - into buf (unpadded).
// Rows of a multiple of 16 bytes go by async copies through L2; other row sizes (hd = 32 or
// 64) by plain L2 loads, complete when this returns.
DPUF_DEV void attn_q8_issue(char* buf, const char* src, int t, int n_rows, int rb, int tid) {
  const int t0 = t * kAttnKeyTile;
  const int nbytes = max(0, min(kAttnKeyTile, n_rows - t0)) * rb;
  const char* s = src + (size_t)t0 * rb;
  if ((rb & 15) == 0) {
    for (int i = tid * 16; i < nbytes; i += kAttnThreads * 16) cp_async16_cg(buf + i, s + i);
  } else {
    for (int i = tid * 4; i < nbytes; i += kAttnThreads * 4) *(int*)(buf + i) = __ldcg((const int*)(s + i));
  }
  cp_async_commit();
}

// gqa_attn_head_pair_q8 (dpuf_engine.c:621-749) for nh <= 4 query heads of one KV head over
// its Q8 rows kc / vc (n_buf tiles kt of kAttnKeyTile rows in flight), in the layout of
// attn_pair_body.  Scores: pair heads take keys two at a time - per block and lane l,
// t = fma(q[l], k[l], fma(q[l+8], k[l+8], t)) over the two 16-wide halves, then
// fma(t, k_scale, acc), pairs tree; the odd last key and the lone head use
// dot_f32_q8_blk32_avx2 (dpuf_engine.c:603-619): lane accumulators over (l, l+16) and
// (l+8, l+24), fma(a0 + a1, k_scale, acc), split tree.  Softmax as attn_softmax.  PV for
// output d of every head: fma(p_k * vs_k[d/32], v_kd, acc) over k ascending.
template <typename Sync>
DPUF_DEV void attn_q8_body(float* qs, int nh, bool last_lone, int hd, int kv_len, const char* kc, const char* vc,
                           int sc_stride, float* sc, char* kt, int n_buf, AttnShared* sh, float* out,
                           const ExpfTable& et, int tid, Sync sync) {
  const int rb = hd + hd / 8, nb = hd >> 5;
  const size_t tile = (size_t)kAttnKeyTile * rb;  // bytes
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int kv2 = kv_len & ~1;
  const int n_t = (kv_len + kAttnKeyTile - 1) / kAttnKeyTile;
  float lmax[kAttnMaxHeads] = {-1e30f, -1e30f, -1e30f, -1e30f};
  // ---- scores
  for (int t = 0; t < min(n_buf, n_t); t++) attn_q8_issue(kt + (size_t)t * tile, kc, t, kv_len, rb, tid);
  for (int t = 0; t < n_t; t++) {
    const int t0 = t * kAttnKeyTile;
    const int nk = min(kAttnKeyTile, kv_len - t0);
    char* buf = kt + (size_t)(t % n_buf) * tile;
    cp_async_wait_pending(min(n_buf - 1, n_t - 1 - t));
    sync();
    const int key = tid >> 3, l = tid & 7;
    const int tk = t0 + key;
    const bool valid = key < nk;
    const int8_t* kp = (const int8_t*)(buf + key * rb);
    const float* ks = (const float*)(buf + key * rb + hd);
#pragma unroll
    for (int h = 0; h < kAttnMaxHeads; h++) {
      if (h >= nh) break;
      const float* qv = qs + h * hd;
      const bool tail = (last_lone && h == nh - 1) || tk >= kv2;
      float acc = 0.0f;
      if (valid) {
        if (!tail) {
          for (int b = 0; b < nb; b++) {
            const int c0 = b << 5;
            float u = __fmaf_rn(qv[c0 + 8 + l], (float)kp[c0 + 8 + l], 0.0f);
            u = __fmaf_rn(qv[c0 + l], (float)kp[c0 + l], u);
            u = __fmaf_rn(qv[c0 + 24 + l], (float)kp[c0 + 24 + l], u);
            u = __fmaf_rn(qv[c0 + 16 + l], (float)kp[c0 + 16 + l], u);
            acc = __fmaf_rn(u, ks[b], acc);
          }
        } else {
          for (int b = 0; b < nb; b++) {
            const int c0 = b << 5;
            float a0 = __fmaf_rn(qv[c0 + l], (float)kp[c0 + l], 0.0f);
            float a1 = __fmaf_rn(qv[c0 + 8 + l], (float)kp[c0 + 8 + l], 0.0f);
            a0 = __fmaf_rn(qv[c0 + 16 + l], (float)kp[c0 + 16 + l], a0);
            a1 = __fmaf_rn(qv[c0 + 24 + l], (float)kp[c0 + 24 + l], a1);
            acc = __fmaf_rn(__fadd_rn(a0, a1), ks[b], acc);
          }
        }
      }
      // both trees run on all lanes (a warp's four keys may take different forms)
      const float tp = tree8_pairs(acc), ts = tree8_split(acc);
      const float sv = __fmul_rn(tail ? ts : tp, scale);
      if (valid && l == 0) {
        sc[h * sc_stride + tk] = sv;
        lmax[h] = max_ps(lmax[h], sv);
      }
    }
    sync();  // the buffer is free again
    if (t + n_buf < n_t) attn_q8_issue(buf, kc, t + n_buf, kv_len, rb, tid);
  }
  // the first value tiles load while the softmax runs
  for (int t = 0; t < min(n_buf, n_t); t++) attn_q8_issue(kt + (size_t)t * tile, vc, t, kv_len, rb, tid);
  attn_softmax(sc, sc_stride, nh, kv_len, lmax, sh, et, tid, sync);
  // ---- PV: thread o owns outputs o and o + kAttnThreads
  float acc[2] = {0.0f, 0.0f};
  for (int t = 0; t < n_t; t++) {
    const int t0 = t * kAttnKeyTile;
    const int nk = min(kAttnKeyTile, kv_len - t0);
    char* buf = kt + (size_t)(t % n_buf) * tile;
    cp_async_wait_pending(min(n_buf - 1, n_t - 1 - t));
    sync();
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int o = tid + j * kAttnThreads;
      if (o >= nh * hd) break;
      const int h = o / hd, d = o % hd;
      const float* pp = sc + h * sc_stride + t0;
      const int8_t* vt = (const int8_t*)buf + d;
      const char* vs = buf + hd + 4 * (d >> 5);
      float a = acc[j];
      for (int k = 0; k < nk; k++)
        a = __fmaf_rn(__fmul_rn(pp[k], *(const float*)(vs + k * rb)), (float)vt[k * rb], a);
      acc[j] = a;
    }
    sync();  // the buffer is free again
    if (t + n_buf < n_t) attn_q8_issue(buf, vc, t + n_buf, kv_len, rb, tid);
  }
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int o = tid + j * kAttnThreads;
    if (o < nh * hd) out[o] = acc[j];
  }
}

}  // namespace dpuf
