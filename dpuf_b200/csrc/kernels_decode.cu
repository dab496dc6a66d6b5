// kernels_decode.cu - batch-1 decode as one persistent cooperative kernel.
//
// One CTA per SM runs every step of a greedy decode (or one forward_token step): embedding,
// all layers, final norm, LM head and argmax.  The per-element arithmetic is the same as the
// per-step kernels' (layer_dev.cuh, and the GEMV's exact block chain), so logits and ids are
// bit-identical to the reference's.
//
// Weight stream.  The weights never depend on activations, so a producer warp per CTA walks
// the CTA's share of every projection of every layer and step in order, moving stage s (32
// blocks: the two 8-row groups' scales and nibbles, 4608 bytes per group) of two 16-row units
// at a time into a shared-memory ring slot with cp.async.bulk (TMA, this CTA's own copy)
// completed on an mbarrier.  It runs ahead across phases and barriers, bounded only by the
// ring, so HBM keeps streaming while the consumers normalise, attend or wait.
//
// Consumers (warps 0..8).  Per slot, eight dot warps compute the exact integer block dots
// sum_k u_k q_k with dp4a (lane = unit and row, four blocks each, independent chains), turn
// them into pairs p = float(dot - xm), s = ws * xs (0, 0 for a skipped block) and hand them to
// the chain warp through a 4-deep ring of pair buffers (named-barrier hand-off); the chain
// warp runs acc = fma(p, s, acc) per row over the blocks in order (dpuf_avx2.c:2601-2640),
// lanes 0..15 for unit A and 16..31 for unit B, and writes the units' outputs (SwiGLU for a
// gate/up pair - gate tile in A, up tile in B - and the running argmax for the LM head).
// Between projections the consumers do the row-wide steps redundantly in every CTA (the
// residual stream h lives in each CTA's shared memory): residual add, RMSNorm, activation
// prep; attention runs on one CTA per (KV head, query-head pair) and preps its output for the
// o projection; the gate/up output is prepped for the down projection in 64-column chunks,
// one chunk per CTA.
//
// Exchange between CTAs.  The vectors a phase produces for all CTAs (q/k/v, o, gate/up, down
// outputs, the LM head's argmax partials) are 64-bit words: the value and the generation of
// the producing phase.  A reader stages them and re-reads any word that does not carry the
// generation it expects yet, so no grid barrier separates a projection from its readers;
// every phase reads the whole output of the phase before it, so no producer can overwrite a
// word that a reader still needs.  Grid barriers remain after attention (the o projection's
// prepped input) and, on one GPU, after the down-input prep.
//
// Tensor parallelism (tp_world > 1, one process per GPU).  Every projection's units are dealt
// over all ranks' CTAs; producers store the tagged words into every rank's exchange buffer
// (peer stores over NVLink), the down-input prep publishes tagged codes and scales, and the
// per-GPU steps (norms, attention, the preps' inputs) run on every rank.  No cross-GPU barrier
// is needed: the tags carry the ordering.
//
// Work split.  Each projection's 16-row units are dealt in contiguous ranges, and the CTA that
// receives the remainder units rotates from one projection to the next, so every CTA streams
// about the same bytes per layer and the ring absorbs the one-unit imbalance of a projection.
//
// Every wait is bounded: an mbarrier, grid-barrier, counter or tagged-word wait gives up after
// kWaitNs (kTpWaitNs across ranks), sets the error word (of every rank) and the CTA's abort
// flag.  After that every wait returns at once, but the consumers keep their control flow
// (every loop runs its full trip count and reaches every named barrier, with all addresses
// depending on shapes only), so no warp is left waiting at a barrier; the producer stops
// issuing and waits, bounded, for the copies it issued.
#include <algorithm>

#include "kernels.cuh"
#include "layer_dev.cuh"

namespace dpuf {

namespace {

constexpr int kTeamWarps = 8;                   // dot warps per team (one slot per team at a time)
constexpr int kTeams = 1;                       // teams take alternate slots
constexpr int kMmaWarps = kTeamWarps * kTeams;  // dot warps
constexpr int kChainWarp = kMmaWarps;
constexpr int kProdWarp = kMmaWarps + 1;
constexpr int kThreads = (kMmaWarps + 2) * 32;  // 576
constexpr int kConsumers = (kMmaWarps + 1) * 32;
// A ring slot holds stage s (32 blocks) of two 16-row units A and B; per unit: nibbles of
// group 0 | group 1 (+32 pad) | scales of group 0 | group 1, and unit B starts 64 bytes past
// a unit's size so that A's and B's lanes read different banks.
constexpr int kNib1 = 4128, kSc0 = 8256, kSc1 = 8800;
constexpr int kHalf = 9408;
constexpr int kSlotBytes = 2 * kHalf;
constexpr int kMaxRing = 24;
constexpr int kNPs = 4;             // pair buffers between the dot warps and the chain warp
constexpr int kPsRow = 34;          // float2 per row of a pair buffer: 32 blocks + pad (banks)
constexpr int kPsBuf = 2 * 16 * kPsRow;  // float2 per pair buffer: [unit][row][block]
// Named barriers: 1 consumers, 2 attention, then per pair buffer "filled" and "emptied".
constexpr int kBarFilled = 3, kBarEmptied = kBarFilled + kNPs;
static_assert(kBarEmptied + kNPs <= 16, "named barrier ids");
constexpr int kHandoff = (kTeamWarps + 1) * 32;  // threads of a pair-buffer hand-off
constexpr int kBarConsumers = 1, kBarAttn = 2;
constexpr unsigned long long kWaitNs = 2000000000ull;    // 2 s
constexpr unsigned long long kTpWaitNs = 5000000000ull;  // 5 s: other ranks' hosts may launch later
enum { kQKV = 0, kO = 1, kGU = 2, kDown = 3, kLM = 4 };

// ------------------------------------------------------------------ PTX helpers
DPUF_DEV unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
DPUF_DEV void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
DPUF_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
DPUF_DEV void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
DPUF_DEV bool mbar_try(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that lets the hardware park the thread until the phase completes or `ns` pass, so
// a waiting thread takes no issue slots from the warps doing the work.
DPUF_DEV bool mbar_try_for(uint64_t* b, unsigned parity, unsigned ns) {
  unsigned ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Weight bytes are read once per step, so their L2 lines are marked evict-first: the stream
// then does not push the KV cache, the activations and the barrier words out of L2.
DPUF_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
DPUF_DEV void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
DPUF_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
DPUF_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
DPUF_DEV void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
DPUF_DEV void named_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Shared state of a CTA that is not in the dynamic buffer.
struct DecShared {
  uint64_t full[kMaxRing], empty[kMaxRing];
  AttnShared attn;
  float lanes[8];
  float inv;
  float arg_v[kConsumers / 32];  // per-warp argmax of the LM partials
  int arg_i[kConsumers / 32];
  int next_id;
  volatile int abort;
};

// ------------------------------------------------------------------ exchange of vectors
// A value other CTAs read is one 64-bit word: the value's bits, and the generation of the
// phase that produced it in the high half.  It is stored to this rank's buffer and to every
// other rank's copy (stores to the peer's memory over NVLink); a reader waits until the word
// carries the generation it expects.  Every phase reads the whole output of the phase before,
// so no producer can overwrite a word (with a later generation) that a reader still needs.
DPUF_DEV uint64_t tagged(float v, unsigned gen) { return ((uint64_t)gen << 32) | __float_as_uint(v); }
DPUF_DEV void st_tagged_sys(uint64_t* p, uint64_t w) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
DPUF_DEV void st_tagged_gpu(uint64_t* p, uint64_t w) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// (one GPU: device scope; several ranks: system scope, every rank's copy)
DPUF_DEV void put_tagged(const DecodeArgs& A, uint64_t* p, uint64_t w) {
  if (A.tp_world == 1) {
    st_tagged_gpu(p, w);
    return;
  }
  st_tagged_sys(p, w);
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) st_tagged_sys((uint64_t*)((char*)p + A.tp_delta[r]), w);
}
DPUF_DEV void put_float(const DecodeArgs& A, float* p, float v) {
  *p = v;
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) *(float*)((char*)p + A.tp_delta[r]) = v;
}
// Adds 1 to completion counter i of this rank and of every other rank (relaxed: no fence; the
// tags, not the count, say whether a value has arrived).
DPUF_DEV void count_done(const DecodeArgs& A, int i) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(A.ctr + i) : "memory");
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank)
      asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"((char*)(A.ctr + i) + A.tp_delta[r]) : "memory");
}
DPUF_DEV ulonglong2 ld_tagged2(const uint64_t* p, bool sys) {
  ulonglong2 v;
  if (sys)
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
DPUF_DEV unsigned tag_of(uint64_t w) { return (unsigned)(w >> 32); }
DPUF_DEV float value_of(uint64_t w) { return __uint_as_float((unsigned)w); }
// Records a failure in the error word of this rank and of every other rank, whose waits then
// stop at once instead of running into their own limits.
DPUF_DEV void raise_err(const DecodeArgs& A, int code) {
  atomicCAS(A.err, 0, code);
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) atomicCAS((int*)((char*)A.err + A.tp_delta[r]), 0, code);
}

// Bounded mbarrier wait by one thread: false (and the CTA abort flag and the error word set)
// once kWaitNs pass, or when the CTA or another CTA has aborted.  Each try parks the thread
// for up to 20 us unless the phase completes first.
DPUF_DEV bool wait_bar(uint64_t* b, unsigned parity, DecShared& S, const DecodeArgs& A) {
  int* err = A.err;
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    if (mbar_try_for(b, parity, 20000u)) return true;
    if (S.abort) return false;
    if (*(volatile int*)err) {
      S.abort = 1;
      return false;
    }
    if (globaltimer() - t0 > kWaitNs) {
      S.abort = 1;
      raise_err(A, 1);
      return false;
    }
  }
}

// Bounded wait of one thread for a pair of tagged words to carry generation `gen`: re-reads
// until they do; gives up (returning what it read) once the CTA or another CTA or rank has
// aborted, or the wait limit has passed (error word 3).  Under tensor parallelism the limit
// allows for other ranks' hosts launching later.
DPUF_DEV ulonglong2 wait_tagged2(const uint64_t* p, unsigned gen, const DecodeArgs& A, DecShared& S) {
  unsigned long long t0 = 0;
  const unsigned long long limit = A.tp_world > 1 ? kTpWaitNs : kWaitNs;
  for (int it = 0;; it++) {
    const ulonglong2 w = ld_tagged2(p, A.tp_world > 1);
    if ((tag_of(w.x) == gen && tag_of(w.y) == gen) || S.abort) return w;
    if (it >= 4) __nanosleep(64);  // polls of many threads share L2 with the weight stream
    if ((it & 31) == 31) {
      if (*(volatile int*)A.err) {
        S.abort = 1;
        return w;
      }
      const unsigned long long now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit) {
        raise_err(A, 3);
        S.abort = 1;
        return w;
      }
    }
  }
}

// ------------------------------------------------------------------ work plan
struct Unit {
  const uint8_t* tile;
  int n_r;         // rows in the tile
  int row;         // first row of the tile in its matrix
  uint64_t* tout;  // tagged output of row `row` (chain epilogue), or null
  float* out;      // plain output of row `row` (the LM head's logits), or null
};

DPUF_DEV int kind_cols(const DecodeArgs& A, int kind) {
  return kind == kO ? A.qd : (kind == kDown ? A.I : A.H);
}
DPUF_DEV int kind_units(const DecodeArgs& A, int kind) {
  const int tq = (A.qd + 15) >> 4, tkv = (A.kvd + 15) >> 4, th = (A.H + 15) >> 4, ti = (A.I + 15) >> 4;
  switch (kind) {
    case kQKV: return tq + 2 * tkv;
    case kO: return th;
    case kGU: return ti;
    case kDown: return A.keep_down;
    default: return (A.V + 15) >> 4;
  }
}

DPUF_DEV Unit make_unit(const uint8_t* tiles, long long stride, int rows, int t, uint64_t* tout,
                       float* out = nullptr) {
  Unit u;
  u.tile = tiles + (size_t)t * stride;
  u.row = t * kTileRows;
  u.n_r = min(kTileRows, rows - u.row);
  u.tout = tout ? tout + u.row : nullptr;
  u.out = out ? out + u.row : nullptr;
  return u;
}

DPUF_DEV Unit unit_of(const DecodeArgs& A, const DecLayer& Ly, int kind, int u, int sub) {
  switch (kind) {
    case kQKV: {
      const int tq = (A.qd + 15) >> 4, tkv = (A.kvd + 15) >> 4;
      if (u < tq) return make_unit(Ly.tiles[0], Ly.stride[0], A.qd, u, A.q);
      if (u < tq + tkv) return make_unit(Ly.tiles[1], Ly.stride[1], A.kvd, u - tq, A.k);
      return make_unit(Ly.tiles[2], Ly.stride[2], A.kvd, u - tq - tkv, A.v);
    }
    case kO: return make_unit(Ly.tiles[3], Ly.stride[3], A.H, u, A.o_out);
    case kGU: return sub == 0 ? make_unit(Ly.tiles[4], Ly.stride[4], A.I, u, nullptr)
                              : make_unit(Ly.tiles[5], Ly.stride[5], A.I, u, A.s_out);
    case kDown: return make_unit(Ly.tiles[6], Ly.stride[6], A.H, u, A.d_out);
    default: return make_unit(A.lm_tiles, A.lm_stride, A.V, u, nullptr, A.logits);
  }
}

// Contiguous unit range of CTA c in a projection of U units; the remainder units go to the
// `U % G` CTAs starting at `rot`, which then advances by U % G.  With tensor parallelism the
// G CTAs are all ranks' CTAs, interleaved (c = blockIdx.x * ranks + rank), so that every rank
// gets units of every projection with at least `ranks` units: each rank then takes part in
// every phase, which is what keeps a fast rank from overwriting an exchanged vector (with a
// later generation) before a slow rank has read it.
DPUF_DEV void take_range(const DecodeArgs& A, int U, int& rot, int& u0, int& n) {
  const int G = gridDim.x * A.tp_world, c = blockIdx.x * A.tp_world + A.tp_rank;
  const int v = (c - rot + G) % G;
  const int base = U / G, ext = U % G;
  n = base + (v < ext ? 1 : 0);
  u0 = v * base + min(v, ext);
  rot = (rot + ext) % G;
}

// ------------------------------------------------------------------ producer
struct Producer {
  int slot = 0;
  unsigned phase = 0;     // parity of the slot's current use
  long long issued = 0;
  uint64_t policy = 0;    // L2 policy of the weight copies
};

// Copies of stage s of unit un into the half-slot dst; returns the bytes.
DPUF_DEV unsigned copy_stage(const Unit& un, int n_blk, int s, unsigned char* dst, uint64_t* bar, uint64_t pol) {
  const int groups = un.n_r > 8 ? 2 : 1;
  const int kb = min(32, n_blk - s * 32);
  for (int g = 0; g < groups; g++) {
    const uint8_t* gp = un.tile + 16 + (size_t)g * n_blk * 144;
    bulk_g2s(dst + (g ? kNib1 : 0), gp + (size_t)n_blk * 16 + (size_t)s * 4096, (unsigned)kb * 128, bar, pol);
    bulk_g2s(dst + (g ? kSc1 : kSc0), gp + (size_t)s * 512, (unsigned)kb * 16, bar, pol);
  }
  return (unsigned)(groups * kb * 144);
}

DPUF_DEV bool produce_pair(const Unit& ua, const Unit& ub, bool has_b, int n_blk, int n_st, unsigned char* ring,
                           int n_ring, Producer& P, DecShared& S, const DecodeArgs& A) {
  for (int s = 0; s < n_st; s++) {
    if (!wait_bar(&S.empty[P.slot], P.phase ^ 1u, S, A)) return false;
    const int kb = min(32, n_blk - s * 32);
    const unsigned bytes = (unsigned)(((ua.n_r > 8 ? 2 : 1) + (has_b ? (ub.n_r > 8 ? 2 : 1) : 0)) * kb * 144);
    uint64_t* bar = &S.full[P.slot];
    unsigned char* dst = ring + (size_t)P.slot * kSlotBytes;
    mbar_expect_tx(bar, bytes);
    copy_stage(ua, n_blk, s, dst, bar, P.policy);
    if (has_b) copy_stage(ub, n_blk, s, dst + kHalf, bar, P.policy);
    P.issued++;
    if (++P.slot == n_ring) {
      P.slot = 0;
      P.phase ^= 1u;
    }
  }
  return true;
}

// Units of a projection are consumed in pairs: for gate/up, (gate tile u, up tile u); for the
// others, consecutive units of the CTA's range (the last one alone when the count is odd).
DPUF_DEV void pair_of(const DecodeArgs& A, const DecLayer& Ly, int kind, int u, int u_end, Unit& ua, Unit& ub,
                      bool& has_b, int& step) {
  if (kind == kGU) {
    ua = unit_of(A, Ly, kind, u, 0);
    ub = unit_of(A, Ly, kind, u, 1);
    has_b = true;
    step = 1;
  } else {
    ua = unit_of(A, Ly, kind, u, 0);
    has_b = u + 1 < u_end;
    ub = has_b ? unit_of(A, Ly, kind, u + 1, 0) : ua;
    step = 2;
  }
}

DPUF_DEV bool produce_phase(const DecodeArgs& A, const DecLayer* layers, int l, int kind, int& rot,
                            unsigned char* ring, int n_ring, Producer& P, DecShared& S) {
  int u0, n;
  take_range(A, kind_units(A, kind), rot, u0, n);
  const int n_blk = kind_cols(A, kind) >> 5, n_st = (n_blk + 31) >> 5;
  const DecLayer& Ly = layers[kind == kLM ? 0 : l];
  for (int u = u0, step = 1; u < u0 + n; u += step) {
    Unit ua, ub;
    bool has_b;
    pair_of(A, Ly, kind, u, u0 + n, ua, ub, has_b, step);
    if (!produce_pair(ua, ub, has_b, n_blk, n_st, ring, n_ring, P, S, A)) return false;
  }
  return true;
}

// ------------------------------------------------------------------ consumers
struct Consumer {
  int slot = 0;
  unsigned phase = 0;  // ring parity
  int pb = 0;
  int rot = 0;
  unsigned item = 0;   // slots consumed so far (team of a slot = item % kTeams)
};

DPUF_DEV void cbar() { named_sync(kBarConsumers, kConsumers); }
// Barrier of the consumer threads that also returns whether any of them passed true.
DPUF_DEV bool cbar_or(bool v) {
  unsigned r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 q, %1, 0; bar.red.or.pred p, %2, %3, q; selp.u32 %0, 1, 0, p; }"
      : "=r"(r)
      : "r"((unsigned)v), "r"(kBarConsumers), "r"(kConsumers)
      : "memory");
  return r != 0;
}

// Dot warp w: blocks 4w..4w+3 of both units of the slot; lane = (unit lane/16, row lane%16)
// computes dot = sum_k u_k q_k with dp4a on the row's nibbles (low nibbles against x bytes
// 8c..8c+3, high against 8c+4..8c+7) and stores p = float(dot - xm), s = ws * xs (0, 0 for
// a skipped block) at buf[unit][row][block].  kAll: all four blocks exist (a full stage), so
// the four independent computations are scheduled together without guards.
DPUF_DEV float2 dot_pair(const unsigned char* wb, const unsigned char* sb, const int8_t* xq, const float* xs,
                         const int* xm, int b0, int bb) {
  const int4 xa = *(const int4*)(xq + (b0 + bb) * 32), xc = *(const int4*)(xq + (b0 + bb) * 32 + 16);
  const uint32_t w0 = *(const uint32_t*)(wb + bb * 128), w1 = *(const uint32_t*)(wb + bb * 128 + 32);
  const uint32_t w2 = *(const uint32_t*)(wb + bb * 128 + 64), w3 = *(const uint32_t*)(wb + bb * 128 + 96);
  int d0 = __dp4a((int)(w0 & 0x0F0F0F0Fu), xa.x, 0);
  int d1 = __dp4a((int)((w0 >> 4) & 0x0F0F0F0Fu), xa.y, 0);
  d0 = __dp4a((int)(w1 & 0x0F0F0F0Fu), xa.z, d0);
  d1 = __dp4a((int)((w1 >> 4) & 0x0F0F0F0Fu), xa.w, d1);
  d0 = __dp4a((int)(w2 & 0x0F0F0F0Fu), xc.x, d0);
  d1 = __dp4a((int)((w2 >> 4) & 0x0F0F0F0Fu), xc.y, d1);
  d0 = __dp4a((int)(w3 & 0x0F0F0F0Fu), xc.z, d0);
  d1 = __dp4a((int)((w3 >> 4) & 0x0F0F0F0Fu), xc.w, d1);
  const int b = b0 + bb;
  const float bsc = xs[b];
  const float ws = f16bits_to_f32(*(const uint16_t*)(sb + bb * 16));
  const float2 pr = make_float2((float)(d0 + d1 - xm[b]), __fmul_rn(ws, bsc));
  return bsc > 0.0f ? pr : make_float2(0.0f, 0.0f);
}

template <bool kAll>
DPUF_DEV void dot_stage(const unsigned char* st, const int8_t* xq, const float* xs, const int* xm, int b0, int kb,
                        bool has_b, int warp, int lane, float2* buf) {
  const int unit = lane >> 4, r = lane & 15, g = r >> 3, ri = r & 7;
  if (unit == 1 && !has_b) return;
  const unsigned char* ut = st + unit * kHalf;
  const unsigned char* wb = ut + (g ? kNib1 : 0) + ri * 4;
  const unsigned char* sb = ut + (g ? kSc1 : kSc0) + ri * 2;
  float2* o = buf + (unit * 16 + r) * kPsRow + warp * 4;
  if (kAll) {
    float2 pr[4];
#pragma unroll
    for (int j = 0; j < 4; j++) pr[j] = dot_pair(wb, sb, xq, xs, xm, b0, warp * 4 + j);
    *(float4*)o = make_float4(pr[0].x, pr[0].y, pr[1].x, pr[1].y);
    *(float4*)(o + 2) = make_float4(pr[2].x, pr[2].y, pr[3].x, pr[3].y);
  } else {
    for (int j = 0; j < 4; j++)
      if (warp * 4 + j < kb) o[j] = dot_pair(wb, sb, xq, xs, xm, b0, warp * 4 + j);
  }
}

DPUF_DEV void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// One projection on the consumer side.
DPUF_DEV void consume_phase(const DecodeArgs& A, const DecLayer& Ly, int kind, unsigned gen, Consumer& C,
                            unsigned char* ring, int n_ring, const int8_t* xq, const float* xs, const int* xm,
                            float2* ps, DecShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, r = lane & 15;
  int u0, n;
  take_range(A, kind_units(A, kind), C.rot, u0, n);
  const int n_blk = kind_cols(A, kind) >> 5, n_st = (n_blk + 31) >> 5;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int u = u0, step = 1; u < u0 + n; u += step) {
    Unit ua, ub;
    bool has_b;
    pair_of(A, Ly, kind, u, u0 + n, ua, ub, has_b, step);
    float acc = 0.0f;
    for (int s = 0; s < n_st; s++) {
      const int kb = min(32, n_blk - s * 32);
      float2* buf = ps + C.pb * kPsBuf;
      if (warp < kMmaWarps) {
        if ((int)(C.item % kTeams) == warp / kTeamWarps) {
          const int wt = warp % kTeamWarps;
          bool ok = true;
          if (lane == 0) ok = wait_bar(&S.full[C.slot], C.phase, S, A);
          named_sync(kBarEmptied + C.pb, kHandoff);  // the chain is done with this pair buffer
          if (__shfl_sync(kFull, (int)ok, 0)) {
            if (kb == 32)
              dot_stage<true>(ring + (size_t)C.slot * kSlotBytes, xq, xs, xm, s * 32, kb, has_b, wt, lane, buf);
            else
              dot_stage<false>(ring + (size_t)C.slot * kSlotBytes, xq, xs, xm, s * 32, kb, has_b, wt, lane, buf);
          }
          __syncwarp();
          named_arrive(kBarFilled + C.pb, kHandoff);
          if (lane == 0) mbar_arrive(&S.empty[C.slot]);
        }
      } else {
        named_sync(kBarFilled + C.pb, kHandoff);  // the dot warps filled this pair buffer
        if (!S.abort && (half == 0 || has_b)) {
          const float2* row = buf + (half * 16 + r) * kPsRow;
          if (kb == 32) {
            // all 32 pairs are loaded (two per 16-byte load) before the chain starts
            float4 v[16];
#pragma unroll
            for (int q = 0; q < 16; q++) v[q] = *(const float4*)(row + 2 * q);
#pragma unroll
            for (int q = 0; q < 16; q++) {
              acc = __fmaf_rn(v[q].x, v[q].y, acc);
              acc = __fmaf_rn(v[q].z, v[q].w, acc);
            }
          } else {
            for (int b = 0; b < kb; b++) {
              const float2 v = row[b];
              acc = __fmaf_rn(v.x, v.y, acc);
            }
          }
        }
        named_arrive(kBarEmptied + C.pb, kHandoff);
      }
      C.item++;
      if (++C.slot == n_ring) {
        C.slot = 0;
        C.phase ^= 1u;
      }
      if (++C.pb == kNPs) C.pb = 0;
    }
    // ---- epilogue of the pair (chain warp: lanes 0..15 unit A's rows, 16..31 unit B's)
    if (warp == kChainWarp) {
      if (kind == kGU) {
        const float up = __shfl_down_sync(kFull, acc, 16);
        if (half == 0 && r < ua.n_r) {
          const int row = ua.row + r;
          put_tagged(A, A.s_out + row,
                     tagged(swiglu_one(acc, up, A.deadzone, swiglu_vector_elem(row, A.I, A.nt_ref, false), A.et),
                            gen));
        }
      } else if (half == 0 || has_b) {
        const Unit& un = half ? ub : ua;
        if (r < un.n_r) {
          if (kind == kLM) {
            if (A.write_logits) put_float(A, un.out + r, acc);
            better(bv, bi, acc, un.row + r);
          } else {
            put_tagged(A, un.tout + r, tagged(acc, gen));
          }
        }
      }
    }
  }
  if (kind == kLM && warp == kChainWarp) {
    for (int m = 16; m; m >>= 1) {
      const float ov = __shfl_xor_sync(kFull, bv, m);
      const int oi = __shfl_xor_sync(kFull, bi, m);
      better(bv, bi, ov, oi);
    }
    // other ranks' hosts read this CTA's logits once they have seen its partial
    if (A.tp_world > 1 && A.write_logits) __threadfence_system();
    if (lane == 0) {
      const int g_all = gridDim.x * A.tp_world;
      uint64_t* pw = A.part + ((size_t)(gen & 1) * g_all + A.tp_rank * gridDim.x + blockIdx.x) * 2;
      put_tagged(A, pw, tagged(bv, gen));
      put_tagged(A, pw + 1, ((uint64_t)gen << 32) | (unsigned)bi);
    }
  }
  if (warp == kChainWarp) {
    __syncwarp();
    if (lane == 0) count_done(A, 0);
  }
}

// Bounded poll by one thread until a counter has reached `target` (wrap-safe), the CTA or
// another CTA (or rank) has aborted, or the wait limit has passed (error word 2).
DPUF_DEV void wait_count(const DecodeArgs& A, const unsigned* ctr, unsigned target, DecShared& S) {
  unsigned long long t0 = 0;
  const unsigned long long limit = A.tp_world > 1 ? kTpWaitNs : kWaitNs;
  for (int it = 0; !S.abort; it++) {
    if ((int)(ld_acquire(ctr) - target) >= 0) break;
    if (*(volatile int*)A.err) {
      S.abort = 1;
      break;
    }
    if ((it & 15) == 15) {
      const unsigned long long now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit) {
        raise_err(A, 2);
        S.abort = 1;
        break;
      }
    }
    __nanosleep(20);
  }
}

// Grid-wide barrier of the consumer threads of this GPU (the producer never joins): arrive on
// a global counter (release) and wait, bounded, until every CTA has arrived `target /
// gridDim.x` times (acquire).
DPUF_DEV void grid_sync(const DecodeArgs& A, unsigned& target, DecShared& S) {
  cbar();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(A.bar) : "memory");
    wait_count(A, A.bar, target, S);
  }
  cbar();
}

// Async copies by the consumer threads into shared memory: 16-byte pieces through L2 (data
// other CTAs wrote; bytes % 16 == 0) and 8-byte pieces of read-only tables (bytes % 8 == 0).
DPUF_DEV void stage16(void* dst, const void* src, int bytes) {
  for (int i = threadIdx.x * 16; i < bytes; i += kConsumers * 16)
    cp_async16_cg((unsigned char*)dst + i, (const unsigned char*)src + i);
}
DPUF_DEV void stage8(void* dst, const void* src, int bytes) {
  for (int i = threadIdx.x * 8; i < bytes; i += kConsumers * 8)
    cp_async8_ca((unsigned char*)dst + i, (const unsigned char*)src + i);
}

// Stages words [0, n) (n even) of a tagged vector that other CTAs (or ranks) produce in
// generation `gen`, together with whatever async copies the caller has issued (all consumer
// threads call this).  Each thread copies its 16-byte pieces and waits; if any thread finds a
// piece that predates `gen`, thread 0 alone waits (bounded) until completion counter ctr_i
// reaches `target`, then every thread re-copies its stale pieces, and repeats (waiting on its
// first stale piece itself) until no thread has one.  On return every staged word carries
// `gen` (or the CTA has aborted) and the consumer threads have passed a CTA barrier.
DPUF_DEV void stage_tagged(uint64_t* dst, const uint64_t* src, int n, unsigned gen, int ctr_i, unsigned target,
                           const DecodeArgs& A, DecShared& S) {
  for (int i = threadIdx.x * 2; i < n; i += kConsumers * 2) cp_async16_cg(dst + i, src + i);
  cp_async_commit_wait_all();
  auto first_stale = [&]() {
    for (int i = threadIdx.x * 2; i < n; i += kConsumers * 2) {
      const ulonglong2 w = *(const ulonglong2*)(dst + i);
      if (tag_of(w.x) != gen || tag_of(w.y) != gen) return i;
    }
    return -1;
  };
  int first = first_stale();
  if (!cbar_or(first >= 0)) return;
  if (threadIdx.x == 0) wait_count(A, A.ctr + ctr_i, target, S);
  cbar();
  for (int round = 0;; round++) {
    if (first >= 0 && !S.abort) {
      if (round > 0) *(ulonglong2*)(dst + first) = wait_tagged2(src + first, gen, A, S);
      for (int i = first; i < n; i += kConsumers * 2) {
        const ulonglong2 w = *(const ulonglong2*)(dst + i);
        if (tag_of(w.x) != gen || tag_of(w.y) != gen) cp_async16_cg(dst + i, src + i);
      }
      cp_async_commit_wait_all();
      first = first_stale();
    }
    if (!cbar_or(first >= 0 && !S.abort)) return;
  }
}

// Residual add, RMSNorm and activation prep of the result (add_and_rms_norm_f32 /
// rms_norm_f32, dpuf_engine.c:225-272, then the prep).  The residual (optional; tagged words of
// generation `gen` from other CTAs; rows >= n_valid add 0, as the pruned down projection's
// zero rows do), the gains and the sign bytes are staged in one async round (plus re-copies
// of residual words staged before they were produced); all threads add the residual, then
// threads 0..7 run the eight "AVX lane" chains over h after the residual add, 32 elements at
// a time.
DPUF_DEV void norm_prep(const DecodeArgs& A, float* h, const uint64_t* res, unsigned gen, int n_valid, const float* w,
                        int H, float eps, const uint8_t* signs, int8_t* xq, float* xs, int* xm, float* stage,
                        DecShared& S) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* sr = (uint64_t*)stage;  // [H] tagged residual
  float* sw = stage + 2 * H;         // [H] gains
  uint8_t* sg = (uint8_t*)(stage + 3 * H);
  stage16(sw, w, H * 4);
  if (signs) stage8(sg, signs, H / 8);
  if (res)
    stage_tagged(sr, res, min(H, n_valid), gen, 0, gen * (unsigned)(gridDim.x * A.tp_world), A, S);
  else
    cp_async_commit_wait_all();
  cbar();
  if (res) {
    for (int i = tid; i < H; i += kConsumers) h[i] = __fadd_rn(h[i], i < n_valid ? value_of(sr[i]) : 0.0f);
    cbar();
  }
  if (tid < 8) S.lanes[tid] = sumsq_lane32(h, H & ~7, tid);
  cbar();
  if (tid == 0) S.inv = rms_inv(S.lanes, h, H, eps);
  cbar();
  const float inv = S.inv;
  const int nch = H / 64;
  for (int cb = warp * 4; cb < nch; cb += kConsumers / 8) {
    const int c = cb + (lane >> 3);
    const bool active = c < nch;
    const int col = (active ? c * 64 : 0) + (lane & 7) * 8;
    float v[8];
    const float4 h0 = *(const float4*)(h + col), h1 = *(const float4*)(h + col + 4);
    const float4 w0 = *(const float4*)(sw + col), w1 = *(const float4*)(sw + col + 4);
    v[0] = __fmul_rn(__fmul_rn(h0.x, inv), w0.x);
    v[1] = __fmul_rn(__fmul_rn(h0.y, inv), w0.y);
    v[2] = __fmul_rn(__fmul_rn(h0.z, inv), w0.z);
    v[3] = __fmul_rn(__fmul_rn(h0.w, inv), w0.w);
    v[4] = __fmul_rn(__fmul_rn(h1.x, inv), w1.x);
    v[5] = __fmul_rn(__fmul_rn(h1.y, inv), w1.y);
    v[6] = __fmul_rn(__fmul_rn(h1.z, inv), w1.z);
    v[7] = __fmul_rn(__fmul_rn(h1.w, inv), w1.w);
    prep_chunk_g8(v, signs ? sg[col >> 3] : 0, active, active ? c * 64 : 0, lane, xq, xs, xm);
  }
}

// Distributed prep of the gate/up output (tagged words of generation `gen`) for the down
// projection: 64-column chunk ch is prepped by one CTA of all ranks (virtual CTA ch mod the
// CTA count; eight lanes per chunk, so a warp preps four).  One GPU: the CTA stores the codes,
// block scales and block sums as plain values, read by every CTA after a grid barrier.
// Several ranks: it publishes them to every rank as tagged words of the same generation (four
// codes per word) and counts its prep on completion counter 1.
DPUF_DEV void prep_slices(const DecodeArgs& A, const uint8_t* signs, unsigned gen, DecShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x * A.tp_world, vc = blockIdx.x * A.tp_world + A.tp_rank;
  const int nch = A.I / 64;
  uint64_t* dq = A.dprep;
  uint64_t* ds = dq + A.I / 4;
  uint64_t* dm = ds + A.I / 32;
  for (int k0 = warp * 4; vc + k0 * G < nch; k0 += kConsumers / 8) {
    const int ch = vc + (k0 + (lane >> 3)) * G;
    const bool active = ch < nch;
    const int col = (active ? ch : 0) * 64 + (lane & 7) * 8;
    const uint8_t sbyte = (active && signs) ? __ldg(signs + (col >> 3)) : 0;  // issued before the waits
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      ulonglong2 w = make_ulonglong2(0, 0);
      if (active) {
        w = ld_tagged2(A.s_out + col + j, A.tp_world > 1);
        if (tag_of(w.x) != gen || tag_of(w.y) != gen) w = wait_tagged2(A.s_out + col + j, gen, A, S);
      }
      v[j] = value_of(w.x);
      v[j + 1] = value_of(w.y);
    }
    const PrepOut o = prep_chunk_g8_core(v, sbyte, lane);
    if (active && A.tp_world == 1) {
      *(uint2*)(A.xd_q8 + col) = make_uint2(o.lo, o.hi);
      if ((lane & 3) == 0) {
        A.xd_xs[col >> 5] = o.xs;
        A.xd_xm[col >> 5] = o.xm;
      }
    } else if (active) {
      const uint64_t tg = (uint64_t)gen << 32;
      put_tagged(A, dq + col / 4, tg | o.lo);
      put_tagged(A, dq + col / 4 + 1, tg | o.hi);
      if ((lane & 3) == 0) {
        put_tagged(A, ds + (col >> 5), tagged(o.xs, gen));
        put_tagged(A, dm + (col >> 5), tg | (unsigned)o.xm);
      }
    }
  }
  if (A.tp_world > 1) {
    cbar();
    if (threadIdx.x == 0) count_done(A, 1);
  }
}

// The down projection's prepped input (prep_slices, generation `gen`, the `dgen`-th prep) into
// x: the tagged words are staged, then unpacked to codes, block scales and block sums.
// K % 64 == 0.
DPUF_DEV void load_prepped_tagged(const DecodeArgs& A, int K, unsigned gen, unsigned dgen, int8_t* xq, float* xs,
                                  int* xm, float* stage, DecShared& S) {
  uint64_t* st = (uint64_t*)stage;
  const int nq = K / 4, nb = K / 32;
  // the chunks are published by all CTAs at about the same time, shortly after this CTA's own:
  // wait for the count first, so that the one staging round finds them
  const unsigned target = dgen * (unsigned)(gridDim.x * A.tp_world);
  if (threadIdx.x == 0) wait_count(A, A.ctr + 1, target, S);
  cbar();
  stage_tagged(st, A.dprep, nq + 2 * nb, gen, 1, target, A, S);
  cbar();
  for (int i = threadIdx.x; i < nq; i += kConsumers) *(uint32_t*)(xq + 4 * i) = (uint32_t)st[i];
  for (int b = threadIdx.x; b < nb; b += kConsumers) {
    xs[b] = value_of(st[nq + b]);
    xm[b] = (int)(unsigned)st[nq + nb + b];
  }
}

// Prep of a whole tagged vector (generation `gen`, complete at count `target` of completion
// counter 0) by this CTA: staged in one piece with its sign bytes, then prepped from shared
// memory (for vectors small enough that one hop beats the distributed prep's two).
DPUF_DEV void prep_tagged(const DecodeArgs& A, const uint64_t* src, unsigned gen, unsigned target, int K,
                          const uint8_t* signs, int8_t* xq, float* xs, int* xm, float* stage, DecShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* st = (uint64_t*)stage;
  uint8_t* sg = (uint8_t*)(st + K);
  if (signs) stage8(sg, signs, K / 8);
  stage_tagged(st, src, K, gen, 0, target, A, S);
  const int nch = K / 64;
  for (int cb = warp * 4; cb < nch; cb += kConsumers / 8) {
    const int c = cb + (lane >> 3);
    const bool active = c < nch;
    const int col = (active ? c * 64 : 0) + (lane & 7) * 8;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = value_of(st[col + k]);
    prep_chunk_g8(v, signs ? sg[col >> 3] : 0, active, active ? c * 64 : 0, lane, xq, xs, xm);
  }
}

// Copies a prepped activation (codes, block scales, block sums of K columns; K % 128 == 0)
// written by other CTAs into x.
DPUF_DEV void load_prepped(const int8_t* q8, const float* bxs, const int32_t* bxm, int K, int8_t* xq, float* xs,
                           int* xm) {
  stage16(xq, q8, K);
  stage16(xs, bxs, K / 8);
  stage16(xm, bxm, K / 8);
  cp_async_commit_wait_all();
}

// Activation prep of a vector written by other CTAs before a grid barrier: pieces of `cap`
// columns (a multiple of 128) are staged into shared memory with their sign bytes, then
// prepped from there.
DPUF_DEV void prep_global(const float* src, int K, const uint8_t* signs, int8_t* xq, float* xs, int* xm, float* stage,
                          int cap) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* sg = (uint8_t*)(stage + cap);
  for (int p0 = 0; p0 < K; p0 += cap) {
    const int n = min(cap, K - p0);
    stage16(stage, src + p0, n * 4);
    if (signs) stage8(sg, signs + p0 / 8, n / 8);
    cp_async_commit_wait_all();
    cbar();
    const int nch = n / 64;
    for (int cb = warp * 4; cb < nch; cb += kConsumers / 8) {
      const int c = cb + (lane >> 3);
      const bool active = c < nch;
      const int col = (active ? c * 64 : 0) + (lane & 7) * 8;
      const float4 a0 = *(const float4*)(stage + col), a1 = *(const float4*)(stage + col + 4);
      float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      prep_chunk_g8(v, signs ? sg[col >> 3] : 0, active, p0 + (active ? c * 64 : 0), lane, xq, xs, xm);
    }
    cbar();
  }
}

struct AttnSync {
  DPUF_DEV void operator()() const { named_sync(kBarAttn, kAttnThreads); }
};

// Attention items (KV head, query-head pair) of this CTA: the pair's query heads, the KV
// head's key and value, the QK-norm gains and the RoPE row are staged in one async round;
// QK-norm + RoPE of the queries and the key, K/V rows stored at `pos` (both pairs of a KV head
// store the same bits), then attn_pair_body.  With fuse_o the item also preps its output
// columns (whole 64-column chunks) for the o projection.  Threads 0..255 only.
DPUF_DEV void attention_items(const DecodeArgs& A, const DecLayer& Ly, int l, int pos, unsigned gen, float* scratch,
                              DecShared& S) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int groups = A.nq / A.nkv, n_pairs = (groups + 1) / 2, hd = A.hd;
  // scratch: qs [2][hd] | inputs (key, value, gains, RoPE row) [5 hd] | scores [2][kv_len
  // padded to 4] | n_buf key/value tiles (as many as fit, at most kAttnMaxBuf)
  const int kv_len = pos + 1, sc_stride = (kv_len + 3) & ~3;
  float* qs = scratch;
  float *kin = qs + 2 * hd, *vin = kin + hd, *qn = vin + hd, *kn = qn + hd, *cs = kn + hd, *sn = cs + hd / 2;
  float* sc = qs + 7 * hd;
  float* kt = sc + 2 * sc_stride;
  const int n_t = (kv_len + kAttnKeyTile - 1) / kAttnKeyTile;
  const int n_buf = max(1, min(kAttnMaxBuf, (int)((A.attn_floats - 7 * hd - 2 * sc_stride) / attn_tile_floats(hd))));
  const int pre = min(n_buf, n_t);  // history key tiles fetched while q/k/v arrive
  for (int it = blockIdx.x; it < A.nkv * n_pairs; it += gridDim.x) {
    const int kvh = it / n_pairs, pr = it % n_pairs;
    const int g0 = pr * 2, nh = (g0 + 1 < groups) ? 2 : 1, qh0 = kvh * groups + g0;
    float* kc = A.kv_k + ((size_t)l * A.nkv + kvh) * A.S * hd;
    float* vc = A.kv_v + ((size_t)l * A.nkv + kvh) * A.S * hd;
    named_sync(kBarAttn, kAttnThreads);  // scratch free (previous item done)
    {
      const int q4 = hd / 4;  // 16-byte pieces per vector
      // gains and the RoPE row asynchronously (one group), then the first key tiles of the
      // history (rows < pos: they do not depend on this step), while the pair's query heads,
      // the key and the value (tagged words of the q/k/v phase) are read, one pair of
      // elements per thread
      for (int i = tid; i < q4; i += kAttnThreads) {
        if (Ly.q_norm) cp_async16_cg(qn + i * 4, Ly.q_norm + i * 4);
        if (Ly.k_norm) cp_async16_cg(kn + i * 4, Ly.k_norm + i * 4);
        if (i < q4 / 2) {
          cp_async16_cg(cs + i * 4, A.cos_tab + (size_t)pos * (hd >> 1) + i * 4);
          cp_async16_cg(sn + i * 4, A.sin_tab + (size_t)pos * (hd >> 1) + i * 4);
        }
      }
      cp_async_commit();
      for (int t = 0; t < pre; t++) attn_issue_tile(kt + (size_t)t * attn_tile_floats(hd), kc, t, pos, hd, tid);
      for (int i = tid * 2; i < (nh + 2) * hd; i += kAttnThreads * 2) {
        const int v = i / hd, o = i % hd;
        const uint64_t* src = (v < nh ? A.q + (size_t)(qh0 + v) * hd : (v == nh ? A.k : A.v) + (size_t)kvh * hd) + o;
        float* dst = (v < nh ? qs + v * hd : (v == nh ? kin : vin)) + o;
        ulonglong2 w = ld_tagged2(src, A.tp_world > 1);
        if (tag_of(w.x) != gen || tag_of(w.y) != gen) w = wait_tagged2(src, gen, A, S);
        *(float2*)dst = make_float2(value_of(w.x), value_of(w.y));
      }
      cp_async_wait_pending(pre);  // the gains and the RoPE row (the tiles may stay in flight)
    }
    named_sync(kBarAttn, kAttnThreads);
    if (warp == 0) {
      qk_norm_rope_warp(kin, Ly.k_norm ? kn : nullptr, A.eps, hd, cs, sn, lane);
      for (int i = lane; i < hd; i += 32) kc[(size_t)pos * hd + i] = kin[i];
    } else if (warp == 1) {
      for (int i = lane; i < hd; i += 32) vc[(size_t)pos * hd + i] = vin[i];
    } else if (warp < 2 + nh) {
      qk_norm_rope_warp(qs + (warp - 2) * hd, Ly.q_norm ? qn : nullptr, A.eps, hd, cs, sn, lane);
    }
    named_sync(kBarAttn, kAttnThreads);  // rotated queries and key in place
    attn_pair_body(qs, nh, nh == 1, hd, kv_len, kc, vc, sc_stride, sc, kt, n_buf, pre, kin, vin, &S.attn,
                   A.att + (size_t)qh0 * hd, A.et, tid, AttnSync{}, A.fuse_o != 0);
    if (A.fuse_o) {
      named_sync(kBarAttn, kAttnThreads);
      const int n_ch = nh * hd / 64;
      if (warp * 4 < n_ch) {
        const int c = warp * 4 + (lane >> 3);
        const bool active = c < n_ch;
        const int col = (active ? c * 64 : 0) + (lane & 7) * 8;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = qs[col + k];
        const int gcol = qh0 * hd + col;  // column of the o-projection input
        prep_chunk_g8(v, Ly.signs[1] ? Ly.signs[1][gcol >> 3] : 0, active, qh0 * hd + (active ? c * 64 : 0), lane,
                      A.xo_q8, A.xo_xs, A.xo_xm);
      }
    }
  }
}

// Optional trace of the last step: per CTA, the time (globaltimer, ns) at which each phase of
// the consumer side ended (14 per layer, then 6 per step) and at which the producer began each
// projection (4 per layer + the LM head).
enum {
  kEvNorm1, kEvQKV, kEvB1, kEvAttn, kEvB2, kEvPrepO, kEvO, kEvB3, kEvNorm2, kEvGU, kEvB4, kEvPrepD, kEvDown, kEvB5,
  kEvPerLayer
};
enum { kEvStart, kEvEmbed, kEvNormF, kEvLM, kEvBLM, kEvArg, kEvPerStep };
DPUF_DEV void trace_at(const DecodeArgs& A, int step, int ev) {
  if (A.trace && step == A.n_steps - 1) A.trace[(size_t)blockIdx.x * A.trace_per_cta + ev] = globaltimer();
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(DecodeArgs A) {
  static_assert(kAttnThreads <= kTeamWarps * 32, "attention runs on the first team");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ DecShared S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_ring = A.n_ring;
  unsigned char* ring = smem;
  DecLayer* layers = (DecLayer*)(smem + (size_t)n_ring * kSlotBytes);
  float* h = (float*)(layers + max(A.L, 1));
  unsigned char* uni = (unsigned char*)(h + A.H);
  int8_t* xq = (int8_t*)uni;
  float* xs = (float*)(uni + A.kmax);
  int* xm = (int*)(xs + A.kmax / 32);
  float2* ps = (float2*)(xm + A.kmax / 32);
  float* stage = (float*)(xm + A.kmax / 32);  // staging area (overlaps the pair buffers)
  float* attn_scratch = (float*)uni;

  if (tid == 0) {
    for (int i = 0; i < n_ring; i++) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], kTeamWarps);
    }
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  {
    const int4* src = (const int4*)A.layers;
    int4* dst = (int4*)layers;
    for (int i = tid; i < A.L * (int)(sizeof(DecLayer) / 16); i += kThreads) dst[i] = src[i];
  }
  __syncthreads();

  // ---------------------------------------------------------------- producer warp
  if (warp == kProdWarp) {
    if (lane != 0) return;
    Producer P;
    P.policy = l2_evict_first_policy();
    int rot = 0;
    bool ok = true;
    const int ev0 = kEvPerLayer * A.L + kEvPerStep;
    for (int step = 0; ok && step < A.n_steps; step++) {
      for (int l = 0; ok && l < A.L; l++)
        for (int kind = kQKV; ok && kind <= kDown; kind++) {
          trace_at(A, step, ev0 + 4 * l + kind);
          ok = produce_phase(A, layers, l, kind, rot, ring, n_ring, P, S);
        }
      trace_at(A, step, ev0 + 4 * A.L);
      if (ok) ok = produce_phase(A, layers, 0, kLM, rot, ring, n_ring, P, S);
    }
    if (!ok) {
      // copies still in flight must land before the CTA exits: wait (bounded) for the last
      // use of every slot
      const unsigned long long t0 = globaltimer();
      for (int sl = 0; sl < n_ring; sl++) {
        const long long uses = P.issued / n_ring + (sl < P.issued % n_ring ? 1 : 0);
        if (uses == 0) continue;
        const unsigned par = (unsigned)((uses - 1) & 1);
        while (!mbar_try(&S.full[sl], par) && globaltimer() - t0 < kWaitNs) {
        }
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumer warps
  // Pair-buffer hand-off on named barriers: the dot warps bar.sync "emptied" before filling a
  // buffer and bar.arrive "filled"; the chain warp bar.syncs "filled" and bar.arrives
  // "emptied".  The chain's first arrivals here free every buffer; the dot warps' syncs at the
  // end take its last ones, so every barrier generation completes.
  if (warp == kChainWarp)
    for (int i = 0; i < kNPs; i++) named_arrive(kBarEmptied + i, kHandoff);
  Consumer C;
  unsigned target = 0;
  const int H = A.H;
  const int n_chunks = A.H / 64;
  for (int step = 0; step < A.n_steps; step++) {
    const int pos = A.pos0 + step;
    const int id = step == 0 ? A.first_id : S.next_id;
    const int sb = kEvPerLayer * A.L;
    if (tid == 0) trace_at(A, step, sb + kEvStart);
    // embedding row -> h: the row's 8-row group of its tile and the sign table are staged in
    // shared memory, then every warp expands its chunks from there
    {
      const int n_blk = H >> 5, lr = id % kTileRows;
      const uint8_t* grp = A.tok_tiles + (size_t)(id / kTileRows) * A.tok_stride + 16 + (size_t)(lr >> 3) * n_blk * 144;
      uint8_t* sgrp = (uint8_t*)stage;
      uint8_t* sg = sgrp + n_blk * 144;
      stage16(sgrp, grp, n_blk * 144);
      if (A.tok_signs) stage8(sg, A.tok_signs, H / 8);
      cp_async_commit_wait_all();
      cbar();
      for (int c = warp; c < n_chunks; c += kConsumers / 32) {
        float a, b;
        embed_chunk_warp(sgrp - 16, n_blk, lr & 7, A.tok_signs ? sg : nullptr, c * 64, lane, a, b);
        h[c * 64 + lane] = a;
        h[c * 64 + 32 + lane] = b;
      }
    }
    cbar();
    if (tid == 0) trace_at(A, step, sb + kEvEmbed);
    // exchange generations: 4 per layer (q/k/v, o, gate/up, down) and the LM head's
    const unsigned g_step = A.gen0 + (unsigned)step * (unsigned)decode_phases(A.L);
    for (int l = 0; l < A.L; l++) {
      const DecLayer& Ly = layers[l];
      const int lb = kEvPerLayer * l;
      const unsigned g = g_step + 4u * l;
      // the previous layer's down output (generation g - 1) is the residual
      norm_prep(A, h, l > 0 ? A.d_out : nullptr, g - 1, A.keep_down * kTileRows, Ly.attn_norm, H, A.eps, Ly.signs[0],
                xq, xs, xm, stage, S);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvNorm1);
      consume_phase(A, Ly, kQKV, g + kQKV, C, ring, n_ring, xq, xs, xm, ps, S);
      if (tid == 0) trace_at(A, step, lb + kEvQKV);
      cbar();  // the attention scratch overlaps the pair buffers
      if (tid == 0) trace_at(A, step, lb + kEvB1);
      if (tid < kAttnThreads) attention_items(A, Ly, l, pos, g + kQKV, attn_scratch, S);
      if (tid == 0) trace_at(A, step, lb + kEvAttn);
      grid_sync(A, target, S);
      if (tid == 0) trace_at(A, step, lb + kEvB2);
      if (A.fuse_o)
        load_prepped(A.xo_q8, A.xo_xs, A.xo_xm, A.qd, xq, xs, xm);
      else
        prep_global(A.att, A.qd, Ly.signs[1], xq, xs, xm, stage, A.stage_cap);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvPrepO);
      consume_phase(A, Ly, kO, g + kO, C, ring, n_ring, xq, xs, xm, ps, S);
      if (tid == 0) trace_at(A, step, lb + kEvO);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvB3);
      norm_prep(A, h, A.o_out, g + kO, H, Ly.ffn_norm, H, A.eps, Ly.signs[2], xq, xs, xm, stage, S);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvNorm2);
      consume_phase(A, Ly, kGU, g + kGU, C, ring, n_ring, xq, xs, xm, ps, S);
      if (tid == 0) trace_at(A, step, lb + kEvGU);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvB4);
      if (A.dprep_local) {
        prep_tagged(A, A.s_out, g + kGU, (g + kGU) * (unsigned)(gridDim.x * A.tp_world), A.I, Ly.signs[3], xq, xs,
                    xm, stage, S);
      } else {
        prep_slices(A, Ly.signs[3], g + kGU, S);
        if (A.tp_world == 1) {
          grid_sync(A, target, S);
          load_prepped(A.xd_q8, A.xd_xs, A.xd_xm, A.I, xq, xs, xm);
        } else {
          load_prepped_tagged(A, A.I, g + kGU, A.dgen0 + (unsigned)(step * A.L + l + 1), xq, xs, xm, stage, S);
        }
      }
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvPrepD);
      consume_phase(A, Ly, kDown, g + kDown, C, ring, n_ring, xq, xs, xm, ps, S);
      if (tid == 0) trace_at(A, step, lb + kEvDown);
      cbar();
      if (tid == 0) trace_at(A, step, lb + kEvB5);
    }
    const unsigned g_lm = g_step + 4u * A.L;
    norm_prep(A, h, A.L > 0 ? A.d_out : nullptr, g_lm - 1, A.keep_down * kTileRows, A.out_norm, H, A.eps, A.lm_signs,
              xq, xs, xm, stage, S);
    cbar();
    if (tid == 0) trace_at(A, step, sb + kEvNormF);
    consume_phase(A, layers[0], kLM, g_lm, C, ring, n_ring, xq, xs, xm, ps, S);
    if (tid == 0) trace_at(A, step, sb + kEvLM);
    cbar();
    if (tid == 0) trace_at(A, step, sb + kEvBLM);
    {
      // every CTA's partial (of every rank), tagged with the LM generation, read by all
      // consumer threads; the two partial buffers alternate with the generation's parity, so
      // a CTA already at the next step's LM head never overwrites a partial another CTA has
      // yet to read
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      const int g_all = gridDim.x * A.tp_world;
      const uint64_t* part = A.part + (size_t)(g_lm & 1) * g_all * 2;
      for (int c = tid; c < g_all; c += kConsumers) {
        ulonglong2 w = ld_tagged2(part + 2 * c, A.tp_world > 1);
        if (tag_of(w.x) != g_lm || tag_of(w.y) != g_lm) w = wait_tagged2(part + 2 * c, g_lm, A, S);
        better(bv, bi, value_of(w.x), (int)(unsigned)w.y);
      }
      // the logits other ranks stored before their partials are visible to this rank's host
      if (A.tp_world > 1 && A.write_logits) __threadfence_system();
      for (int m = 16; m; m >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, m);
        const int oi = __shfl_xor_sync(kFull, bi, m);
        better(bv, bi, ov, oi);
      }
      if (lane == 0) {
        S.arg_v[warp] = bv;
        S.arg_i[warp] = bi;
      }
      cbar();
      if (tid == 0) {
        for (int w = 1; w < kConsumers / 32; w++) better(bv, bi, S.arg_v[w], S.arg_i[w]);
        // the winner is a row of the head; anything else (all logits NaN, or an aborted run)
        // feeds row 0 so that the embedding lookup stays in bounds
        const int id_next = (bi >= 0 && bi < A.V && bi < A.tok_rows) ? bi : 0;
        S.next_id = id_next;
        if (blockIdx.x == 0) A.hist[step] = id_next;
      }
    }
    if (tid == 0) trace_at(A, step, sb + kEvArg);
    cbar();
  }
  if (warp < kMmaWarps)
    for (int i = 0; i < kNPs; i++) named_sync(kBarEmptied + i, kHandoff);
}

}  // namespace

// Shared memory of one CTA: ring | layer table | h | a union of {activation x + pair buffers
// or staging area} and the attention scratch.  The staging area (after x) holds an embedding
// group with its sign table (4.625 H bytes), a tagged residual with the norm gains and signs
// (12.125 H), the down projection's tagged prepped input (2.5 I) or a piece of a vector being
// prepped (4.125 bytes per column).
size_t decode_x_bytes(const DecodeArgs& A) { return (size_t)A.kmax + (size_t)(A.kmax / 32) * 8; }
size_t decode_uni_bytes(const DecodeArgs& A) {
  const size_t xb = decode_x_bytes(A);
  const size_t uni_x = xb + (size_t)kNPs * kPsBuf * sizeof(float2);
  // tagged residual + gains + signs of a norm, or a whole plain vector of kmax columns with
  // its signs
  const size_t uni_stage =
      xb + std::max((size_t)A.H * 12 + (size_t)A.H / 8, (size_t)A.kmax * 4 + (size_t)A.kmax / 8) + 128;
  const size_t uni_attn = ((size_t)7 * A.hd + attn_sc_floats(A.S) + attn_tile_floats(A.hd)) * sizeof(float);
  return std::max(std::max(uni_x, uni_stage), uni_attn);
}
int decode_stage_cap(const DecodeArgs& A) {
  const size_t bytes = decode_uni_bytes(A) - decode_x_bytes(A);
  return (int)(bytes * 8 / 33 / 128 * 128);  // 4 + 1/8 bytes per column
}
size_t decode_smem_bytes(const DecodeArgs& A) {
  return (size_t)A.n_ring * kSlotBytes + (size_t)std::max(A.L, 1) * sizeof(DecLayer) + (size_t)A.H * 4 +
         decode_uni_bytes(A);
}

int decode_ring_slots(const DecodeArgs& A, size_t smem_limit) {
  DecodeArgs B = A;
  B.n_ring = 0;
  const size_t fixed = decode_smem_bytes(B);
  if (fixed >= smem_limit) return 0;
  return (int)std::min<size_t>(kMaxRing, (smem_limit - fixed) / kSlotBytes);
}

int decode_trace_events(int L) { return kEvPerLayer * L + kEvPerStep + 4 * L + 1; }

cudaError_t configure_decode_kernel() { return set_max_dyn_smem(decode_kernel); }

cudaError_t decode_max_dyn_smem(size_t* bytes) {
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, (const void*)decode_kernel);
  if (e == cudaSuccess) *bytes = (size_t)a.maxDynamicSharedSizeBytes;
  return e;
}

cudaError_t decode_blocks_per_sm(const DecodeArgs& A, int* blocks) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, decode_kernel, kThreads, decode_smem_bytes(A));
}

cudaError_t launch_decode(cudaStream_t stream, const DecodeArgs& A) {
  if (A.n_ring < 2 || A.n_ring > kMaxRing) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)A.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = decode_smem_bytes(A);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_kernel, A);
}

}  // namespace dpuf
