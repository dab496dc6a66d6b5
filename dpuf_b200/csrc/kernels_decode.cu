// kernels_decode.cu - batch-1 decode as one persistent cooperative kernel.
//
// One CTA per SM runs every step of a greedy decode (or one forward_token step): embedding, all
// layers, final norm, LM head and argmax.  The per-element arithmetic is the reference's
// (layer_dev.cuh and the exact block chain below), so logits and ids are bit-identical to the
// reference engine's.
//
// Weight stream.  The weights never depend on activations.  A producer warp (one thread) walks
// the CTA's sequence of stages - every projection of every layer and step - and moves each stage
// (32 blocks of one 8-row group: 512 bytes of fp16 row scales and 4096 bytes of nibbles, two
// cp.async.bulk copies on one mbarrier) into the next slot of a ring shared by the CTA's consumer
// warps, as soon as the slot's previous stage has been released.  So while the consumers
// normalise, attend or wait for another CTA, the ring fills with the next projection's weights.
//
// Projections.  Every consumer warp owns whole units - 8-row groups, or gate/up pairs - of every
// projection (the CTA's contiguous range of units, dealt to its warps in turn); the warps'
// stages are interleaved round by round in the ring, so a phase in which only a few warps have
// units still has the whole ring in flight for them.  Lane (ri = lane % 8, q = lane / 8) of the
// owning warp computes row ri's exact integer block dots of blocks 8q .. 8q+7 of a stage (dp4a on
// the nibbles, chunk reads rotated by q so the four octets use different banks) and the pairs
// (p, s) = (dot - xm, ws * xs); the in-order chain acc = fma(p, s, acc) then runs octet by octet,
// handed on by shuffles (dpuf_avx2.c:2601-2640).  Outputs other CTAs read are stored as tagged
// 64-bit words (value, generation of the layer), so readers wait on exactly the words they need.
//
// Per layer:
//   norm1   every CTA: residual += the previous down output (tagged), RMSNorm, prep -> x
//   q/k/v   projection; outputs tagged
//   attn    one CTA per query head (all its warps): QK-norm, RoPE, K/V store, scores, softmax,
//           PV, and the prep of the head's output columns for the o projection (tagged)
//   o       every CTA loads the prepped o input, projection; outputs tagged
//   norm2   residual += o output, RMSNorm, prep -> x
//   gate/up pairs (gate group and up group of the same rows in one warp), SwiGLU (tagged); the
//           warp holding the last pair of a 64-column chunk preps the chunk for the down
//           projection (tagged)
//   down    every CTA loads the prepped down input, projection; outputs tagged
// then the final norm, the LM head (logits and per-CTA argmax partials, tagged) and the argmax.
//
// Tensor parallelism (tp_world > 1, one process per GPU): every projection's units are dealt over
// all ranks' CTAs; producers store their tagged words into every rank's exchange buffer (peer
// stores over NVLink); every rank normalises and attends over all heads itself, so its KV cache
// stays complete.
//
// Every wait is bounded (wait_ns): a wait that gives up sets the error word (of every rank) and
// the CTA's abort flag, after which waits return at once and the control flow stays uniform (so
// every barrier completes); the producer stops issuing and waits, bounded, for the copies it
// issued before the CTA exits.
#include <algorithm>

#include "kernels.cuh"
#include "layer_dev.cuh"

namespace dpuf {

namespace {


constexpr int kConsWarps = kDecodeConsWarps;   // consumer warps
constexpr int kProdWarp = kConsWarps;           // the producer warp
constexpr int kThreads = (kConsWarps + 1) * 32;  // 384
constexpr int kConsThreads = kConsWarps * 32;    // 352
constexpr int kKB = 32;                // blocks per stage
constexpr int kScBytes = kKB * 16;     // 512: fp16 scales [32][8]
constexpr int kSlotBytes = kScBytes + kKB * 128;  // 4608
constexpr int kMaxSlots = 48;          // ring slots (shared by the CTA's consumer warps)
constexpr int kMailbox = 64;           // accumulator hand-over entries (a power of two)
constexpr int kHandMax = 6;            // at most this many units per CTA: stages spread over all warps
constexpr int kSvUnits = kDecodeSvUnits;  // gate/up units per CTA (their SwiGLU outputs stay in shared memory)
// Bytes of the norm staging at the start of the union (gains, sign bytes), 16-byte rounded.
DPUF_HD size_t decode_norm_stage_bytes(const DecodeArgs& A) {
  return ((size_t)A.H * 4 + (size_t)A.H / 8 + 15) & ~(size_t)15;
}
static_assert(kMailbox >= 2 * kHandMax + kMaxSlots + 1, "hand-over entries must outlive their readers");
constexpr int kChunkWords = 20;        // tagged words of one prepped 64-column chunk
constexpr int kVTile = 8;              // keys per staged value tile (attention)
constexpr int kKeyGroups = kConsThreads / 8;
enum { kQKV = 0, kO = 1, kGU = 2, kDown = 3, kLM = 4 };
constexpr int kPhasesPerLayer = 4;  // q/k/v, o, gate/up, down

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
// Weight bytes are read once per step, so their L2 lines are marked evict-first: the stream
// then does not push the KV cache, the activations and the exchange words out of L2.
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
DPUF_DEV void prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
DPUF_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// u8 (weight nibbles, 0..15 or 16 * 0..15) x s8 (activation codes) dot of four byte pairs
DPUF_DEV int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One phase as seen by this CTA: units u0 .. u0+n-1, in the stage order of Item.
struct Phase {
  int u0, n;       // the CTA's units
  int n_st, n_sub; // stages per group, groups per unit
  int spu;         // stages per unit
  int B;           // units per batch: kConsWarps (a warp per unit), or n (hand-over, n <= kHandMax)
  long long total; // ring positions of the phase in this CTA (batches of B units, padded)
};

// Shared state of a CTA outside the dynamic buffer.
struct DecShared {
  uint64_t full[kMaxSlots], empty[kMaxSlots];
  float red[kConsWarps];
  float lanes[8];
  float arg_v[kConsWarps];
  int arg_i[kConsWarps];
  int next_id;
  volatile int abort;
  const uint8_t* pg[kConsWarps];  // producer: the current round's group of each consumer warp
  Phase ph[5];                     // this CTA's share of each phase kind (fixed for the launch)
  // the layer table of the current and the next layer (by running layer index step * L + l, mod
  // 2): the next one is copied during the current one's norm2, so that no consumer step waits
  // on a global read of a pointer
  alignas(16) DecLayer lay[2];     // 16-byte aligned: filled by 16-byte cp.async / int4 stores
  float sv[kSvUnits][8];           // this CTA's SwiGLU outputs (gate/up unit - u0, row), for the down prep
  uint64_t mb_bar[kMailbox];       // accumulator hand-over between consumer warps (mb_put / mb_get)
  float mb_val[kMailbox][8];
};

// ------------------------------------------------------------------ exchange
DPUF_DEV uint64_t tagged(float v, unsigned gen) { return ((uint64_t)gen << 32) | __float_as_uint(v); }
DPUF_DEV unsigned tag_of(uint64_t w) { return (unsigned)(w >> 32); }
DPUF_DEV float value_of(uint64_t w) { return __uint_as_float((unsigned)w); }
DPUF_DEV void st_relaxed(uint64_t* p, uint64_t w, bool sys) {
  if (sys)
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
  else
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
DPUF_DEV uint64_t ld_relaxed(const uint64_t* p, bool sys) {
  uint64_t w;
  if (sys)
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
template <typename T>
DPUF_DEV T* peer_ptr(const DecodeArgs& A, T* p, int r) {
  return (T*)((char*)p + A.tp_delta[r]);
}
// A tagged word into this rank's buffer and every other rank's copy.
DPUF_DEV void put_tagged(const DecodeArgs& A, uint64_t* p, uint64_t w) {
  const bool sys = A.tp_world > 1;
  st_relaxed(p, w, sys);
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) st_relaxed(peer_ptr(A, p, r), w, true);
}
DPUF_DEV void put_float(const DecodeArgs& A, float* p, float v) {
  *p = v;
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) *peer_ptr(A, p, r) = v;
}
// Records a failure in this rank's error word and every other rank's, whose waits then stop.
DPUF_DEV void raise_err(const DecodeArgs& A, int code) {
  atomicCAS(A.err, 0, code);
  for (int r = 0; r < A.tp_world; r++)
    if (r != A.tp_rank) atomicCAS(peer_ptr(A, A.err, r), 0, code);
}
DPUF_DEV bool check_abort(const DecodeArgs& A, DecShared& S) {
  if (S.abort) return true;
  if (*(volatile int*)A.err) {
    S.abort = 1;
    return true;
  }
  return false;
}

// Waits (bounded) until every word j of wv whose bit is set in `stale` carries generation `gen`
// (wv[j] holds a first read of *addr(j)); on abort, wv holds whatever was read last.  Each round
// re-reads all the still-stale words at once, so a thread waiting for n words pays one memory
// round trip per round, not one per word.  Rounds back off from 32 to 256 ns: thousands of
// threads may poll at once, and every poll is an L2 request beside the weight stream.
template <int N, class Addr>
DPUF_DEV void wait_words(const DecodeArgs& A, uint64_t (&wv)[N], unsigned stale, Addr addr, unsigned gen,
                         DecShared& S) {
  if (!stale || S.abort) return;
  const bool sys = A.tp_world > 1;
  const unsigned long long t0 = globaltimer();
  unsigned ns = 32;
  for (int it = 1; stale; it++) {
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
#pragma unroll
    for (int j = 0; j < N; j++)
      if ((stale >> j) & 1u) wv[j] = ld_relaxed(addr(j), sys);
#pragma unroll
    for (int j = 0; j < N; j++)
      if (((stale >> j) & 1u) && tag_of(wv[j]) == gen) stale &= ~(1u << j);
    if (stale && (it & 7) == 0) {
      if (check_abort(A, S)) return;
      if (globaltimer() - t0 > A.wait_ns) {
        raise_err(A, 3);
        S.abort = 1;
        return;
      }
    }
  }
}
// The stale mask of N first reads.
template <int N>
DPUF_DEV unsigned stale_mask(const uint64_t (&wv)[N], unsigned valid, unsigned gen) {
  unsigned m = 0;
#pragma unroll
  for (int j = 0; j < N; j++)
    if (((valid >> j) & 1u) && tag_of(wv[j]) != gen) m |= 1u << j;
  return m;
}

// ------------------------------------------------------------------ work plan
// A projection phase is a list of units: 8-row groups (q/k/v, o, down, LM head) or gate/up pairs
// (the gate group and the up group of the same 8 rows).  The units are dealt in contiguous
// ranges to the CTAs of all ranks (virtual CTA v = blockIdx.x * tp_world + tp_rank, so every
// rank holds units of every phase), and a CTA's units to its consumer warps in turn.
DPUF_DEV int phase_units(const DecodeArgs& A, int kind) {
  switch (kind) {
    case kQKV: return (A.qd + 2 * A.kvd) / 8;
    case kO: return A.H / 8;
    case kGU: return A.I / 8;
    case kDown: return 2 * A.keep_down;
    default: return 2 * ((A.V + 15) / 16);
  }
}
DPUF_DEV int phase_cols(const DecodeArgs& A, int kind) {
  return kind == kO ? A.qd : (kind == kDown ? A.I : A.H);
}
DPUF_DEV int vcta(const DecodeArgs& A) { return blockIdx.x * A.tp_world + A.tp_rank; }

// (Computed once per launch into DecShared: the 64-bit divisions cost ~1 us of one thread.)
DPUF_DEV Phase compute_phase(const DecodeArgs& A, int kind) {
  Phase P;
  const int U = phase_units(A, kind), G = gridDim.x * A.tp_world, c = vcta(A);
  P.u0 = (int)((long long)U * c / G);
  P.n = (int)((long long)U * (c + 1) / G) - P.u0;
  P.n_st = ((phase_cols(A, kind) >> 5) + kKB - 1) / kKB;
  P.n_sub = kind == kGU ? 2 : 1;
  P.spu = P.n_st * P.n_sub;
  if (P.n <= kHandMax) {
    P.B = max(P.n, 1);
    P.total = (long long)P.n * P.spu;
  } else {
    P.B = kConsWarps;
    P.total = (long long)((P.n + kConsWarps - 1) / kConsWarps) * kConsWarps * P.spu;
  }
  return P;
}

// The stages of a phase in production (ring) order, position p going to consumer warp
// p % kConsWarps.  The CTA's units go in batches of B; a batch's stages are ordered (stage, group
// of the unit, unit).
//  - Many units (B = kConsWarps): warp w takes every stage of unit w of each batch, in order, its
//    running accumulators in registers.  The last batch is padded with empty units (no rows:
//    nothing copied, nothing computed), so that this holds for it too.
//  - Few units (n <= kHandMax, one batch of B = n): stage s+1 of a group is n_sub * B positions
//    after stage s, on another warp; the running accumulator is handed over through shared
//    memory (consume_phase).  Every warp then has stages to compute although only n units exist
//    (q/k/v, o and down have 3 to 6 units per CTA on the 8B shape).
struct Item {
  int b;       // batch
  int t;       // position within the batch
  int j;       // unit within the batch
  int sub, s;  // group of the unit (gate/up: 0, 1) and stage
};
DPUF_DEV void item_at(const Phase& ph, int p, Item& it) {
  const int per_batch = ph.spu * ph.B;
  it.b = p / per_batch;
  it.t = p - it.b * per_batch;
  const int r = it.t / ph.B;
  it.j = it.t - r * ph.B;
  it.s = r / ph.n_sub;
  it.sub = r - it.s * ph.n_sub;
}
// The item kConsWarps positions later (valid while that position is < ph.total).
DPUF_DEV void item_next(const Phase& ph, Item& it) {
  it.t += kConsWarps;
  it.j += kConsWarps;
  while (it.j >= ph.B) {
    it.j -= ph.B;
    if (++it.sub == ph.n_sub) {
      it.sub = 0;
      if (++it.s == ph.n_st) {  // (a warp per unit) the same unit of the next batch
        it.s = 0;
        it.b++;
        it.t -= ph.spu * ph.B;
      }
    }
  }
}
// The item's unit, or -1 for a padding unit.
DPUF_DEV int item_unit(const Phase& ph, const Item& it) {
  const int v = it.b * ph.B + it.j;
  return v < ph.n ? ph.u0 + v : -1;
}

// One 8-row group: where its scales start (the group's data: [n_blk][8] fp16 scales, then
// [n_blk][4][8][4] nibbles), its rows and its first output row.
struct Group {
  const uint8_t* base;
  int n_r;   // rows (0: an empty second group of a short last tile)
  int row;   // first output row
  int mat;   // q/k/v: 0, 1, 2; gate/up pair: 0 gate, 1 up
};
DPUF_DEV Group rows_of(int rows, int gi, int mat) {
  Group g;
  g.row = (gi >> 1) * kTileRows + (gi & 1) * 8;
  g.n_r = max(0, min(8, rows - g.row));
  g.base = nullptr;
  g.mat = mat;
  return g;
}
DPUF_DEV Group make_group(const uint8_t* tiles, long long stride, int rows, int n_blk, int gi, int mat) {
  Group g = rows_of(rows, gi, mat);
  g.base = tiles + (size_t)(gi >> 1) * stride + 16 + (size_t)(gi & 1) * n_blk * 144;
  return g;
}
DPUF_DEV const uint8_t* ldg_ptr(const uint8_t* const* p) { return (const uint8_t*)__ldg((const unsigned long long*)p); }
// Group `sub` (gate/up: 0 gate, 1 up; else 0) of unit u of phase `kind` in layer l.
DPUF_DEV Group group_of(const DecodeArgs& A, int l, int kind, int u, int sub) {
  const int n_blk = phase_cols(A, kind) >> 5;
  if (kind == kLM) return make_group(A.lm_tiles, A.lm_stride, A.V, n_blk, u, 0);
  const DecLayer* Ly = A.layers + l;
  switch (kind) {
    case kQKV: {
      const int gq = A.qd / 8, gk = A.kvd / 8;
      if (u < gq) return make_group(ldg_ptr(&Ly->tiles[0]), __ldg(&Ly->stride[0]), A.qd, n_blk, u, 0);
      if (u < gq + gk) return make_group(ldg_ptr(&Ly->tiles[1]), __ldg(&Ly->stride[1]), A.kvd, n_blk, u - gq, 1);
      return make_group(ldg_ptr(&Ly->tiles[2]), __ldg(&Ly->stride[2]), A.kvd, n_blk, u - gq - gk, 2);
    }
    case kO: return make_group(ldg_ptr(&Ly->tiles[3]), __ldg(&Ly->stride[3]), A.H, n_blk, u, 0);
    case kGU: return make_group(ldg_ptr(&Ly->tiles[4 + sub]), __ldg(&Ly->stride[4 + sub]), A.I, n_blk, u, sub);
    default: return make_group(ldg_ptr(&Ly->tiles[6]), __ldg(&Ly->stride[6]), A.H, n_blk, u, 0);
  }
}

// The rows of that group without its address (no memory access: the consumers' view).
DPUF_DEV Group group_rows(const DecodeArgs& A, int kind, int u, int sub) {
  switch (kind) {
    case kQKV: {
      const int gq = A.qd / 8, gk = A.kvd / 8;
      if (u < gq) return rows_of(A.qd, u, 0);
      if (u < gq + gk) return rows_of(A.kvd, u - gq, 1);
      return rows_of(A.kvd, u - gq - gk, 2);
    }
    case kO: return rows_of(A.H, u, 0);
    case kGU: return rows_of(A.I, u, sub);
    case kDown: return rows_of(A.H, u, 0);
    default: return rows_of(A.V, u, 0);
  }
}

// ------------------------------------------------------------------ producer
// The producer warp walks the CTA's stage sequence (every step, layer and phase) round by round:
// lane w moves consumer warp w's stage of the round into ring slot (cursor + w) once that slot's
// previous use is released.  One round (up to kConsWarps stages) then costs one pass of the
// warp, not kConsWarps passes of one thread: the issue rate keeps up with the stream (a 4.6 KB
// stage arrives every ~100 ns at the full rate, about one thread-iteration's worth of latency).
struct Producer {
  long long issued = 0;
  int slot = 0;      // ring slot of the round's first stage
  unsigned par = 0;  // parity of that slot's current use
  uint64_t pol = 0;
};

// A bounded wait for the completion of the phase of parity `par` of barrier `bar` (a slot's
// release, or a stage's arrival); polls the abort flag.
DPUF_DEV bool wait_bar(const DecodeArgs& A, uint64_t* bar, unsigned par, DecShared& S) {
  if (mbar_try(bar, par)) return true;
  const unsigned long long t0 = globaltimer();
  for (int it = 1; !mbar_try(bar, par); it++) {
    if ((it & 63) == 0) {
      if (check_abort(A, S)) return false;
      if (globaltimer() - t0 > A.wait_ns) {
        raise_err(A, 1);
        S.abort = 1;
        return false;
      }
    }
  }
  return true;
}

DPUF_DEV bool produce_phase(const DecodeArgs& A, int l, int kind, unsigned char* ring, Producer& P, DecShared& S) {
  const int lane = threadIdx.x & 31;
  const Phase ph = S.ph[kind];
  const int n_blk = phase_cols(A, kind) >> 5;
  const size_t nib0 = (size_t)n_blk * 16;
  const int total = (int)ph.total;
  for (int p0 = 0; p0 < total; p0 += kConsWarps) {
    const int W = min(kConsWarps, total - p0);
    const bool mine = lane < W;
    const uint8_t* gb = nullptr;  // the lane's group (null: padding or no rows, nothing to copy)
    int st = 0, kb = 0;           // its stage and that stage's blocks
    if (mine) {
      Item it;
      item_at(ph, p0 + lane, it);
      const int u = item_unit(ph, it);
      if (u >= 0) {
        const Group g = group_of(A, l, kind, u, it.sub);
        st = it.s;
        kb = min(kKB, n_blk - st * kKB);
        if (g.n_r > 0) gb = g.base;
      }
    }
    int slot = P.slot + lane;
    unsigned par = P.par;
    if (slot >= A.n_slots) {  // W <= n_slots: one wrap at most
      slot -= A.n_slots;
      par ^= 1u;
    }
    // at most max_inflight stages requested and not yet landed: the round's last stage waits
    // for the one max_inflight positions before it (copies land about in order).
    // max_inflight >= W puts that position before this round; n_slots > max_inflight + W keeps
    // its slot from being reissued before it.
    bool ok = true;
    const int back = W - 1 - A.max_inflight;
    if (lane == 0 && P.issued + back >= 0) {
      int qs = P.slot + back;
      unsigned qp = P.par;
      if (qs < 0) {
        qs += A.n_slots;
        qp ^= 1u;
      }
      ok = wait_bar(A, &S.full[qs], qp, S);
    }
    // the slot's previous use must be released (the first use passes at once)
    if (ok && mine) ok = wait_bar(A, &S.empty[slot], par ^ 1u, S);
    if (!__all_sync(kFull, ok)) return false;
    if (mine) {
      uint64_t* bar = &S.full[slot];
      if (gb == nullptr) {
        mbar_arrive(bar);  // empty group: nothing to copy, the consumer skips it
      } else {
        // the stage's scales (16 B per block) and nibbles (128 B per block, after the group's
        // n_blk scales)
        unsigned char* dst = ring + (size_t)slot * kSlotBytes;
        mbar_expect_tx(bar, (unsigned)kb * 144);
        bulk_g2s(dst, gb + (size_t)st * kScBytes, (unsigned)kb * 16, bar, P.pol);
        bulk_g2s(dst + kScBytes, gb + nib0 + (size_t)st * (kKB * 128), (unsigned)kb * 128, bar, P.pol);
      }
    }
    P.slot += W;
    if (P.slot >= A.n_slots) {
      P.slot -= A.n_slots;
      P.par ^= 1u;
    }
    P.issued += W;
    if (S.abort) return false;
  }
  return true;
}

// ------------------------------------------------------------------ one stage of one group
// Lane (ri, q): row ri's blocks 8q .. 8q+7 of the stage; then the in-order chain over the
// stage's blocks, octet by octet (octet q continues the accumulator of octet q-1).
template <bool kFull>
DPUF_DEV void stage_terms(const unsigned char* slot, const int8_t* xq, const float* xs, const int* xm, int b0, int kb,
                          int ri, int q, float (&pp)[8], float (&ss)[8]) {
  const unsigned char* nib = slot + kScBytes;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int bl = q * 8 + j;
    pp[j] = 0.0f;
    ss[j] = 0.0f;
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
      // a block with xs == 0 is skipped by the reference: (0, 0) leaves the chain unchanged
      ss[j] = bsc > 0.0f ? __fmul_rn(ws, bsc) : 0.0f;
      if (!(bsc > 0.0f)) pp[j] = 0.0f;
    }
  }
}
// The stage's chain: octet q continues the accumulator of octet q-1 (every lane ends with its
// row's running accumulator).
DPUF_DEV void octet_chain(const float (&pp)[8], const float (&ss)[8], int ri, int q, float& acc) {
#pragma unroll
  for (int qq = 0; qq < 4; qq++) {
    if (q == qq) {
#pragma unroll
      for (int j = 0; j < 8; j++) acc = __fmaf_rn(pp[j], ss[j], acc);
    }
    acc = __shfl_sync(kFull, acc, ri + 8 * qq);
  }
}

DPUF_DEV void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// Per-warp consuming state.
struct Consumer {
  int slot = 0;          // ring slot of the current phase's first stage
  unsigned par = 0;      // parity of that slot's use
  unsigned hpos = 0;     // positions of the hand-over phases so far (the hand-over tags)
  float bv = -INFINITY;  // running argmax of the LM head (lanes of octet 0)
  int bi = 0x7fffffff;
};

// Waits (bounded, every lane) for a stage to land; false once the CTA aborted.
DPUF_DEV bool ring_wait(const DecodeArgs& A, uint64_t* bar, unsigned ph, DecShared& S) {
  if (S.abort) return false;
  if (mbar_try(bar, ph)) return true;
  const unsigned long long t0 = globaltimer();
  for (int it = 1;; it++) {
    if (mbar_try(bar, ph)) return true;
    if ((it & 63) == 0) {
      if (check_abort(A, S)) return false;
      if (globaltimer() - t0 > A.wait_ns) {
        raise_err(A, 1);
        S.abort = 1;
        return false;
      }
    }
  }
}

// The prep of the down projection's input chunks this CTA owns - chunk ch belongs to the CTA
// holding gate/up unit 8ch + 7 - after the gate/up phase: lane group 8 lanes per chunk (lane qi:
// unit 8ch + qi, its eight SwiGLU outputs from shared memory if this CTA computed them, else the
// tagged words of the previous CTA (or rank)), then the reference's activation prep, stored as
// tagged words (generation gen) into every rank's dprep.  One warp per owned chunk.
DPUF_DEV void prep_down_owned(const DecodeArgs& A, const Phase& ph, unsigned gen, const uint8_t* dsg, DecShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qi = lane & 7;
  if (ph.n <= 0) return;
  const int u0 = ph.u0, u_end = ph.u0 + ph.n;
  const int ch_lo = u0 / 8, ch_hi = u_end >= 8 ? (u_end - 8) / 8 : -1;  // chunks with 8ch + 7 in [u0, u_end)
  for (int ch = ch_lo + warp; ch <= ch_hi; ch += kConsWarps) {
    const int u = ch * 8 + qi;
    float v[8];
    if (u >= u0) {
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = S.sv[u - u0][j];
    } else {
      const uint64_t* src = A.s_raw + (size_t)u * 8;
      uint64_t wv[8];
#pragma unroll
      for (int j = 0; j < 8; j++) wv[j] = ld_relaxed(src + j, A.tp_world > 1);
      wait_words(A, wv, stale_mask(wv, 0xFFu, gen), [&](int j) { return src + j; }, gen, S);
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = value_of(wv[j]);
    }
    const PrepOut o = prep_chunk_g8_core(v, dsg ? dsg[ch * 8 + qi] : (uint8_t)0, lane);
    if (lane < 8) {
      uint64_t* dst = A.dprep + (size_t)ch * kChunkWords;
      const uint64_t tg = (uint64_t)gen << 32;
      put_tagged(A, dst + 2 * qi, tg | o.lo);
      put_tagged(A, dst + 2 * qi + 1, tg | o.hi);
      if ((qi & 3) == 0) {
        put_tagged(A, dst + 16 + (qi >> 2), tagged(o.xs, gen));
        put_tagged(A, dst + 18 + (qi >> 2), tg | (unsigned)o.xm);
      }
    }
  }
}

// Optional trace of the last step: per CTA, the time (globaltimer, ns) at which each phase ended.
enum {
  kEvNorm1Res, kEvNorm1Chain, kEvNorm1, kEvQKV, kEvAttnIn, kEvAttnWait, kEvAttnRope, kEvAttnScores, kEvAttnSoftmax,
  kEvAttnPV, kEvAttn, kEvLoadO, kEvO, kEvNorm2Res, kEvNorm2Chain, kEvNorm2, kEvGUStages, kEvGU, kEvLoadD, kEvDown,
  kEvPerLayer
};
enum { kEvStart, kEvEmbed, kEvNormF, kEvLM, kEvArg, kEvPerStep };
DPUF_DEV void trace_at(const DecodeArgs& A, int step, int ev) {
  if (A.trace && step == A.n_steps - 1 && threadIdx.x == 0)
    A.trace[(size_t)blockIdx.x * A.trace_per_cta + ev] = globaltimer();
}

// Hand-over of running accumulators between consumer warps: entry (tag mod kMailbox) holds the
// eight rows' accumulators after the stage with tag `tag` - its position counted over the
// hand-over phases only, from 0 in each launch.  Its mbarrier completes one phase per tag: the
// warp of every position of a hand-over phase arrives once (mb_done, after writing the values if
// anyone reads them), so tag `tag` is phase tag / kMailbox of its entry (parity
// (tag / kMailbox) & 1).  Phases with a warp per unit do not use it.
// An entry is rewritten kMailbox positions later.  Its reader is at most 2 * kHandMax positions
// after the writer, and every position releases its ring stage only after its hand-over reads
// and its own arrival; a stage is only produced once every position n_slots or more before it
// has been released.  So with kMailbox >= 2 * kHandMax + kMaxSlots + 1, when a reader waits on
// an entry, the entry's previous use has completed its phase (the parity test cannot pass on a
// stale phase) and its next use has not been written.
DPUF_DEV void mb_put(DecShared& S, unsigned tag, int lane, float acc) {
  if (lane < 8) S.mb_val[tag & (kMailbox - 1)][lane] = acc;  // lane ri of octet 0: row ri
}
DPUF_DEV void mb_done(DecShared& S, unsigned tag, int lane) {
  __syncwarp();
  if (lane == 0) {
    __threadfence_block();
    mbar_arrive(&S.mb_bar[tag & (kMailbox - 1)]);  // release: the values before the phase completes
  }
}
DPUF_DEV float mb_get(const DecodeArgs& A, DecShared& S, unsigned tag, int ri) {
  const int e = (int)(tag & (kMailbox - 1));
  const unsigned par = (tag / kMailbox) & 1u;
  if (!mbar_try(&S.mb_bar[e], par)) {
    const unsigned long long t0 = globaltimer();
    for (int it = 1; !mbar_try(&S.mb_bar[e], par); it++) {
      if ((it & 63) == 0) {
        if (check_abort(A, S)) break;
        if (globaltimer() - t0 > A.wait_ns) {
          raise_err(A, 4);
          S.abort = 1;
          break;
        }
      }
    }
  }
  return S.mb_val[e][ri];
}

// The terms of one stage (in ring slot `slot`, stage s of a group with rows): false without rows
// or after an abort.
DPUF_DEV bool stage_at(const DecodeArgs& A, DecShared& S, const unsigned char* ring, int slot, unsigned par, int s,
                       int n_r, int n_blk, const int8_t* xq, const float* xs, const int* xm, int ri, int q,
                       float (&pp)[8], float (&ss)[8]) {
  const bool ok = __all_sync(kFull, ring_wait(A, &S.full[slot], par, S));
  if (!ok || n_r <= 0) return false;
  const int b0 = s * kKB, kb = min(kKB, n_blk - b0);
  const unsigned char* st = ring + (size_t)slot * kSlotBytes;
  if (kb == kKB)
    stage_terms<true>(st, xq, xs, xm, b0, kb, ri, q, pp, ss);
  else
    stage_terms<false>(st, xq, xs, xm, b0, kb, ri, q, pp, ss);
  return true;
}
// Releases a ring slot once every lane is done with it.
DPUF_DEV void release_slot(DecShared& S, int slot, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(&S.empty[slot]);
}

// The epilogue of unit u (final accumulators a0, and a1 for the up half of a gate/up pair;
// lanes of octet 0 hold rows g.row + ri): stores the rows, as the phase's consumers read them.
DPUF_DEV void unit_epilogue(const DecodeArgs& A, DecShared& S, int kind, int u, const Group& g, float a0, float a1,
                            unsigned gen, bool stall, const uint8_t* dsg, Consumer& C, int lane) {
  const int ri = lane & 7, q = lane >> 3;
  const bool mine = q == 0 && ri < g.n_r;
  const int row = g.row + ri;
  if (kind == kQKV) {
    uint64_t* dst = g.mat == 0 ? A.q : (g.mat == 1 ? A.k : A.v);
    if (mine && !stall) put_tagged(A, dst + row, tagged(a0, gen));
  } else if (kind == kO) {
    if (mine) put_tagged(A, A.o_out + row, tagged(a0, gen));
  } else if (kind == kDown) {
    if (mine) put_tagged(A, A.d_out + row, tagged(a0, gen));
  } else if (kind == kLM) {
    if (mine) {
      if (A.write_logits) put_float(A, A.logits + row, a0);
      better(C.bv, C.bi, a0, row);
    }
  } else {
    // gate/up: SwiGLU with the reference's vector/scalar split: kept in shared memory for this
    // CTA's down-input preps (prep_down_owned) and stored as tagged words to every rank for
    // the next CTA's
    (void)dsg;
    if (mine) {
      const float sw = swiglu_one(a0, a1, A.deadzone, swiglu_vector_elem(row, A.I, A.nt_ref, false), A.et);
      S.sv[u - S.ph[kGU].u0][ri] = sw;
      put_tagged(A, A.s_raw + row, tagged(sw, gen));
    }
  }
}

// One projection phase on the consumer side of warp `warp`: its positions warp, warp +
// kConsWarps, ... of the phase (Item).  A warp per unit: for each batch, the stages of the
// warp's unit in a tight loop (accumulators in registers), then its epilogue, so that the loop
// body stays small.  Hand-over: each position's stage terms, the accumulator chain continued from
// the hand-over, and at a unit's last stage the epilogue.  dsg: the down projection's
// column-sign bytes in shared memory (gate/up only).
DPUF_DEV void consume_phase(const DecodeArgs& A, int step, int l, int kind, unsigned gen, unsigned char* ring,
                            Consumer& C, const int8_t* xq, const float* xs, const int* xm, const uint8_t* dsg,
                            DecShared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ri = lane & 7, q = lane >> 3;
  const Phase ph = S.ph[kind];
  const int total = (int)ph.total;
  const int n_blk = phase_cols(A, kind) >> 5;
  const bool stall = step == 0 && l == 0 && kind == kQKV && A.stall_unit >= ph.u0 && A.stall_unit < ph.u0 + ph.n;
  int slot = C.slot + warp;
  unsigned par = C.par;
  while (slot >= A.n_slots) {
    slot -= A.n_slots;
    par ^= 1u;
  }
  auto advance = [&]() {
    slot += kConsWarps;
    while (slot >= A.n_slots) {
      slot -= A.n_slots;
      par ^= 1u;
    }
  };
  const bool own = ph.B == kConsWarps;
  if (own) {
    // unit b * kConsWarps + warp of batch b: its stage r (r = s * n_sub + sub) is at position
    // b * kConsWarps * spu + r * kConsWarps + warp
    const int nb = total / (kConsWarps * ph.spu);
    for (int b = 0; b < nb; b++) {
      const int v = b * kConsWarps + warp;
      const int u = v < ph.n ? ph.u0 + v : -1;  // -1: padding (nothing copied, nothing computed)
      const Group g0 = u >= 0 ? group_rows(A, kind, u, 0) : rows_of(0, 0, 0);
      const Group g1 = u >= 0 && ph.n_sub == 2 ? group_rows(A, kind, u, 1) : g0;
      float acc0 = 0.0f, acc1 = 0.0f;
      for (int r = 0; r < ph.spu; r++) {
        const int sub = ph.n_sub == 2 ? (r & 1) : 0, s = ph.n_sub == 2 ? (r >> 1) : r;
        float pp[8], ss[8];
        const bool live = stage_at(A, S, ring, slot, par, s, sub ? g1.n_r : g0.n_r, n_blk, xq, xs, xm, ri, q, pp, ss);
        if (live) {
          if (sub) octet_chain(pp, ss, ri, q, acc1);
          else octet_chain(pp, ss, ri, q, acc0);
        }
        release_slot(S, slot, lane);
        advance();
      }
      if (kind == kGU && b == nb - 1) trace_at(A, step, kEvPerLayer * l + kEvGUStages);
      if (u >= 0) unit_epilogue(A, S, kind, u, ph.n_sub == 2 ? g1 : g0, acc0, acc1, gen, stall, dsg, C, lane);
    }
    if (kind == kGU && nb == 0) trace_at(A, step, kEvPerLayer * l + kEvGUStages);
  } else {
    Item it;
    if (warp < total) item_at(ph, warp, it);
    if (kind == kGU && warp >= total) trace_at(A, step, kEvPerLayer * l + kEvGUStages);
    for (int p = warp; p < total; p += kConsWarps) {
      const int u = item_unit(ph, it);  // (no padding in this mode)
      const Group g = group_rows(A, kind, u, it.sub);
      float pp[8], ss[8];
      const bool live = stage_at(A, S, ring, slot, par, it.s, g.n_r, n_blk, xq, xs, xm, ri, q, pp, ss);
      float acc = 0.0f;
      if (it.s > 0) acc = mb_get(A, S, C.hpos + (unsigned)(p - ph.n_sub * ph.B), ri);
      if (live) octet_chain(pp, ss, ri, q, acc);
      const bool last = it.s == ph.n_st - 1 && it.sub == ph.n_sub - 1;  // the unit's last stage
      const float a0 = last && ph.n_sub == 2 ? mb_get(A, S, C.hpos + (unsigned)(p - ph.B), ri) : acc;
      if (!last) mb_put(S, C.hpos + (unsigned)p, lane, acc);
      mb_done(S, C.hpos + (unsigned)p, lane);
      // the slot goes back only now: after this position's hand-over reads and its own arrival
      release_slot(S, slot, lane);
      if (kind == kGU && p + kConsWarps >= total) trace_at(A, step, kEvPerLayer * l + kEvGUStages);
      if (last) unit_epilogue(A, S, kind, u, g, a0, acc, gen, stall, dsg, C, lane);
      advance();
      if (p + kConsWarps < total) item_next(ph, it);
    }
  }
  {  // the next phase starts ph.total positions later
    const int q2 = total / A.n_slots;
    C.slot += total - q2 * A.n_slots;
    C.par ^= (unsigned)q2 & 1u;
    if (C.slot >= A.n_slots) {
      C.slot -= A.n_slots;
      C.par ^= 1u;
    }
    if (!own) C.hpos += (unsigned)total;
  }
}

// ------------------------------------------------------------------ row-wide steps
DPUF_DEV void cta_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kConsThreads) : "memory"); }


// Residual add (tagged words of generation `gen`; rows >= n_valid add 0, as the pruned down
// projection's zero rows do), RMSNorm (add_and_rms_norm_f32 / rms_norm_f32,
// dpuf_engine.c:225-272) and the activation prep of the result into x.  The gains and the sign
// bytes go to shared memory (stage) asynchronously before the residual is waited for.
DPUF_DEV void norm_prep(const DecodeArgs& A, float* h, const uint64_t* res, unsigned gen, int n_valid, const float* w,
                        const uint8_t* signs, int8_t* xq, float* xs, int* xm, float* stage, DecShared& S, int step,
                        int ev, const DecLayer* next_src = nullptr, DecLayer* next_dst = nullptr,
                        const uint8_t* xsrc = nullptr, uint8_t* xdst = nullptr, int xbytes = 0) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, H = A.H;
  float* sw = stage;
  uint8_t* sg = (uint8_t*)(stage + H);
  for (int i = tid * 4; i < H; i += kConsThreads * 4) cp_async16_cg(sw + i, w + i);
  if (signs)
    for (int i = tid * 8; i < H / 8; i += kConsThreads * 8) cp_async8_ca(sg + i, signs + i);
  // the next layer's table and extra bytes (the down projection's sign bytes) ride along, waited
  // for with the gains
  if (next_src && tid < (int)(sizeof(DecLayer) / 16))
    cp_async16_cg((unsigned char*)next_dst + tid * 16, (const unsigned char*)next_src + tid * 16);
  if (xsrc)
    for (int i = tid * 8; i < xbytes; i += kConsThreads * 8) cp_async8_ca(xdst + i, xsrc + i);
  cp_async_commit();
  if (res) {
    // every word is loaded first (all in flight), then the stale ones are waited for
    constexpr int kPer = 12;
    const bool sys = A.tp_world > 1;
    for (int i0 = tid; i0 < H; i0 += kConsThreads * kPer) {
      uint64_t wv[kPer];
      unsigned valid = 0;
#pragma unroll
      for (int j = 0; j < kPer; j++) {
        const int i = i0 + j * kConsThreads;
        const bool ok = i < H && i < n_valid;
        wv[j] = ok ? ld_relaxed(res + i, sys) : 0;
        if (ok) valid |= 1u << j;
      }
      wait_words(A, wv, stale_mask(wv, valid, gen), [&](int j) { return res + i0 + j * kConsThreads; }, gen, S);
#pragma unroll
      for (int j = 0; j < kPer; j++) {
        const int i = i0 + j * kConsThreads;
        if (i < H) h[i] = __fadd_rn(h[i], ((valid >> j) & 1u) ? value_of(wv[j]) : 0.0f);
      }
    }
    cta_sync();
  }
  if (ev >= 0) trace_at(A, step, ev);
  if (tid < 8) S.lanes[tid] = sumsq_lane32(h, H & ~7, tid);
  cp_async_wait_pending(0);
  cta_sync();
  if (ev >= 0) trace_at(A, step, ev + 1);
  const float inv = rms_inv(S.lanes, h, H, A.eps);  // every thread, same bits
  const int nch = H / 64;
  for (int cb = warp * 4; cb < nch; cb += kConsThreads / 8) {
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
  cta_sync();
}

// A prepped projection input (n_ch chunks of kChunkWords tagged words, generation `gen`) into x:
// codes, block scales, block sums.
DPUF_DEV void load_prepped(const DecodeArgs& A, const uint64_t* src, int n_ch, unsigned gen, int8_t* xq, float* xs,
                           int* xm, DecShared& S) {
  const int n = n_ch * kChunkWords;
  const bool sys = A.tp_world > 1;
  constexpr int kPer = 12;
  for (int i0 = threadIdx.x; i0 < n; i0 += kConsThreads * kPer) {
    uint64_t wv[kPer];
    unsigned valid = 0;
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      const int i = i0 + j * kConsThreads;
      wv[j] = i < n ? ld_relaxed(src + i, sys) : 0;
      if (i < n) valid |= 1u << j;
    }
    wait_words(A, wv, stale_mask(wv, valid, gen), [&](int j) { return src + i0 + j * kConsThreads; }, gen, S);
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      const int i = i0 + j * kConsThreads;
      if (i >= n) continue;
      const uint64_t x = wv[j];
      const int ch = i / kChunkWords, o = i - ch * kChunkWords;
      if (o < 16) *(uint32_t*)(xq + ch * 64 + o * 4) = (uint32_t)x;
      else if (o < 18) xs[ch * 2 + (o - 16)] = value_of(x);
      else xm[ch * 2 + (o - 18)] = (int)(unsigned)x;
    }
  }
  cta_sync();
}

// ------------------------------------------------------------------ attention of one head
// gqa_attn_head_pair_f32 (dpuf_engine.c:341-577) for query head h at position pos by the CTA's
// consumer threads, with the pair path's arithmetic (the lone path's for the last head of an odd
// group): QK-norm and RoPE of the query and the key, the K/V store (by the group's first head),
// scores (eight threads per key, the reference's 8-lane accumulation and trees), softmax, PV (one
// thread per output dimension, keys in order), then the prep of the head's output columns for
// the o projection, stored as tagged words of this GPU.  Everything that does not depend on this
// step - the QK-norm gains, the RoPE row, the o projection's sign bytes, the first value tiles
// and each thread's first history key - is requested before the query, key and value are
// waited for.
// The attention scratch of one head in the union (all float offsets from U).
struct AttnScratch {
  float *qs, *kin, *vin, *outv, *qn, *kn, *cs, *sn, *sc, *vt;
  uint8_t* osg;
};
DPUF_DEV AttnScratch attn_scratch(const DecodeArgs& A, float* U) {
  const int hd = A.hd;
  AttnScratch X;
  X.qs = U;
  X.kin = X.qs + hd;
  X.vin = X.kin + hd;
  X.outv = X.vin + hd;
  X.qn = X.outv + hd;
  X.kn = X.qn + hd;
  X.cs = X.kn + hd;
  X.sn = X.cs + hd / 2;
  X.osg = (uint8_t*)(X.sn + hd / 2);  // hd / 8 sign bytes (16-byte padded)
  X.sc = (float*)(X.osg + 16 * ((hd / 8 + 15) / 16));
  X.vt = X.sc + ((A.S + 3) & ~3);  // two value tiles [kVTile][hd]
  return X;
}
DPUF_DEV float* kv_rows(const DecodeArgs& A, float* base, int l, int kvh) {
  return base + ((size_t)l * A.nkv + kvh) * A.S * A.hd;
}
// Value tile t (keys t*kVTile .., history rows only) into buffer t & 1, one commit group.
DPUF_DEV void issue_vtile(const DecodeArgs& A, const AttnScratch& X, const float* vc, int n_rows, int t) {
  const int hd = A.hd, t0 = t * kVTile, nk = max(0, min(kVTile, n_rows - t0)), per_row = hd / 4;
  float* buf = X.vt + (size_t)(t & 1) * kVTile * hd;
  for (int i = threadIdx.x; i < nk * per_row; i += kConsThreads) {
    const int r = i / per_row, c = (i - r * per_row) * 4;
    cp_async16_cg(buf + r * hd + c, vc + (size_t)(t0 + r) * hd + c);
  }
  cp_async_commit();
}

// Everything the attention of head h at position pos needs that does not depend on this step's
// q/k/v: the QK-norm gains, the RoPE row and the o projection's sign bytes (one commit group),
// the first two value tiles (a group each), and the key and value history rows into L2.  Issued
// by the hosting CTA before its q/k/v stages, so that it lands while they run.
DPUF_DEV void attention_prefetch(const DecodeArgs& A, const DecLayer* Ly, int l, int pos, int h, float* U) {
  const int tid = threadIdx.x, hd = A.hd, kvh = h / (A.nq / A.nkv), n_rows = pos;
  const AttnScratch X = attn_scratch(A, U);
  // the history rows were stored by other CTAs in earlier steps, before tagged outputs this CTA
  // has since read: order this CTA's reads of the cache after them
  __threadfence();
  for (int i = tid * 4; i < hd; i += kConsThreads * 4) {
    if (Ly->q_norm) cp_async16_cg(X.qn + i, Ly->q_norm + i);
    if (Ly->k_norm) cp_async16_cg(X.kn + i, Ly->k_norm + i);
    if (i < hd / 2) {
      cp_async16_cg(X.cs + i, A.cos_tab + (size_t)pos * (hd >> 1) + i);
      cp_async16_cg(X.sn + i, A.sin_tab + (size_t)pos * (hd >> 1) + i);
    }
  }
  const uint8_t* so = Ly->signs[1];
  if (so && tid == 0)
    for (int i = 0; i < hd / 8; i += 8) cp_async8_ca(X.osg + i, so + (size_t)h * hd / 8 + i);
  cp_async_commit();
  const float* kc = kv_rows(A, A.kv_k, l, kvh);
  const float* vc = kv_rows(A, A.kv_v, l, kvh);
  const int n_vt = (n_rows + 1 + kVTile - 1) / kVTile;
  issue_vtile(A, X, vc, n_rows, 0);
  if (n_vt > 1) issue_vtile(A, X, vc, n_rows, 1);
  else cp_async_commit();
  // the key rows, and the value rows past the first two tiles, into L2 (32 KB pieces)
  const size_t row_b = (size_t)hd * 4, kb = (size_t)n_rows * row_b;
  const size_t v0 = min(kb, (size_t)2 * kVTile * row_b);
  constexpr size_t kPiece = 32768;
  const size_t nk = (kb + kPiece - 1) / kPiece, nv = (kb - v0 + kPiece - 1) / kPiece;
  for (size_t i = tid; i < nk + nv; i += kConsThreads) {
    const char* src = i < nk ? (const char*)kc + i * kPiece : (const char*)vc + v0 + (i - nk) * kPiece;
    const size_t end = i < nk ? kb : kb - v0;
    const size_t off = i < nk ? i * kPiece : (i - nk) * kPiece;
    prefetch_l2(src, (unsigned)min(kPiece, end - off));
  }
}

// gqa_attn_head_pair_f32 (dpuf_engine.c:341-577) for query head h at position pos by the CTA's
// consumer threads, with the pair path's arithmetic (the lone path's for the last head of an odd
// group): QK-norm and RoPE of the query and the key, the K/V store (by the group's first head),
// scores (eight threads per key, the reference's 8-lane accumulation and trees), softmax, PV (one
// thread per output dimension, keys in order), then the prep of the head's output columns for
// the o projection, stored as tagged words of this GPU.  attention_prefetch (by this call when
// `prefetched` is false) has requested the step-independent inputs.
DPUF_DEV void attention_head(const DecodeArgs& A, const DecLayer* Ly, int l, int pos, int h, unsigned gen, float* U,
                             bool prefetched, DecShared& S, int step, int ev) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = A.hd, groups = A.nq / A.nkv, kvh = h / groups, kv_len = pos + 1;
  const bool lone = (groups & 1) && (h % groups == groups - 1);
  const int kv4 = kv_len & ~3, kv8 = kv_len & ~7;
  if (!prefetched) attention_prefetch(A, Ly, l, pos, h, U);
  const AttnScratch X = attn_scratch(A, U);
  float* qs = X.qs;
  float* kin = X.kin;
  float* vin = X.vin;
  float* outv = X.outv;
  float* qn = X.qn;
  float* kn = X.kn;
  float* cs = X.cs;
  float* sn = X.sn;
  uint8_t* osg = X.osg;
  float* sc = X.sc;
  float* vt = X.vt;
  float* kc = kv_rows(A, A.kv_k, l, kvh);
  float* vc = kv_rows(A, A.kv_v, l, kvh);
  const int n_rows = kv_len - 1;  // history rows read from the cache (the current one comes from vin)
  const int n_vt = (kv_len + kVTile - 1) / kVTile;
  const uint8_t* so = Ly->signs[1];
  // each key group's first key (history rows only) into registers
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int j = tid & 7, kg = tid >> 3;
  const int warp_kg0 = warp * 4;  // key groups of this warp: warp_kg0 .. +3
  float kv[16];
  {
    const int t = kg;
    const bool pre = t < n_rows;
#pragma unroll
    for (int m = 0; m < 16; m++) kv[m] = (pre && j + 8 * m < hd) ? __ldcg(kc + (size_t)t * hd + j + 8 * m) : 0.0f;
  }
  // this step's query head, key and value (tagged words of the q/k/v phase; 3 * hd <= 2 threads'
  // worth, hd <= 128)
  {
    auto src = [&](int j) {
      const int i = tid + j * kConsThreads;
      return i < hd ? A.q + (size_t)h * hd + i
                    : (i < 2 * hd ? A.k + (size_t)kvh * hd + (i - hd) : A.v + (size_t)kvh * hd + (i - 2 * hd));
    };
    uint64_t wv[2];
    unsigned valid = 0;
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const bool ok = tid + j * kConsThreads < 3 * hd;
      wv[j] = ok ? ld_relaxed(src(j), A.tp_world > 1) : 0;
      if (ok) valid |= 1u << j;
    }
    wait_words(A, wv, stale_mask(wv, valid, gen), src, gen, S);
#pragma unroll
    for (int j = 0; j < 2; j++)
      if ((valid >> j) & 1u) qs[tid + j * kConsThreads] = value_of(wv[j]);  // qs, kin, vin are contiguous
  }
  trace_at(A, step, ev);  // thread 0's q/k/v words are in
  cp_async_wait_pending(n_vt > 1 ? 2 : 1);  // the constants (the value tiles may stay in flight)
  cta_sync();
  trace_at(A, step, ev + 1);
  if (warp == 0) qk_norm_rope_warp(qs, Ly->q_norm ? qn : nullptr, A.eps, hd, cs, sn, lane);
  if (warp == 1) qk_norm_rope_warp(kin, Ly->k_norm ? kn : nullptr, A.eps, hd, cs, sn, lane);
  cta_sync();
  trace_at(A, step, ev + 2);
  if (h % groups == 0) {  // the group's first head stores the key and value at pos
    if (warp == 2)
      for (int i = lane; i < hd; i += 32) kc[(size_t)pos * hd + i] = kin[i];
    if (warp == 3)
      for (int i = lane; i < hd; i += 32) vc[(size_t)pos * hd + i] = vin[i];
  }
  // ---- scores: key group kg takes keys kg, kg + kKeyGroups, ...; lane j of the group
  // accumulates elements j, j+8, ... of the dot
  float qv[16];
#pragma unroll
  for (int m = 0; m < 16; m++) qv[m] = (j + 8 * m < hd) ? qs[j + 8 * m] : 0.0f;
  float lmax = -1e30f;
  for (int t0 = warp_kg0; t0 < kv_len; t0 += kKeyGroups) {
    const int t = t0 + (kg - warp_kg0);
    const bool valid = t < kv_len;
    if (t0 != warp_kg0) {  // keys past the first round come from the cache now
#pragma unroll
      for (int m = 0; m < 16; m++)
        kv[m] = (t < n_rows && j + 8 * m < hd) ? __ldcg(kc + (size_t)t * hd + j + 8 * m) : 0.0f;
    }
    if (t == pos) {
#pragma unroll
      for (int m = 0; m < 16; m++) kv[m] = (j + 8 * m < hd) ? kin[j + 8 * m] : 0.0f;
    }
    float acc = 0.0f, a0 = 0.0f, a1 = 0.0f;
    if (valid) {
#pragma unroll
      for (int m = 0; m < 16; m++)
        if (j + 8 * m < hd) acc = __fmaf_rn(qv[m], kv[m], acc);
      if (lone && t >= kv4) {
        // lone head, tail key: dot_f32_avx2 (dpuf_engine.c:325-339), two accumulators over
        // 16-wide steps (hd % 64 == 0: no 8-wide remainder), summed lane-wise before the split tree
#pragma unroll
        for (int p2 = 0; p2 < 8; p2++)
          if (16 * p2 < hd) {
            a0 = __fmaf_rn(qv[2 * p2], kv[2 * p2], a0);
            a1 = __fmaf_rn(qv[2 * p2 + 1], kv[2 * p2 + 1], a1);
          }
      }
    }
    const float t_pairs = tree8_pairs(acc);
    const float t_split = tree8_split(acc);
    const float t_lone = tree8_split(__fadd_rn(a0, a1));
    const float sv = __fmul_rn(t < kv4 ? t_pairs : (lone ? t_lone : t_split), scale);
    if (valid && j == 0) {
      sc[t] = sv;
      lmax = max_ps(lmax, sv);
    }
  }
  {
    const float v = warp_max(lmax);
    if (lane == 0) S.red[warp] = v;
  }
  cta_sync();
  trace_at(A, step, ev + 3);
  float mx = -1e30f;
  for (int w = 0; w < kConsWarps; w++) mx = max_ps(mx, S.red[w]);
  // ---- softmax (vec_softmax_avx2, dpuf_engine.c:579-601)
  for (int t = tid; t < kv8; t += kConsThreads) sc[t] = exp_poly(__fsub_rn(sc[t], mx));
  if (tid >= kConsThreads - 8) {
    const int t = kv8 + (tid - (kConsThreads - 8));
    if (t < kv_len) sc[t] = glibc_expf(__fsub_rn(sc[t], mx), A.et);
  }
  cta_sync();
  if (tid < 8) {
    float acc = 0.0f;
    for (int t = tid; t < kv8; t += 8) acc = __fadd_rn(acc, sc[t]);
    S.lanes[tid] = acc;
  }
  cta_sync();
  float su = tree8_split_arr(S.lanes);
  for (int t = kv8; t < kv_len; t++) su = __fadd_rn(su, sc[t]);
  const float inv = __fdiv_rn(1.0f, __fadd_rn(su, 1e-12f));
  cta_sync();  // every thread has read the lane sums and the tail
  for (int t = tid; t < kv_len; t += kConsThreads) sc[t] = __fmul_rn(sc[t], inv);
  trace_at(A, step, ev + 4);
  // ---- PV: thread d < hd, keys in order (pair path: fma(p_k, v_kd, acc); lone path: keys two at
  // a time, k+1 first, dpuf_engine.c:541-548)
  float acc = 0.0f;
  const int hd8 = hd & ~7;
  for (int t = 0; t < n_vt; t++) {
    cp_async_wait_pending(t + 1 < n_vt ? 1 : 0);
    cta_sync();
    const float* buf = vt + (size_t)(t & 1) * kVTile * hd;
    const int t0 = t * kVTile, nk = min(kVTile, kv_len - t0);
    if (tid < hd) {
      const int d = tid;
      auto vat = [&](int k) { return (t0 + k == pos) ? vin[d] : buf[k * hd + d]; };
      if (!lone) {
        for (int k = 0; k < nk; k++) acc = __fmaf_rn(sc[t0 + k], vat(k), acc);
      } else if ((hd & 63) == 0) {
        int k = 0;
        for (; k + 1 < nk; k += 2) {
          const float t1 = __fmaf_rn(sc[t0 + k + 1], vat(k + 1), acc);
          acc = __fmaf_rn(sc[t0 + k], vat(k), t1);
        }
        if (k < nk) acc = __fmaf_rn(sc[t0 + k], vat(k), acc);
      } else {
        for (int k = 0; k < nk; k++) {
          const float pv = sc[t0 + k], vv = vat(k);
          acc = (d < hd8) ? __fmaf_rn(pv, vv, acc) : __fadd_rn(acc, __fmul_rn(pv, vv));
        }
      }
    }
    cta_sync();  // the tile buffer is free again
    if (t + 2 < n_vt) issue_vtile(A, X, vc, n_rows, t + 2);
    else cp_async_commit();
  }
  trace_at(A, step, ev + 5);
  if (tid < hd) outv[tid] = acc;
  if (h % groups == 0) __threadfence();  // the K/V rows stored above, before the tagged outputs
  cta_sync();
  // ---- prep of the head's output columns (hd / 64 chunks) for the o projection
  const int n_ch = hd / 64;
  if (warp * 4 < n_ch) {
    const int c = warp * 4 + (lane >> 3), qi = lane & 7;
    const bool active = c < n_ch;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = outv[(active ? c * 64 : 0) + qi * 8 + k];
    const int gch = (h * hd) / 64 + (active ? c : 0);  // chunk of the o-projection input
    const PrepOut o = prep_chunk_g8_core(v, so ? osg[(active ? c : 0) * 8 + qi] : 0, lane);
    if (active) {
      uint64_t* dst = A.oprep + (size_t)gch * kChunkWords;
      const uint64_t tg = (uint64_t)gen << 32;
      st_relaxed(dst + 2 * qi, tg | o.lo, false);
      st_relaxed(dst + 2 * qi + 1, tg | o.hi, false);
      if ((qi & 3) == 0) {
        st_relaxed(dst + 16 + (qi >> 2), tagged(o.xs, gen), false);
        st_relaxed(dst + 18 + (qi >> 2), tg | (unsigned)o.xm, false);
      }
    }
  }
  cta_sync();
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(DecodeArgs A) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ DecShared S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = A.H;
  unsigned char* ring = smem;
  float* h = (float*)(smem + (size_t)A.n_slots * kSlotBytes);
  int8_t* xq = (int8_t*)(h + H);
  float* xs = (float*)(xq + A.kmax);
  int* xm = (int*)(xs + A.kmax / 32);
  float* U = (float*)(((uintptr_t)(xm + A.kmax / 32) + 15) & ~(uintptr_t)15);  // union (16-byte aligned)
  // the down projection's sign bytes (staged by norm2, read by the gate/up epilogues), after the
  // norm staging in the union
  uint8_t* dsg = (uint8_t*)U + decode_norm_stage_bytes(A);

  if (tid == 0) {
    for (int i = 0; i < A.n_slots; i++) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1);
    }
    for (int i = 0; i < kMailbox; i++) mbar_init(&S.mb_bar[i], 1);
    S.abort = 0;
    for (int k = kQKV; k <= kLM; k++) S.ph[k] = compute_phase(A, k);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // ---------------------------------------------------------------- producer warp
  if (warp == kProdWarp) {
    Producer P;
    P.pol = l2_evict_first_policy();
    bool ok = true;
    // one call site for every phase (the body is inlined once: see the consumer loop)
    const int n_ph = kPhasesPerLayer * A.L + 1;
    for (int i = 0; ok && i < A.n_steps * n_ph; i++) {
      const int k = i % n_ph, l = k / kPhasesPerLayer;
      ok = produce_phase(A, l, l < A.L ? k % kPhasesPerLayer : kLM, ring, P, S);
    }
    // copies still in flight must land before the CTA exits: every slot's last fill
    if (lane == 0) {
      const unsigned long long t0 = globaltimer();
      for (long long p = max(0LL, P.issued - A.n_slots); p < P.issued; p++)
        while (!mbar_try(&S.full[p % A.n_slots], (unsigned)((p / A.n_slots) & 1)) && globaltimer() - t0 < A.wait_ns) {
        }
    }
    return;
  }

  // ---------------------------------------------------------------- consumer warps
  Consumer C;
  // query heads of this CTA: hh with floor(hh * grid / nq) == blockIdx.x, i.e. [head_lo, head_hi)
  const int head_lo = (int)((blockIdx.x * A.nq + gridDim.x - 1) / gridDim.x);
  const int head_hi = (int)(((blockIdx.x + 1) * A.nq + gridDim.x - 1) / gridDim.x);
  // the first layer's table (later ones are staged one layer ahead)
  if (A.L > 0 && tid < (int)(sizeof(DecLayer) / 16))
    ((int4*)&S.lay[0])[tid] = __ldg((const int4*)A.layers + tid);
  cta_sync();
  const int n_chunks = H / 64;
  for (int step = 0; step < A.n_steps; step++) {
    const int pos = A.pos0 + step;
    const int id = step == 0 ? A.first_id : S.next_id;
    const unsigned g_step = A.gen0 + (unsigned)step * (unsigned)decode_phases(A.L);
    trace_at(A, step, kEvPerLayer * A.L + kEvStart);
    // ---- embedding row -> h: the row's 8-row group of its tile and the sign bytes are staged,
    // then every warp expands its chunks from there
    {
      const int n_blk = H >> 5, lr = id % kTileRows;
      const uint8_t* grp = A.tok_tiles + (size_t)(id / kTileRows) * A.tok_stride + 16 + (size_t)(lr >> 3) * n_blk * 144;
      uint8_t* sgrp = (uint8_t*)U;
      uint8_t* sg = sgrp + n_blk * 144;
      for (int i = tid * 16; i < n_blk * 144; i += kConsThreads * 16) cp_async16_cg(sgrp + i, grp + i);
      if (A.tok_signs)
        for (int i = tid * 8; i < H / 8; i += kConsThreads * 8) cp_async8_ca(sg + i, A.tok_signs + i);
      cp_async_commit_wait_all();
      cta_sync();
      for (int c = warp; c < n_chunks; c += kConsWarps) {
        float a, b;
        embed_chunk_warp(sgrp - 16, n_blk, lr & 7, A.tok_signs ? sg : nullptr, c * 64, lane, a, b);
        h[c * 64 + lane] = a;
        h[c * 64 + 32 + lane] = b;
      }
      cta_sync();
    }
    trace_at(A, step, kEvPerLayer * A.L + kEvEmbed);
    // The layers' phases and the LM head as one sequence, so that every phase body (norm, prep
    // loads, attention, the projection) is inlined once: the kernel re-executes all of it every
    // layer, and a footprint that the instruction cache holds keeps instruction fetches off L2,
    // which is busy with the weight stream.
    const int n_ph = kPhasesPerLayer * A.L + 1;
    const unsigned g_lm = g_step + (unsigned)A.L;
    const int sb = kEvPerLayer * A.L;
    C.bv = -INFINITY;
    C.bi = 0x7fffffff;
    for (int k = 0; k < n_ph; k++) {
      const int l = k / kPhasesPerLayer, kind = l < A.L ? k % kPhasesPerLayer : kLM;
      const int gl = step * A.L + l;  // running layer index: table buffer gl & 1
      const DecLayer* Ly = &S.lay[gl & 1];
      const int lb = kEvPerLayer * l;
      const unsigned g = g_step + (unsigned)l;
      // ---- before the projection: its input
      if (kind == kQKV || kind == kGU || kind == kLM) {
        // residual add + RMSNorm + prep: attention norm (the previous layer's down output, none
        // before layer 0), FFN norm (the o output; the next layer's table and the down
        // projection's sign bytes ride along), final norm
        const bool ffn = kind == kGU, more = l + 1 < A.L || step + 1 < A.n_steps;
        const uint64_t* res = ffn ? A.o_out : (l > 0 ? A.d_out : nullptr);
        norm_prep(A, h, res, ffn ? g : g - 1, ffn ? H : A.keep_down * kTileRows,
                  kind == kLM ? A.out_norm : (ffn ? Ly->ffn_norm : Ly->attn_norm),
                  kind == kLM ? A.lm_signs : (ffn ? Ly->signs[2] : Ly->signs[0]), xq, xs, xm, U, S, step,
                  kind == kLM ? -1 : lb + (ffn ? kEvNorm2Res : kEvNorm1Res),
                  ffn && more ? A.layers + (l + 1 < A.L ? l + 1 : 0) : nullptr, &S.lay[(gl + 1) & 1],
                  ffn ? Ly->signs[3] : nullptr, dsg, A.I / 8);
        trace_at(A, step, kind == kLM ? sb + kEvNormF : lb + (ffn ? kEvNorm2 : kEvNorm1));
        // the first head this CTA hosts: its step-independent inputs are requested now
        if (kind == kQKV && head_lo < head_hi) attention_prefetch(A, Ly, l, pos, head_lo, U);
      } else {
        if (kind == kO) {
          for (int hh = head_lo; hh < head_hi; hh++)
            attention_head(A, Ly, l, pos, hh, g, U, hh == head_lo, S, step, lb + kEvAttnIn);
          if (head_lo == head_hi)
            for (int ev = kEvAttnIn; ev <= kEvAttnPV; ev++) trace_at(A, step, lb + ev);
          trace_at(A, step, lb + kEvAttn);
        }
        // the prepped input of o (from the attention CTAs) or of down (from the gate/up epilogues)
        load_prepped(A, kind == kO ? A.oprep : A.dprep, (kind == kO ? A.qd : A.I) / 64, g, xq, xs, xm, S);
        trace_at(A, step, lb + (kind == kO ? kEvLoadO : kEvLoadD));
      }
      consume_phase(A, step, l, kind, kind == kLM ? g_lm : g, ring, C, xq, xs, xm,
                    kind == kGU && Ly->signs[3] ? dsg : nullptr, S);
      if (kind != kLM) {
        cta_sync();
        if (kind == kGU) prep_down_owned(A, S.ph[kGU], g, Ly->signs[3] ? dsg : nullptr, S);
        trace_at(A, step, lb + (kind == kQKV ? kEvQKV : (kind == kO ? kEvO : (kind == kGU ? kEvGU : kEvDown))));
      }
    }
    trace_at(A, step, sb + kEvLM);
    {
      // this CTA's argmax partial (lanes of octet 0 of every warp hold running maxima)
      float bv = C.bv;
      int bi = C.bi;
      for (int m = 16; m; m >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, m);
        const int oi = __shfl_xor_sync(kFull, bi, m);
        better(bv, bi, ov, oi);
      }
      if (lane == 0) {
        S.arg_v[warp] = bv;
        S.arg_i[warp] = bi;
      }
      cta_sync();
      const int G_all = gridDim.x * A.tp_world;
      uint64_t* part = A.part + (size_t)(g_lm & 1) * G_all * 2;
      if (tid == 0) {
        for (int w = 1; w < kConsWarps; w++) better(bv, bi, S.arg_v[w], S.arg_i[w]);
        // other ranks' hosts read this CTA's logits once they have seen its partial
        if (A.write_logits) {
          if (A.tp_world > 1) __threadfence_system();
          else __threadfence();
        }
        put_tagged(A, part + 2 * vcta(A), tagged(bv, g_lm));
        put_tagged(A, part + 2 * vcta(A) + 1, ((uint64_t)g_lm << 32) | (unsigned)bi);
      }
      // every CTA reduces every CTA's partial (the partial buffers alternate with the
      // generation's parity, so a CTA already at the next step never overwrites one still read)
      bv = -INFINITY;
      bi = 0x7fffffff;
      for (int c0 = tid; c0 < G_all; c0 += 4 * kConsThreads) {
        // four CTAs' partials per round (value and index words)
        auto src = [&](int j) { return part + 2 * (c0 + (j >> 1) * kConsThreads) + (j & 1); };
        uint64_t wv[8];
        unsigned valid = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const bool ok = c0 + (j >> 1) * kConsThreads < G_all;
          wv[j] = ok ? ld_relaxed(src(j), A.tp_world > 1) : 0;
          if (ok) valid |= 1u << j;
        }
        wait_words(A, wv, stale_mask(wv, valid, g_lm), src, g_lm, S);
#pragma unroll
        for (int j = 0; j < 8; j += 2)
          if ((valid >> j) & 1u) better(bv, bi, value_of(wv[j]), (int)(unsigned)wv[j + 1]);
      }
      if (A.tp_world > 1 && A.write_logits) __threadfence_system();
      for (int m = 16; m; m >>= 1) {
        const float ov = __shfl_xor_sync(kFull, bv, m);
        const int oi = __shfl_xor_sync(kFull, bi, m);
        better(bv, bi, ov, oi);
      }
      cta_sync();
      if (lane == 0) {
        S.arg_v[warp] = bv;
        S.arg_i[warp] = bi;
      }
      cta_sync();
      if (tid == 0) {
        for (int w = 1; w < kConsWarps; w++) better(bv, bi, S.arg_v[w], S.arg_i[w]);
        // the winner is a row of the head; anything else (all logits NaN, or an aborted run)
        // feeds row 0 so that the embedding lookup stays in bounds
        const int id_next = (bi >= 0 && bi < A.V && bi < A.tok_rows) ? bi : 0;
        S.next_id = id_next;
        if (blockIdx.x == 0) A.hist[step] = id_next;
      }
      cta_sync();
    }
    trace_at(A, step, sb + kEvArg);
  }
}

}  // namespace

// Shared memory of one CTA: the ring | h | x (codes, block scales, block sums) | a union of the
// attention scratch (q, k, v, output, QK-norm gains, RoPE row, sign bytes, scores over max_seq
// keys, two value tiles), the norm staging (gains, sign bytes; and after norm2 the down
// projection's sign bytes, read by the gate/up epilogues) and the embedding staging (the row's
// group and the sign bytes).
size_t decode_union_bytes(const DecodeArgs& A) {
  const size_t attn = ((size_t)7 * A.hd + (((size_t)A.S + 3) & ~(size_t)3) + (size_t)2 * kVTile * A.hd) * sizeof(float) +
                      16 * (((size_t)A.hd / 8 + 15) / 16);
  const size_t norm = decode_norm_stage_bytes(A) + (size_t)A.I / 8;  // + the down projection's sign bytes
  const size_t embed = (size_t)(A.H / 32) * 144 + (size_t)A.H / 8 + 16;
  return std::max(attn, std::max(norm, embed));
}
size_t decode_smem_bytes(const DecodeArgs& A) {
  const size_t head = (size_t)A.n_slots * kSlotBytes + (size_t)A.H * 4 + (size_t)A.kmax + (size_t)(A.kmax / 32) * 8;
  return ((head + 15) & ~(size_t)15) + decode_union_bytes(A);
}

int decode_ring_slots(const DecodeArgs& A, size_t smem_limit) {
  DecodeArgs B = A;
  B.n_slots = 0;
  const size_t fixed = decode_smem_bytes(B);
  if (fixed >= smem_limit) return 0;
  return (int)std::min<size_t>(kMaxSlots, (smem_limit - fixed) / kSlotBytes);
}

int decode_trace_events(int L) { return kEvPerLayer * L + kEvPerStep; }

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
  if (A.n_slots < 2 * kConsWarps + 2 || A.n_slots > kMaxSlots || A.max_inflight < kConsWarps || A.max_inflight + kConsWarps >= A.n_slots)
    return cudaErrorInvalidValue;
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
