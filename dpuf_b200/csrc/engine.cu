// engine.cu - the persistent DPUF engine on one B200, behind the reference's C ABI
// (dpuf_kernels.h:316-360; semantics of dpuf_engine.c:1182-2170).
//
// Device memory layout (all resident for the engine's lifetime):
//   weight arena   every mode-12 matrix in container layout (tiles, tile offsets rebased to
//                  the tile span, sign bits), norm gains, RoPE tables - uploaded once at create
//   KV slots       up to 8 caches [L][n_kv][max_seq][hd] fp32, allocated on first use
//   prefixes       up to 8 frozen prefixes [L][n_kv][len][hd]
//   activations    h, hn, q, k, v, att, gate, up [256][dim] fp32; three prep slots (int8
//                  codes, block scales, block sums); logits [256][vocab]
// A forward step is one stream of kernels (see enqueue_step) captured once per shape and
// environment knobs into a CUDA graph; token ids and the start position are copied from
// pinned staging by the graph itself, so one graph serves every position.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <set>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "dpuf_cuda.h"
#include "dpuf_kernels.h"
#include "engine_internal.h"
#include "kernels.cuh"

namespace dpuf {

namespace {
thread_local std::string g_err;
}
void set_error(const std::string& msg) { g_err = msg; }

cudaError_t configure_mode12_kernels();
cudaError_t configure_layer_kernels();
cudaError_t configure_attn_kernels();
cudaError_t configure_kernels() {
  cudaError_t e;
  if ((e = configure_mode12_kernels()) != cudaSuccess) return e;
  if ((e = configure_had_engine_kernels()) != cudaSuccess) return e;
  if ((e = configure_layer_kernels()) != cudaSuccess) return e;
  if ((e = configure_decode_kernel()) != cudaSuccess) return e;
  if ((e = configure_gemm_tc_kernels()) != cudaSuccess) return e;
  return configure_attn_kernels();
}

namespace {

constexpr int kMaxSlots = 8;       // the reference's slot count (DPUF_MAX_SLOTS)
constexpr int kMaxSlotsEnv = 256;  // upper bound of env DPUF_CUDA_SLOTS (batched serving)
constexpr int kMaxPrefixes = 8;

#define CK(expr)                                                                                  \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess) {                                                                      \
      set_error(std::string(#expr) + ": " + cudaGetErrorString(_e) + " (" __FILE__ ":" +         \
                std::to_string(__LINE__) + ")");                                                  \
      return _e;                                                                                  \
    }                                                                                             \
  } while (0)

struct LayerDev {
  W12 q, k, v, o, gate, up, down;
  const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
};

struct Slot {
  float* k = nullptr;
  float* v = nullptr;
};
struct Prefix {
  float* k = nullptr;
  float* v = nullptr;
  int len = 0, cap = 0;
  bool valid = false;
};

struct StepKey {
  int M, only_last, keep, za;
  uint32_t margin_bits;
  int slot, greedy_loop, batch;
  bool operator<(const StepKey& o) const {
    return std::tie(M, only_last, keep, za, margin_bits, slot, greedy_loop, batch) <
           std::tie(o.M, o.only_last, o.keep, o.za, o.margin_bits, o.slot, o.greedy_loop, o.batch);
  }
};

// Pinned staging shared by the host and the captured graphs.
struct Staging {
  int32_t ids[kMaxBatch];
  int32_t pos0;
  int32_t pad[3];
};
// Per-row inputs of a batched decode step (rows are independent sequences): position and the
// row's slot cache.
struct BatchStaging {
  int32_t pos[kMaxBatch];
  float* k[kMaxBatch];
  float* v[kMaxBatch];
};

struct Engine {
  DpufModelConfig cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  bool use_pdl = true, use_graphs = true;
  int H, I, L, nq, nkv, hd, qd, kvd, V, S, act_ld;
  float deadzone = 0.005f;
  int nt_ref = 8;

  unsigned char* arena = nullptr;
  std::vector<LayerDev> layers;
  W12 tok, lm;
  const float* out_norm = nullptr;
  float *cos_tab = nullptr, *sin_tab = nullptr;

  std::vector<Slot> slots;  // kMaxSlots, or env DPUF_CUDA_SLOTS for batched serving
  bool stage_neg[kMaxBatch] = {};  // rows of the current step taken from embeds_in
  int kv_kind = kKvF32;     // KvKind: fp32 (kv_type 0), Q8 (kv_type 1), fp16 (env DPUF_CUDA_KV_F16=1, kv_type 0)
  size_t kv_row = 0;        // bytes of one KV head's cache row at one position
  int n_slots = kMaxSlots;
  int active = 0;
  Prefix prefixes[kMaxPrefixes];

  float *h = nullptr, *hn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *gate = nullptr,
        *up = nullptr, *logits = nullptr;
  Act prep[3];
  int8_t* prep_q8 = nullptr;
  float* prep_xs = nullptr;
  int32_t* prep_xm = nullptr;
  int32_t* d_ids = nullptr;
  int32_t* d_pos0 = nullptr;
  int* d_flag = nullptr;
  float* d_b12 = nullptr;
  int32_t* d_argmax = nullptr;
  int32_t* d_hist = nullptr;   // greedy-loop token history [max_seq] and step counter
  int32_t* d_hist_step = nullptr;
  Staging* stage = nullptr;  // pinned
  BatchStaging* bstage = nullptr;  // pinned
  BatchStaging* d_bstage = nullptr;
  int32_t* d_next = nullptr;       // greedy ids of a batched step [kMaxBatch]
  float* d_ds = nullptr;           // DeepStack rows of the current step [3][kMaxBatch][H], on first use
  float* d_tok_rope = nullptr;     // per-token cos | sin rows [2][kMaxBatch][hd/2], on first use
  std::vector<float> h_cos, h_sin; // host copies of the RoPE tables [max_seq][hd/2]
  std::vector<float> h_tok_rope;   // staging of d_tok_rope
  float* h_logits = nullptr; // pinned [256][V] staging is too large; [V] for the last row
  uint2* d_exp_slots = nullptr;
  unsigned* d_counter = nullptr;  // last-block counters of the multi-CTA argmax
  float2* d_part = nullptr;       // per-CTA argmax partials
  GemvSplit split{};              // GEMV scratch for 16-row units shared by CTAs
  ExpfTable et{};

  std::map<StepKey, cudaGraphExec_t> graphs;
  // last step
  int last_rows = 0, last_zone_used = 0;

  bool use_tc_gemm = true;  // M > 1 projections on the tensor cores (else the dp4a GEMM)
  int* d_tc_err = nullptr;  // error word of the tensor-core GEMM
  unsigned char* x8_arena = nullptr;  // expanded copies of the mode-12 matrices (W12::x8)
  bool has_had = false;               // some matrix is in mode 13 or 14

  // persistent batch-1 decode (kernels_decode.cu)
  bool dec_ok = false, use_persistent = true;
  std::string dec_why;     // why the persistent kernel is not used
  DecodeArgs dec{};        // everything but the per-call fields
  DecLayer* d_dec_layers = nullptr;
  // the persistent kernel's exchange area on one GPU (tagged vectors, down-input counters and
  // prep, argmax partials, error word; layout dec_layout) and this GPU's prepped o input
  unsigned char* dec_xbuf = nullptr;
  size_t dec_xbytes = 0;
  uint64_t* dec_oprep = nullptr;
  unsigned dec_gen = 1;  // exchange generation of the next persistent launch's first layer
  int dec_failed = 0;    // the last persistent launch gave up a wait (reset the exchange first)
  int dec_stall_next = -1;  // test hook: q/k/v unit whose rows are withheld in the next launch
  float* last_logits = nullptr;  // where the last step's logits are (per-step or persistent)

  // tensor parallelism of the persistent decode (dpuf_cuda_tp_handle / dpuf_cuda_tp_attach)
  int tp_rank = 0, tp_world = 1;     // world > 1 once attached
  int tp_pending = 0;                // world announced by dpuf_cuda_tp_handle
  unsigned char* tp_buf = nullptr;   // this rank's exchange buffer (exported by IPC handle)
  size_t tp_bytes = 0;
  void* tp_peer[kMaxTp] = {};        // other ranks' exchange buffers, opened
};

// Synchronises the engine's stream; on failure records the CUDA error (a kernel fault surfaces here).
bool sync_ok(const Engine* e) {
  const cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err == cudaSuccess) return true;
  set_error(std::string("stream synchronisation: ") + cudaGetErrorString(err));
  return false;
}

// ------------------------------------------------------------------ helpers
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Bytes of tile data of a matrix: from its first tile to the end of its last tile (computed
// from the last tile's row count, since the tile offset array has n_tiles entries in the ABI).
size_t tile_span(const DpufWeightDesc& w, uint64_t* base_off) {
  uint64_t lo = w.tile_offsets[0], hi = 0;
  // bytes of one 8-row group: mode 12 per 32 columns 144 (scales + nibbles), modes 13 / 14
  // per 64 columns 288 / 416 (d, m, nibbles, mode 14's high bit pairs)
  const uint64_t grp = w.mode == DPUF_MODE_QR_HAD6 ? (uint64_t)(w.cols / 64) * 416
                       : w.mode == DPUF_MODE_QR_HAD4_ASYM ? (uint64_t)(w.cols / 64) * 288
                                                          : (uint64_t)(w.cols / 32) * 144;
  for (int t = 0; t < w.n_tiles; t++) {
    const uint8_t* tp = w.tensor_base + w.tile_offsets[t];
    const int n_r = tp[4] | (tp[5] << 8);
    const uint64_t end = w.tile_offsets[t] + 16 + (uint64_t)((n_r + 7) / 8) * grp;
    lo = std::min<uint64_t>(lo, w.tile_offsets[t]);
    hi = std::max<uint64_t>(hi, end);
  }
  *base_off = lo;
  return (size_t)(hi - lo);
}

// Modes 12 (QR_HAD4_PACKED) and, on the per-step path, 13 / 14 (QR_HAD4_ASYM / QR_HAD6: the
// reference's had4p-hybrid packing, dpuf_engine.c:1079-1088).
bool desc_ok(const DpufWeightDesc& w, int rows, int cols) {
  if (w.mode != DPUF_MODE_QR_HAD4_PACKED && w.mode != DPUF_MODE_QR_HAD4_ASYM && w.mode != DPUF_MODE_QR_HAD6) return false;
  if (!w.tensor_base || !w.tile_offsets || !w.sign_bits) return false;
  if (w.rows != rows || w.cols != cols || (cols % 64) != 0) return false;
  if (w.n_tiles != (rows + kTileRows - 1) / kTileRows) return false;
  for (int t = 0; t < w.n_tiles; t++)  // the GEMV streams tiles with 16-byte async copies
    if (w.tile_offsets[t] % 16 != 0) return false;
  return true;
}

// Arena builder: first pass sizes, second pass uploads.  Matrices shared by pointer (tied
// embeddings) are uploaded once.
struct ArenaPlan {
  size_t bytes = 0;
  std::map<const uint8_t*, size_t> tile_at, toff_at, sign_at;
  std::map<std::string, size_t> sign_by_content;  // equal sign tables share one device copy
  std::map<const float*, size_t> f32_at;
};

void plan_w(ArenaPlan& P, const DpufWeightDesc& w) {
  if (P.tile_at.count(w.tensor_base)) return;
  uint64_t base;
  const size_t span = tile_span(w, &base);
  P.tile_at[w.tensor_base] = P.bytes;
  P.bytes = align256(P.bytes + span);
  P.toff_at[w.tensor_base] = P.bytes;
  P.bytes = align256(P.bytes + (size_t)w.n_tiles * 8);
  const std::string key((const char*)w.sign_bits, (size_t)w.cols / 8);
  auto it = P.sign_by_content.find(key);
  if (it == P.sign_by_content.end()) {
    it = P.sign_by_content.emplace(key, P.bytes).first;
    P.bytes = align256(P.bytes + (size_t)w.cols / 8);
  }
  P.sign_at[w.tensor_base] = it->second;
}

void plan_f(ArenaPlan& P, const float* f, int n) {
  if (!f || P.f32_at.count(f)) return;
  P.f32_at[f] = P.bytes;
  P.bytes = align256(P.bytes + (size_t)n * 4);
}

cudaError_t upload_w(Engine* e, const ArenaPlan& P, const DpufWeightDesc& w, W12* out, std::set<size_t>& done) {
  const size_t t_at = P.tile_at.at(w.tensor_base);
  out->tiles = e->arena + t_at;
  out->toff = (const uint64_t*)(e->arena + P.toff_at.at(w.tensor_base));
  out->signs = e->arena + P.sign_at.at(w.tensor_base);
  out->rows = w.rows;
  out->cols = w.cols;
  out->n_tiles = w.n_tiles;
  out->mode = w.mode;
  if (w.mode != DPUF_MODE_QR_HAD4_PACKED) e->has_had = true;
  if (!done.insert(t_at).second) return cudaSuccess;
  uint64_t base;
  const size_t span = tile_span(w, &base);
  CK(cudaMemcpy(e->arena + t_at, w.tensor_base + base, span, cudaMemcpyHostToDevice));
  std::vector<uint64_t> toff(w.n_tiles);
  for (int t = 0; t < w.n_tiles; t++) toff[t] = w.tile_offsets[t] - base;
  CK(cudaMemcpy((void*)out->toff, toff.data(), toff.size() * 8, cudaMemcpyHostToDevice));
  CK(cudaMemcpy((void*)out->signs, w.sign_bits, (size_t)w.cols / 8, cudaMemcpyHostToDevice));
  return cudaSuccess;
}

const float* upload_f(Engine* e, const ArenaPlan& P, const float* f, int n) {
  if (!f) return nullptr;
  const size_t at = P.f32_at.at(f);
  if (cudaMemcpy(e->arena + at, f, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
  return (const float*)(e->arena + at);
}

// RoPE tables exactly as precompute_rope (dpuf_engine.c:183-223), computed on the host with
// the same libm calls.
void rope_tables(const DpufModelConfig& c, std::vector<float>& cs, std::vector<float>& sn) {
  const int hd = c.head_dim, half = hd / 2;
  std::vector<float> inv(half);
  for (int j = 0; j < half; j++) {
    float freq = 1.0f / powf(c.rope_theta, (float)(2 * j) / (float)hd);
    if (c.use_llama3_rope) {
      const float factor = c.rope_factor, low_f = c.rope_low_freq, high_f = c.rope_high_freq;
      const float orig = (float)c.rope_orig_max_pos;
      const float wavelen = (2.0f * (float)3.14159265358979323846) / freq;
      const float low_w = orig / low_f, high_w = orig / high_f;
      if (wavelen > low_w) {
        freq /= factor;
      } else if (wavelen >= high_w) {
        const float smooth = (orig / wavelen - low_f) / (high_f - low_f);
        freq = (1.0f - smooth) * (freq / factor) + smooth * freq;
      }
    }
    inv[j] = freq;
  }
  cs.resize((size_t)c.max_seq_len * half);
  sn.resize(cs.size());
  for (int p = 0; p < c.max_seq_len; p++) {
    const float pf = (float)p;
    for (int j = 0; j < half; j++) {
      const float ang = pf * inv[j];
      cs[(size_t)p * half + j] = cosf(ang);
      sn[(size_t)p * half + j] = sinf(ang);
    }
  }
}

cudaError_t slot_alloc(Engine* e, int s) {
  if (e->slots[s].k) return cudaSuccess;
  const size_t n = (size_t)e->L * e->S * e->nkv * e->kv_row;  // bytes
  CK(cudaMalloc(&e->slots[s].k, n));
  CK(cudaMalloc(&e->slots[s].v, n));
  CK(cudaMemset(e->slots[s].k, 0, n));
  CK(cudaMemset(e->slots[s].v, 0, n));
  return cudaSuccess;
}

int env_int(const char* name, int def);

// Expanded copies of the mode-12 matrices the tensor-core GEMM streams at M > 1 (W12::x8), one
// per distinct matrix, unless env DPUF_CUDA_TC_EXPAND=0 or DPUF_CUDA_TC_GEMM=0 at create (the
// "tc_gemm" option switched on later then runs the unpacking kernel).  When the allocation fails,
// or a matrix holds a scale that is not finite, the GEMM unpacks that matrix's tiles itself.
cudaError_t build_expanded(Engine* e) {
  if (!e->use_tc_gemm || env_int("DPUF_CUDA_TC_EXPAND", 1) == 0) return cudaSuccess;
  std::vector<W12*> ws;
  for (LayerDev& d : e->layers)
    for (W12* w : {&d.q, &d.k, &d.v, &d.o, &d.gate, &d.up, &d.down}) ws.push_back(w);
  ws.push_back(&e->lm);
  std::map<const uint8_t*, size_t> at;  // by tile data: shared matrices are expanded once
  std::map<const uint8_t*, int> idx;
  size_t bytes = 0;
  for (W12* w : ws)
    if (w->mode == 12 && !at.count(w->tiles)) {
      idx[w->tiles] = (int)at.size();
      at[w->tiles] = bytes;
      bytes = align256(bytes + x8_bytes(*w));
    }
  if (!bytes) return cudaSuccess;
  if (cudaMalloc(&e->x8_arena, bytes) != cudaSuccess) {
    cudaGetLastError();  // not fatal
    e->x8_arena = nullptr;
    return cudaSuccess;
  }
  int* bad = nullptr;
  CK(cudaMalloc(&bad, at.size() * sizeof(int)));
  std::vector<int> h_bad(at.size(), 0);
  cudaError_t err = cudaMemsetAsync(bad, 0, at.size() * sizeof(int), e->stream);
  for (auto it = idx.begin(); err == cudaSuccess && it != idx.end(); ++it) {
    const W12* w = nullptr;
    for (W12* c : ws)
      if (c->tiles == it->first) w = c;
    err = launch_x8_expand(e->stream, *w, e->x8_arena + at[it->first], bad + it->second);
  }
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(h_bad.data(), bad, h_bad.size() * sizeof(int), cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  cudaFree(bad);
  if (err != cudaSuccess) return err;
  for (W12* w : ws)
    if (w->mode == 12 && !h_bad[idx[w->tiles]]) w->x8 = e->x8_arena + at[w->tiles];
  return cudaSuccess;
}

void destroy_engine(Engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& s : e->slots) { cudaFree(s.k); cudaFree(s.v); }
  for (auto& p : e->prefixes) { cudaFree(p.k); cudaFree(p.v); }
  cudaFree(e->arena);
  cudaFree(e->x8_arena);
  cudaFree(e->cos_tab); cudaFree(e->sin_tab);
  cudaFree(e->h); cudaFree(e->hn); cudaFree(e->q); cudaFree(e->k); cudaFree(e->v); cudaFree(e->att);
  cudaFree(e->gate); cudaFree(e->up); cudaFree(e->logits);
  cudaFree(e->prep_q8); cudaFree(e->prep_xs); cudaFree(e->prep_xm);
  cudaFree(e->d_ids); cudaFree(e->d_hist); cudaFree(e->d_flag); cudaFree(e->d_b12); cudaFree(e->d_argmax);
  cudaFree(e->d_exp_slots); cudaFree(e->d_counter); cudaFree(e->d_part); cudaFree(e->d_tc_err);
  cudaFree(e->split.pairs); cudaFree(e->split.acc); cudaFree(e->split.count);
  cudaFree(e->d_dec_layers); cudaFree(e->dec_xbuf); cudaFree(e->dec_oprep); cudaFree(e->dec.trace);
  for (void* p : e->tp_peer)
    if (p) cudaIpcCloseMemHandle(p);
  cudaFree(e->tp_buf);
  cudaFreeHost(e->stage); cudaFreeHost(e->h_logits); cudaFreeHost(e->bstage);
  cudaFree(e->d_bstage); cudaFree(e->d_next); cudaFree(e->d_ds); cudaFree(e->d_tok_rope);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

// ------------------------------------------------------------------ the forward step
struct StepParams {
  int M, only_last, keep, za;
  float margin;
  bool greedy_loop;  // ids/pos live on the device and advance by greedy feedback
  bool batch = false;  // rows are independent sequences (per-row slot and position)
  const float* embeds = nullptr;  // host [M][H] rows for ids < 0 (or all rows without ids)
  bool all_embeds = false;        // every row comes from `embeds`
  int ds_mask = 0;                // layers (bit l, l < 3) whose down output gets d_ds[l] added
  bool tok_rope = false;          // tokens rotate by d_tok_rope rows (forward_batch_ex positions)
};

LinJobs one_job(const W12& w, const Act& a, float* out, int ldo, int t0, int t1) {
  LinJobs J = {};
  J.n = 1;
  J.j[0] = {w, a, out, ldo, t0, t1};
  J.tile_prefix[0] = 0;
  J.tile_prefix[1] = t1 - t0;
  return J;
}

cudaError_t run_linear_m12(const Engine* e, const Launch& Lc, const LinJobs& J, int M, const int* skip) {
  if (J.tile_prefix[J.n] == 0) return cudaSuccess;
  if (M == 1) return launch_gemv(Lc, J, skip, &e->split);
  return e->use_tc_gemm ? launch_gemm_tc(Lc, J, M, e->d_tc_err) : launch_gemm_exact(Lc, J, M);
}

// The jobs' matmuls: mode-12 jobs together (one launch), mode-13/14 jobs one launch each.  A set
// `skip` flag (the Zone-A exit) turns every launch into no work.
cudaError_t run_linear(const Engine* e, const Launch& Lc, const LinJobs& J, int M, const int* skip) {
  bool any_had = false;
  for (int i = 0; i < J.n; i++) any_had |= J.j[i].w.mode != 12;
  if (!any_had) return run_linear_m12(e, Lc, J, M, skip);
  LinJobs J12 = {};
  J12.tile_prefix[0] = 0;
  for (int i = 0; i < J.n; i++) {
    const LinJob& jb = J.j[i];
    if (jb.w.mode == 12) {
      J12.j[J12.n] = jb;
      J12.tile_prefix[J12.n + 1] = J12.tile_prefix[J12.n] + (jb.t_end - jb.t_begin);
      J12.n++;
    } else {
      CK(launch_had_w(Lc.stream, jb.w, jb.act, M, jb.out, jb.ldo, jb.t_begin, jb.t_end, skip, e->d_tc_err));
    }
  }
  return J12.n ? run_linear_m12(e, Lc, J12, M, skip) : cudaSuccess;
}

// Prep targets for weights sharing one input: identical sign tables share a prep slot
// (weights_share_prep, dpuf_engine.c:887-897).  slot_of[i] receives the slot used by w[i].
int prep_targets(Engine* e, const W12* const* ws, int n, PrepTarget* t, int* slot_of) {
  int nt = 0;
  for (int i = 0; i < n; i++) {
    int found = -1;
    for (int j = 0; j < nt; j++)
      if (t[j].signs == ws[i]->signs) found = j;  // same device copy <=> same sign table
    if (found < 0) {
      t[nt].signs = ws[i]->signs;
      t[nt].act = e->prep[nt];
      found = nt++;
    }
    slot_of[i] = found;
  }
  return nt;
}

cudaError_t enqueue_step(Engine* e, const StepParams& P) {
  const Launch Lc{e->stream, e->use_pdl};
  const int M = P.M, H = e->H;
  if (!P.greedy_loop)
    CK(cudaMemcpyAsync(e->d_ids, e->stage, sizeof(Staging), cudaMemcpyHostToDevice, e->stream));
  if (P.batch)
    CK(cudaMemcpyAsync(e->d_bstage, e->bstage, sizeof(BatchStaging), cudaMemcpyHostToDevice, e->stream));
  if (!P.all_embeds)
    CK(e->tok.mode == 12 ? launch_embed(Lc, e->tok, e->d_ids, M, e->h)
                         : launch_had_embed_w(Lc.stream, e->tok, e->d_ids, M, e->h));
  if (P.embeds)  // rows given by the caller (dpuf_engine.c:1658-1672); ids < 0 were staged as 0
    for (int m = 0; m < M; m++)
      if (P.all_embeds || e->stage_neg[m])
        CK(cudaMemcpyAsync(e->h + (size_t)m * H, P.embeds + (size_t)m * H, (size_t)H * 4, cudaMemcpyHostToDevice,
                           e->stream));
  const Slot& sl = e->slots[e->active];
  for (int l = 0; l < e->L; l++) {
    const LayerDev& lw = e->layers[l];
    const size_t layer_off = (size_t)l * e->nkv * e->S * e->kv_row;  // bytes
    KvCache kv{(float*)((char*)sl.k + layer_off), (float*)((char*)sl.v + layer_off), e->S, nullptr, nullptr, nullptr, 0,
               e->kv_kind};
    if (P.batch)
      kv = KvCache{nullptr, nullptr, e->S, e->d_bstage->pos, e->d_bstage->k, e->d_bstage->v, layer_off, e->kv_kind};
    // 1-2. [h += hn] RMSNorm + prep of q/k/v inputs
    {
      const W12* ws[3] = {&lw.q, &lw.k, &lw.v};
      PrepTarget t[3];
      int so[3];
      const int n = prep_targets(e, ws, 3, t, so);
      CK(launch_norm_prep(Lc, e->h, l > 0 ? e->hn : nullptr, lw.attn_norm, e->cfg.rms_eps, M, H, t, n, nullptr));
      LinJobs J = {};
      float* outs[3] = {e->q, e->k, e->v};
      const int ldo[3] = {e->qd, e->kvd, e->kvd};
      J.n = 3;
      J.tile_prefix[0] = 0;
      for (int i = 0; i < 3; i++) {
        J.j[i] = {*ws[i], e->prep[so[i]], outs[i], ldo[i], 0, ws[i]->n_tiles};
        J.tile_prefix[i + 1] = J.tile_prefix[i] + ws[i]->n_tiles;
      }
      CK(run_linear(e, Lc, J, M, nullptr));
    }
    // 3-4. QK norm, RoPE, KV store; attention
    CK(launch_qk_post(Lc, e->q, e->k, e->v, M, e->nq, e->nkv, e->hd, e->cfg.has_qk_norm ? lw.q_norm : nullptr,
                      e->cfg.has_qk_norm ? lw.k_norm : nullptr, e->cfg.rms_eps, e->cos_tab, e->sin_tab, e->d_pos0,
                      kv, P.tok_rope ? e->d_tok_rope : nullptr,
                      P.tok_rope ? e->d_tok_rope + (size_t)kMaxBatch * (e->hd / 2) : nullptr));
    CK(launch_attention(Lc, e->q, M, e->nq, e->nkv, e->hd, e->d_pos0, kv, e->att, e->et));
    // 5. o_proj
    CK(launch_prep(Lc, e->att, e->qd, M, e->qd, lw.o.signs, e->prep[0]));
    CK(run_linear(e, Lc, one_job(lw.o, e->prep[0], e->hn, H, 0, lw.o.n_tiles), M, nullptr));
    // 6-8. h += o; RMSNorm; gate/up
    {
      const W12* ws[2] = {&lw.gate, &lw.up};
      PrepTarget t[2];
      int so[2];
      const int n = prep_targets(e, ws, 2, t, so);
      CK(launch_norm_prep(Lc, e->h, e->hn, lw.ffn_norm, e->cfg.rms_eps, M, H, t, n, nullptr));
      LinJobs J = {};
      J.n = 2;
      J.tile_prefix[0] = 0;
      J.j[0] = {lw.gate, e->prep[so[0]], e->gate, e->I, 0, lw.gate.n_tiles};
      J.tile_prefix[1] = lw.gate.n_tiles;
      J.j[1] = {lw.up, e->prep[so[1]], e->up, e->I, 0, lw.up.n_tiles};
      J.tile_prefix[2] = lw.gate.n_tiles + lw.up.n_tiles;
      CK(run_linear(e, Lc, J, M, nullptr));
    }
    // 9-11. SwiGLU + prep, down (optionally pruned to the first `keep` tiles)
    CK(launch_swiglu_prep(Lc, e->gate, e->up, M, e->I, e->deadzone, e->nt_ref, lw.down.signs, e->prep[0], e->et,
                          P.batch));
    const int keep = (P.keep > 0 && P.keep < lw.down.n_tiles) ? P.keep : lw.down.n_tiles;
    CK(run_linear(e, Lc, one_job(lw.down, e->prep[0], e->hn, H, 0, keep), M, nullptr));
    if (keep < lw.down.n_tiles) CK(launch_zero_rows(Lc, e->hn, M, H, keep * kTileRows));
    if (l < 3 && ((P.ds_mask >> l) & 1))  // DeepStack injection (dpuf_engine.c:2046-2054)
      CK(launch_add_rows(Lc, e->hn, e->d_ds + (size_t)l * kMaxBatch * H, M * H));
  }
  if (P.only_last == 2) return cudaSuccess;
  const int lm_start = P.only_last ? M - 1 : 0, lm_M = M - lm_start;
  {
    const W12* ws[1] = {&e->lm};
    PrepTarget t[1];
    int so[1];
    prep_targets(e, ws, 1, t, so);
    CK(launch_norm_prep(Lc, e->h + (size_t)lm_start * H, e->L > 0 ? e->hn + (size_t)lm_start * H : nullptr,
                        e->out_norm, e->cfg.rms_eps, lm_M, H, t, 1, nullptr));
  }
  if (P.za > 0) {
    const int n_za = std::min(P.za * kTileRows, e->V);
    CK(run_linear(e, Lc, one_job(e->lm, e->prep[0], e->logits, e->V, 0, P.za), 1, nullptr));
    CK(launch_zone_test(Lc, e->logits, n_za, P.margin, e->d_flag, e->d_b12));
    CK(run_linear(e, Lc, one_job(e->lm, e->prep[0], e->logits, e->V, P.za, e->lm.n_tiles), 1, e->d_flag));
    CK(launch_zone_mask(Lc, e->logits, P.za * kTileRows, e->V, e->d_flag));
  } else {
    CK(run_linear(e, Lc, one_job(e->lm, e->prep[0], e->logits, e->V, 0, e->lm.n_tiles), lm_M, nullptr));
  }
  if (P.greedy_loop)
    CK(launch_greedy_advance(Lc, e->logits, e->V, e->d_part, e->d_counter, e->d_ids, e->d_pos0, e->d_hist,
                             e->d_hist_step));
  if (P.batch) CK(launch_argmax_rows(Lc, e->logits, e->V, lm_M, e->d_next));
  return cudaSuccess;
}

cudaError_t run_step(Engine* e, const StepParams& P) {
  if (!e->use_graphs || P.embeds || P.ds_mask || P.tok_rope) return enqueue_step(e, P);  // caller rows: no graph
  uint32_t mb;
  memcpy(&mb, &P.margin, 4);
  // a batched step reads its slots' caches through device pointers, so its graph does not
  // depend on the active slot
  const StepKey key{P.M, P.only_last, P.keep, P.za, mb, P.batch ? -1 : e->active, P.greedy_loop ? 1 : 0,
                    P.batch ? 1 : 0};
  auto it = e->graphs.find(key);
  if (it == e->graphs.end()) {
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t err = enqueue_step(e, P);
    cudaError_t err2 = cudaStreamEndCapture(e->stream, &g);
    if (err != cudaSuccess) return err;
    CK(err2);
    cudaGraphExec_t ge;
    err = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    CK(err);
    it = e->graphs.emplace(key, ge).first;
  }
  CK(cudaGraphLaunch(it->second, e->stream));
  return cudaSuccess;
}

void drop_graphs(Engine* e) {
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  e->graphs.clear();
}

int env_int(const char* name, int def) {
  const char* s = getenv(name);
  return s ? atoi(s) : def;
}

// ------------------------------------------------------------------ persistent decode
// Tile stride of a matrix whose tiles are equally spaced (what the reference's packer writes);
// false otherwise.  *first = byte offset of tile 0 from the start of the uploaded span.
bool uniform_tiles(const DpufWeightDesc& w, long long* stride, long long* first) {
  uint64_t base;
  tile_span(w, &base);
  *first = (long long)(w.tile_offsets[0] - base);
  *stride = w.n_tiles > 1 ? (long long)(w.tile_offsets[1] - w.tile_offsets[0]) : 0;
  if (w.n_tiles > 1 && *stride <= 0) return false;
  for (int t = 0; t < w.n_tiles; t++)
    if ((long long)(w.tile_offsets[t] - w.tile_offsets[0]) != (long long)t * *stride) return false;
  return true;
}

// Exchange area of the persistent kernel on one GPU: the tagged vectors, the down input's raw
// values, chunk counters and prep, the argmax partials, the logits and the error word.  Under
// tensor parallelism every rank holds one (the IPC-shared buffer) and producers store into every
// rank's copy.  Zeroed at allocation: every tag is 0 and the first launch's generation is 1.
struct DecLayout {
  size_t err, q, k, v, o, d, dprep, s_raw, logits, part, total;
};
DecLayout dec_layout(const Engine* e, int world, int grid) {
  DecLayout t{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return o;
  };
  t.err = take(4);
  t.q = take((size_t)e->qd * 8);
  t.k = take((size_t)e->kvd * 8);
  t.v = take((size_t)e->kvd * 8);
  t.o = take((size_t)e->H * 8);
  t.d = take((size_t)e->H * 8);
  t.dprep = take((size_t)(e->I / 64) * 20 * 8);
  t.s_raw = take((size_t)e->I * 8);
  t.logits = take((size_t)e->V * 4);
  t.part = take((size_t)2 * world * grid * 16);
  t.total = off;
  return t;
}
void dec_bind(DecodeArgs& A, unsigned char* base, const DecLayout& t) {
  A.err = (int*)(base + t.err);
  A.q = (uint64_t*)(base + t.q);
  A.k = (uint64_t*)(base + t.k);
  A.v = (uint64_t*)(base + t.v);
  A.o_out = (uint64_t*)(base + t.o);
  A.d_out = (uint64_t*)(base + t.d);
  A.dprep = (uint64_t*)(base + t.dprep);
  A.s_raw = (uint64_t*)(base + t.s_raw);
  A.logits = (float*)(base + t.logits);
  A.part = (uint64_t*)(base + t.part);
}

// Decides whether batch-1 steps run as the persistent kernel and prepares its arguments.
// Falls back (dec_ok = false, reason in dec_why) when a matrix's tiles are not equally
// spaced, when co-inputs use different sign tables, or when the device cannot hold one CTA
// per SM with a ring of at least four stages.
void plan_decode(Engine* e, const DpufLayerWeights* lw, const DpufWeightDesc* tok, const DpufWeightDesc* lm) {
  auto no = [&](const std::string& why) { e->dec_ok = false; e->dec_why = why; };
  if (e->kv_kind == kKvF16) return no("fp16 KV cache (the persistent kernel keeps the reference's fp32 cache)");
  if (e->kv_kind == kKvQ8) return no("Q8 KV cache (kv_type 1 runs on the per-step kernels)");
  int coop = 0, sms = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, e->device) != cudaSuccess || !coop)
    return no("device without cooperative launch");
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, e->device) != cudaSuccess || sms <= 0)
    return no("SM count");
  if (tok->mode != DPUF_MODE_QR_HAD4_PACKED || lm->mode != DPUF_MODE_QR_HAD4_PACKED)
    return no("a mode-13/14 embedding or LM head (the per-step kernels serve it)");
  for (int l = 0; l < e->L; l++) {
    const DpufLayerWeights& w = lw[l];
    for (const DpufWeightDesc* d : {&w.w_q, &w.w_k, &w.w_v, &w.w_o, &w.w_gate, &w.w_up, &w.w_down})
      if (d->mode != DPUF_MODE_QR_HAD4_PACKED) return no("mode-13/14 layers (the per-step kernels serve them)");
  }
  std::vector<DecLayer> tab(e->L);
  for (int l = 0; l < e->L; l++) {
    const DpufLayerWeights& w = lw[l];
    const LayerDev& d = e->layers[l];
    const DpufWeightDesc* ws[7] = {&w.w_q, &w.w_k, &w.w_v, &w.w_o, &w.w_gate, &w.w_up, &w.w_down};
    const W12* dw[7] = {&d.q, &d.k, &d.v, &d.o, &d.gate, &d.up, &d.down};
    for (int i = 0; i < 7; i++) {
      long long first;
      if (!uniform_tiles(*ws[i], &tab[l].stride[i], &first)) return no("tiles not equally spaced");
      tab[l].tiles[i] = dw[i]->tiles + first;
    }
    if (d.q.signs != d.k.signs || d.q.signs != d.v.signs || d.gate.signs != d.up.signs)
      return no("co-inputs with different sign tables");
    tab[l].signs[0] = d.q.signs;
    tab[l].signs[1] = d.o.signs;
    tab[l].signs[2] = d.gate.signs;
    tab[l].signs[3] = d.down.signs;
    tab[l].attn_norm = d.attn_norm;
    tab[l].ffn_norm = d.ffn_norm;
    tab[l].q_norm = e->cfg.has_qk_norm ? d.q_norm : nullptr;
    tab[l].k_norm = e->cfg.has_qk_norm ? d.k_norm : nullptr;
  }
  DecodeArgs& A = e->dec;
  A = DecodeArgs{};
  long long first;
  if (!uniform_tiles(*lm, &A.lm_stride, &first)) return no("tiles not equally spaced");
  A.lm_tiles = e->lm.tiles + first;
  if (!uniform_tiles(*tok, &A.tok_stride, &first)) return no("tiles not equally spaced");
  A.tok_tiles = e->tok.tiles + first;
  A.lm_signs = e->lm.signs;
  A.tok_signs = e->tok.signs;
  A.L = e->L; A.H = e->H; A.I = e->I; A.nq = e->nq; A.nkv = e->nkv; A.hd = e->hd; A.qd = e->qd; A.kvd = e->kvd;
  A.V = e->V; A.S = e->S; A.kmax = std::max(std::max(e->H, e->I), e->qd); A.tok_rows = e->tok.rows;
  A.out_norm = e->out_norm;
  A.eps = e->cfg.rms_eps;
  A.deadzone = e->deadzone;
  A.nt_ref = e->nt_ref;
  A.cos_tab = e->cos_tab;
  A.sin_tab = e->sin_tab;
  A.et = e->et;
  A.hist = e->d_hist;
  A.grid = sms;
  A.tp_rank = 0;
  A.tp_world = 1;
  if (e->hd % 64 || e->hd > 128) return no("head_dim not a multiple of 64 up to 128");
  if (e->I % 64 || e->H % 64 || e->qd % 64) return no("widths not multiples of 64");
  if ((e->I / 8 + sms - 1) / sms > kDecodeSvUnits) return no("gate/up units per CTA above the shared-memory SwiGLU buffer");
  size_t limit = 0;
  if (decode_max_dyn_smem(&limit) != cudaSuccess) return no("kernel attributes");
  // ring slots: as many as shared memory holds (env DPUF_CUDA_RING_SLOTS caps them)
  A.n_slots = std::min(decode_ring_slots(A, limit), std::max(1, env_int("DPUF_CUDA_RING_SLOTS", 1 << 20)));
  if (A.n_slots < 2 * kDecodeConsWarps + 2) return no("shared memory: ring shorter than 24 stages");
  int per_sm = 0;
  if (decode_blocks_per_sm(A, &per_sm) != cudaSuccess || per_sm < 1) return no("occupancy");
  if (cudaMalloc(&e->d_dec_layers, std::max<size_t>(1, tab.size()) * sizeof(DecLayer)) ||
      (!tab.empty() &&
       cudaMemcpy(e->d_dec_layers, tab.data(), tab.size() * sizeof(DecLayer), cudaMemcpyHostToDevice)))
    return no("allocation");
  const DecLayout t = dec_layout(e, 1, sms);
  e->dec_xbytes = t.total;
  const size_t oprep_bytes = (size_t)(e->qd / 64) * 20 * 8;
  if (cudaMalloc(&e->dec_xbuf, t.total) || cudaMemset(e->dec_xbuf, 0, t.total) ||
      cudaMalloc(&e->dec_oprep, oprep_bytes) || cudaMemset(e->dec_oprep, 0, oprep_bytes))
    return no("allocation");
  e->dec_gen = 1;
  dec_bind(A, e->dec_xbuf, t);
  A.oprep = e->dec_oprep;
  A.layers = e->d_dec_layers;
  // every device wait gives up after this long (env DPUF_CUDA_WAIT_MS, default 2000 ms)
  A.wait_ns = (unsigned long long)std::max(1, env_int("DPUF_CUDA_WAIT_MS", 2000)) * 1000000ull;
  A.stall_unit = -1;
  // stages in flight per CTA (env DPUF_CUDA_INFLIGHT): enough to keep HBM busy, few enough that
  // the exchange words between CTAs do not queue behind megabytes of weight requests.  At least
  // one producer round (one stage per consumer warp); the ring must hold a round more.
  A.max_inflight = std::max(kDecodeConsWarps, std::min(A.n_slots - kDecodeConsWarps - 1, env_int("DPUF_CUDA_INFLIGHT", 30)));
  if (env_int("DPUF_CUDA_TRACE_DECODE", 0)) {
    A.trace_per_cta = decode_trace_events(e->L);
    if (cudaMalloc(&A.trace, (size_t)sms * A.trace_per_cta * 8) ||
        cudaMemset(A.trace, 0, (size_t)sms * A.trace_per_cta * 8))
      return no("allocation");
  }
  e->dec_ok = true;
  e->dec_why.clear();
}

bool persistent_step(const Engine* e, const StepParams& P) {
  return P.M == 1 && P.za == 0 && !P.embeds && !P.ds_mask && !P.tok_rope && e->dec_ok && e->use_persistent;
}

// After a launch that gave up a wait, the exchange area holds a partial layer's tags and counts:
// one GPU zeroes it and starts again from generation 1 (under tensor parallelism the ranks
// cannot agree on that here, so their engines stay failed).
cudaError_t dec_recover(Engine* e) {
  if (!e->dec_failed || e->tp_world > 1) return cudaSuccess;
  CK(cudaMemsetAsync(e->dec_xbuf, 0, e->dec_xbytes, e->stream));
  CK(cudaMemsetAsync(e->dec_oprep, 0, (size_t)(e->qd / 64) * 20 * 8, e->stream));
  e->dec_gen = 1;
  e->dec_failed = 0;
  return cudaSuccess;
}

// Launches the persistent kernel for n_steps batch-1 steps from (first_id, pos0) and queues the
// read of its error word into the pinned staging (checked by the caller after synchronising).
cudaError_t run_decode(Engine* e, int first_id, int pos0, int n_steps, bool write_logits, int keep) {
  CK(dec_recover(e));
  DecodeArgs A = e->dec;
  A.first_id = first_id;
  A.pos0 = pos0;
  A.n_steps = n_steps;
  A.write_logits = write_logits ? 1 : 0;
  const int down_tiles = e->L > 0 ? e->layers[0].down.n_tiles : 0;
  A.keep_down = (keep > 0 && keep < down_tiles) ? keep : down_tiles;
  A.kv_k = e->slots[e->active].k;
  A.kv_v = e->slots[e->active].v;
  A.gen0 = e->dec_gen;
  A.stall_unit = e->dec_stall_next;
  e->dec_stall_next = -1;
  e->stage->pad[0] = 0;
  // this GPU's error word (under tensor parallelism it stays set once a rank has failed)
  if (e->tp_world == 1) CK(cudaMemsetAsync(A.err, 0, 4, e->stream));
  CK(launch_decode(e->stream, A));
  e->dec_gen += (unsigned)n_steps * (unsigned)decode_phases(e->L);
  CK(cudaMemcpyAsync(&e->stage->pad[0], A.err, 4, cudaMemcpyDeviceToHost, e->stream));
  return cudaSuccess;
}

// After the stream is synchronised: the persistent kernel's error word.
int32_t decode_status(Engine* e) {
  const int code = e->stage->pad[0];
  if (code == 0) return 0;
  e->dec_failed = 1;
  set_error(code == 1 ? "persistent decode: a weight-stream wait timed out"
                      : "persistent decode: a wait for another CTA's (or rank's) outputs timed out");
  return -6;
}

// Environment knobs read per call, as the reference does (dpuf_engine.c:2022-2027, 2091-2118).
StepParams step_params(const Engine* e, int n, int only_last) {
  StepParams P{};
  P.M = n;
  P.only_last = only_last == 0 ? 0 : (only_last == 2 ? 2 : 1);
  P.keep = 0;
  if (const char* kt = getenv(n > 1 ? "DPUF_PREFILL_KEEP_TILES" : "DPUF_GEN_KEEP_TILES")) {
    const int v = atoi(kt);
    P.keep = (v > 0) ? v : 0;
  }
  const int lm_M = P.only_last == 1 ? 1 : n;
  P.za = 0;
  P.margin = 0.0f;
  P.greedy_loop = false;
  const char* env_t = getenv("DPUF_EARLY_TILES");
  if (env_t && P.only_last != 2 && lm_M == 1 && e->lm.n_tiles > 2048) {
    int za = atoi(env_t);
    za = std::max(za, 256);
    za = std::min(za, e->lm.n_tiles);
    P.za = za;
    const char* env_m = getenv("DPUF_EARLY_MARGIN");
    P.margin = env_m ? (float)atof(env_m) : 1.25f;
  }
  return P;
}


// Validation and environment knobs of dpuf_engine_forward_batch_ex (dpuf_engine.c:1639-1641,
// 2022-2027, 2091-2118), then one step.
int32_t forward_common(Engine* e, int32_t n, const int32_t* ids, int32_t pos0, const float* embeds,
                       const int32_t* pt, const int32_t* ph, const int32_t* pw, const float* const* ds,
                       int32_t only_last, float* logits_out, bool want_logits) {
  if (!e || (!ids && !embeds) || (want_logits && !logits_out && only_last != 2)) return -1;
  if (n <= 0 || n > kMaxBatch) return -2;
  if (pos0 < 0 || pos0 + n > e->S) return -3;
  for (int i = 0; i < n; i++)
    if (ids && (ids[i] >= e->tok.rows || (ids[i] < 0 && !embeds))) {
      set_error("token id out of range");
      return -1;
    }
  if (cudaSetDevice(e->device) != cudaSuccess) return -4;
  StepParams P = step_params(e, n, only_last);
  P.embeds = embeds;
  P.all_embeds = embeds && !ids;
  if (pt || ph || pw) {  // per-token rotation rows (dpuf_engine.c:1679-1696)
    const int half = e->hd / 2;
    e->h_tok_rope.assign((size_t)2 * kMaxBatch * half, 0.0f);
    for (int i = 0; i < n; i++) {
      const int t = pt ? pt[i] : pos0 + i, hh = ph ? ph[i] : pos0 + i, w = pw ? pw[i] : pos0 + i;
      float* cr = &e->h_tok_rope[(size_t)i * half];
      float* sr = &e->h_tok_rope[(size_t)(kMaxBatch + i) * half];
      if (!e->cfg.has_mrope || (t == hh && t == w)) {  // the tables' row at t
        if (t < 0 || t >= e->S) {
          set_error("rotary position outside [0, max_seq_len)");
          return -3;
        }
        memcpy(cr, &e->h_cos[(size_t)t * half], (size_t)half * 4);
        memcpy(sr, &e->h_sin[(size_t)t * half], (size_t)half * 4);
      } else {  // eng_compute_mrope_cos_sin (dpuf_engine.c:1602-1623), the same libm
        const int sec_h = e->cfg.mrope_section[1], len_hw = 3 * sec_h;
        for (int j = 0; j < half; j++) {
          const float freq = 1.0f / powf(e->cfg.rope_theta, (2.0f * (float)j) / (float)e->hd);
          float pv = (float)t;
          if (j < len_hw) pv = (j % 3 == 1) ? (float)hh : ((j % 3 == 2) ? (float)w : (float)t);
          const float ang = pv * freq;
          cr[j] = cosf(ang);
          sr[j] = sinf(ang);
        }
      }
    }
    if (!e->d_tok_rope && cudaMalloc(&e->d_tok_rope, e->h_tok_rope.size() * 4) != cudaSuccess) {
      e->d_tok_rope = nullptr;
      set_error("cudaMalloc (rotary rows)");
      return -4;
    }
    if (cudaMemcpyAsync(e->d_tok_rope, e->h_tok_rope.data(), e->h_tok_rope.size() * 4, cudaMemcpyHostToDevice,
                        e->stream) != cudaSuccess)
      return -4;
    P.tok_rope = true;
  }
  if (ds) {  // DeepStack rows of layers 0..2, [n][H] each (null: none for that layer)
    if (!e->d_ds && cudaMalloc(&e->d_ds, (size_t)3 * kMaxBatch * e->H * 4) != cudaSuccess) {
      e->d_ds = nullptr;
      set_error("cudaMalloc (DeepStack rows)");
      return -4;
    }
    for (int l = 0; l < 3 && l < e->L; l++)
      if (ds[l]) {
        if (cudaMemcpyAsync(e->d_ds + (size_t)l * kMaxBatch * e->H, ds[l], (size_t)n * e->H * 4,
                            cudaMemcpyHostToDevice, e->stream) != cudaSuccess)
          return -4;
        P.ds_mask |= 1 << l;
      }
  }
  const int lm_M = P.only_last == 1 ? 1 : n;
  for (int i = 0; i < n; i++) {  // ids < 0 mark rows taken from embeds_in
    e->stage_neg[i] = ids && ids[i] < 0;
    e->stage->ids[i] = (!ids || ids[i] < 0) ? 0 : ids[i];
  }
  e->stage->pos0 = pos0;
  const bool persistent = persistent_step(e, P);
  cudaError_t err = persistent ? run_decode(e, ids[0], pos0, 1, P.only_last != 2, P.keep) : run_step(e, P);
  if ((embeds || ds || P.tok_rope) && err == cudaSuccess && cudaStreamSynchronize(e->stream) != cudaSuccess) err = cudaErrorUnknown;
  if (err != cudaSuccess) return -4;
  e->last_zone_used = P.za > 0;
  e->last_rows = P.only_last == 2 ? 0 : lm_M;
  e->last_logits = persistent ? e->dec.logits : e->logits;
  if (P.only_last != 2 && want_logits) {
    const size_t bytes = (size_t)lm_M * e->V * 4;
    if (lm_M == 1) {
      if (cudaMemcpyAsync(e->h_logits, e->last_logits, bytes, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
        return -4;
      if (!sync_ok(e)) return -4;
      memcpy(logits_out, e->h_logits, bytes);
    } else {
      if (cudaMemcpyAsync(logits_out, e->logits, bytes, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess) return -4;
      if (!sync_ok(e)) return -4;
    }
  } else {
    if (!sync_ok(e)) return -4;
  }
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) {
    set_error(cudaGetErrorString(le));
    return -4;
  }
  if (!persistent && ((n > 1 && e->use_tc_gemm) || e->has_had)) {
    int tc_err = 0;
    if (cudaMemcpy(&tc_err, e->d_tc_err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -4;
    if (tc_err) {
      set_error("a matmul kernel's bounded wait gave up (tensor-core GEMM or mode-13/14 GEMV)");
      return -6;
    }
  }
  return persistent ? decode_status(e) : 0;
}

Engine* create_engine(const DpufModelConfig* cfg, const DpufLayerWeights* layers, const DpufWeightDesc* tok,
                      const DpufWeightDesc* lm, const float* out_norm) {
  if (!cfg || !layers || !tok || !lm || !out_norm) return nullptr;
  const DpufModelConfig& c = *cfg;
  if (c.hidden_size <= 0 || c.num_layers < 0 || c.num_q_heads <= 0 || c.num_kv_heads <= 0 ||
      c.num_q_heads % c.num_kv_heads != 0 || c.head_dim <= 0 || c.head_dim % 32 != 0 || c.head_dim > 256 ||
      c.max_seq_len <= 0 || (c.kv_type != DPUF_KV_F32 && c.kv_type != DPUF_KV_Q8) || c.hidden_size % 64 != 0 || c.intermediate_size % 64 != 0 ||
      (c.num_q_heads * c.head_dim) % 64 != 0) {
    set_error("unsupported model configuration");
    return nullptr;
  }
  const int H = c.hidden_size, I = c.intermediate_size, qd = c.num_q_heads * c.head_dim,
            kvd = c.num_kv_heads * c.head_dim;
  for (int l = 0; l < c.num_layers; l++) {
    const DpufLayerWeights& w = layers[l];
    if (!desc_ok(w.w_q, qd, H) || !desc_ok(w.w_k, kvd, H) || !desc_ok(w.w_v, kvd, H) || !desc_ok(w.w_o, H, qd) ||
        !desc_ok(w.w_gate, I, H) || !desc_ok(w.w_up, I, H) || !desc_ok(w.w_down, H, I) || !w.attn_norm ||
        !w.ffn_norm) {
      set_error("layer " + std::to_string(l) + ": weights must be mode 12, 13 or 14 with matching shapes");
      return nullptr;
    }
  }
  if (!desc_ok(*tok, tok->rows, H) || !desc_ok(*lm, c.vocab_size, H)) {
    set_error("embedding / LM head must be mode 12, 13 or 14 with cols == hidden_size");
    return nullptr;
  }
  Engine* e = new Engine();
  e->cfg = c;
  if (cudaGetDevice(&e->device) != cudaSuccess) { delete e; return nullptr; }
  if (const char* d = getenv("DPUF_CUDA_DEVICE")) {
    e->device = atoi(d);
    if (cudaSetDevice(e->device) != cudaSuccess) { delete e; return nullptr; }
  }
  e->H = H; e->I = I; e->L = c.num_layers; e->nq = c.num_q_heads; e->nkv = c.num_kv_heads; e->hd = c.head_dim;
  e->qd = qd; e->kvd = kvd; e->V = c.vocab_size; e->S = c.max_seq_len;
  e->act_ld = std::max(std::max(H, I), qd);
  const char* dz = getenv("DPUF_SWIGLU_DEADZONE");
  e->deadzone = dz ? (float)atof(dz) : 0.005f;
  e->nt_ref = c.n_threads <= 0 ? 8 : std::min(c.n_threads, 32);
  e->n_slots = std::max(1, std::min(kMaxSlotsEnv, env_int("DPUF_CUDA_SLOTS", kMaxSlots)));
  e->slots.resize(e->n_slots);
  e->use_pdl = env_int("DPUF_CUDA_PDL", 1) != 0;
  e->use_graphs = env_int("DPUF_CUDA_GRAPHS", 1) != 0;

  auto fail = [&](const char* what) -> Engine* {
    if (g_err.empty()) set_error(what);
    destroy_engine(e);
    return nullptr;
  };
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");
  if (cudaError_t ce = configure_kernels()) {
    set_error(std::string("kernel attributes: ") + cudaGetErrorString(ce));
    return fail("kernel attributes");
  }

  // ---- weights
  ArenaPlan P;
  for (int l = 0; l < c.num_layers; l++) {
    const DpufLayerWeights& w = layers[l];
    for (const DpufWeightDesc* d : {&w.w_q, &w.w_k, &w.w_v, &w.w_o, &w.w_gate, &w.w_up, &w.w_down}) plan_w(P, *d);
    plan_f(P, w.attn_norm, H);
    plan_f(P, w.ffn_norm, H);
    plan_f(P, w.attn_q_norm, c.head_dim);
    plan_f(P, w.attn_k_norm, c.head_dim);
  }
  plan_w(P, *tok);
  plan_w(P, *lm);
  plan_f(P, out_norm, H);
  if (cudaMalloc(&e->arena, P.bytes) != cudaSuccess) return fail("weight arena allocation");
  std::set<size_t> done;
  e->layers.resize(c.num_layers);
  for (int l = 0; l < c.num_layers; l++) {
    const DpufLayerWeights& w = layers[l];
    LayerDev& d = e->layers[l];
    if (upload_w(e, P, w.w_q, &d.q, done) || upload_w(e, P, w.w_k, &d.k, done) || upload_w(e, P, w.w_v, &d.v, done) ||
        upload_w(e, P, w.w_o, &d.o, done) || upload_w(e, P, w.w_gate, &d.gate, done) ||
        upload_w(e, P, w.w_up, &d.up, done) || upload_w(e, P, w.w_down, &d.down, done))
      return fail("weight upload");
    d.attn_norm = upload_f(e, P, w.attn_norm, H);
    d.ffn_norm = upload_f(e, P, w.ffn_norm, H);
    d.q_norm = upload_f(e, P, w.attn_q_norm, c.head_dim);
    d.k_norm = upload_f(e, P, w.attn_k_norm, c.head_dim);
    if (!d.attn_norm || !d.ffn_norm) return fail("norm upload");
  }
  if (upload_w(e, P, *tok, &e->tok, done) || upload_w(e, P, *lm, &e->lm, done)) return fail("embedding upload");
  e->out_norm = upload_f(e, P, out_norm, H);
  if (!e->out_norm) return fail("norm upload");

  // ---- RoPE tables
  {
    std::vector<float> cs, sn;
    rope_tables(c, cs, sn);
    e->h_cos = cs;
    e->h_sin = sn;
    if (cudaMalloc(&e->cos_tab, cs.size() * 4) || cudaMalloc(&e->sin_tab, sn.size() * 4) ||
        cudaMemcpy(e->cos_tab, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) ||
        cudaMemcpy(e->sin_tab, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice))
      return fail("rope tables");
  }
  // ---- expf exception table
  {
    std::vector<uint2> slots;
    uint32_t mask = 0;
    int max_probe = 0;
    expf_exception_hash(slots, &mask, &max_probe);
    if (cudaMalloc(&e->d_exp_slots, slots.size() * sizeof(uint2)) ||
        cudaMemcpy(e->d_exp_slots, slots.data(), slots.size() * sizeof(uint2), cudaMemcpyHostToDevice))
      return fail("expf table");
    e->et = ExpfTable{e->d_exp_slots, mask, max_probe};
  }
  // ---- activations
  const size_t B = kMaxBatch;
  const int ld = e->act_ld;
  if (cudaMalloc(&e->h, B * H * 4) || cudaMalloc(&e->hn, B * H * 4) || cudaMalloc(&e->q, B * qd * 4) ||
      cudaMalloc(&e->k, B * kvd * 4) || cudaMalloc(&e->v, B * kvd * 4) ||
      cudaMalloc(&e->att, B * std::max(qd, H) * 4) || cudaMalloc(&e->gate, B * I * 4) ||
      cudaMalloc(&e->up, B * I * 4) || cudaMalloc(&e->logits, B * (size_t)e->V * 4) ||
      cudaMalloc(&e->prep_q8, 3 * B * ld) || cudaMalloc(&e->prep_xs, 3 * B * (ld / 32) * 4) ||
      cudaMalloc(&e->prep_xm, 3 * B * (ld / 32) * 4) || cudaMalloc(&e->d_ids, sizeof(Staging)) ||
      cudaMalloc(&e->d_flag, 16) || cudaMalloc(&e->d_b12, 16) || cudaMalloc(&e->d_argmax, B * 4) ||
      cudaMalloc(&e->d_hist, (size_t)(e->S + 4) * 4) || cudaMalloc(&e->d_counter, 64) ||
      cudaMalloc(&e->d_part, kArgmaxBlocks * sizeof(float2)) ||
      cudaMallocHost(&e->stage, sizeof(Staging)) || cudaMallocHost(&e->bstage, sizeof(BatchStaging)) ||
      cudaMalloc(&e->d_bstage, sizeof(BatchStaging)) || cudaMalloc(&e->d_next, kMaxBatch * 4) || cudaMallocHost(&e->h_logits, (size_t)e->V * 4))
    return fail("activation buffers");
  if (cudaMalloc(&e->split.pairs, gemv_split_pairs_bytes(ld)) ||
      cudaMalloc(&e->split.acc, (size_t)kGemvMaxCtas * kTileRows * sizeof(float)) ||
      cudaMalloc(&e->split.count, (size_t)kGemvMaxCtas * sizeof(unsigned)) ||
      cudaMemset(e->split.count, 0, (size_t)kGemvMaxCtas * sizeof(unsigned)))
    return fail("GEMV scratch");
  if (cudaMalloc(&e->d_tc_err, 16) || cudaMemset(e->d_tc_err, 0, 16)) return fail("GEMM error word");
  e->use_tc_gemm = env_int("DPUF_CUDA_TC_GEMM", 1) != 0;
  e->d_pos0 = e->d_ids + kMaxBatch;
  e->d_hist_step = e->d_hist + e->S;
  for (int i = 0; i < 3; i++)
    e->prep[i] = Act{e->prep_q8 + i * B * ld, e->prep_xs + i * B * (ld / 32), e->prep_xm + i * B * (ld / 32), ld};
  cudaMemset(e->d_flag, 0, 16);
  cudaMemset(e->d_counter, 0, 64);
  e->kv_kind = c.kv_type == DPUF_KV_Q8 ? kKvQ8 : env_int("DPUF_CUDA_KV_F16", 0) ? kKvF16 : kKvF32;
  e->kv_row = kv_row_bytes(e->kv_kind, e->hd);
  if (slot_alloc(e, 0) != cudaSuccess) return fail("KV slot 0");
  e->use_persistent = env_int("DPUF_CUDA_PERSISTENT", 1) != 0;
  if (build_expanded(e) != cudaSuccess) return fail("expanded weights");
  plan_decode(e, layers, tok, lm);
  return e;
}

}  // namespace
// ------------------------------------------------------------------ tensor parallelism
// What one rank publishes (DPUF_CUDA_TP_BLOB_BYTES): its IPC handle and what the other ranks
// check before mapping it - same rank order, world, grid and model shape, and a GPU of its own
// (ranks whose kernels wait on each other must never share a GPU: nothing guarantees that two
// launches on one GPU run at the same time).
struct TpBlob {
  char magic[8];
  int32_t rank, world, grid, L, H, I, V, qd, kvd, S;
  uint64_t bytes;
  char pci[32];  // PCI bus id of the rank's GPU
  cudaIpcMemHandle_t handle;
};
static_assert(sizeof(TpBlob) <= DPUF_CUDA_TP_BLOB_BYTES, "tensor-parallel blob size");
constexpr char kTpMagic[8] = {'D', 'P', 'U', 'F', 'T', 'P', '1', 0};

}  // namespace dpuf

using dpuf::Engine;

// ==================================================================== C ABI
extern "C" {

DPUF_EXPORT const char* dpuf_cuda_last_error(void) { return dpuf::g_err.c_str(); }

DPUF_EXPORT void* dpuf_engine_create(const DpufModelConfig* cfg, const DpufLayerWeights* layers,
                                     const DpufWeightDesc* w_tok_embd, const DpufWeightDesc* w_lm_head,
                                     const float* output_norm) {
  dpuf::g_err.clear();
  return dpuf::create_engine(cfg, layers, w_tok_embd, w_lm_head, output_norm);
}

DPUF_EXPORT void dpuf_engine_destroy(void* handle) { dpuf::destroy_engine((Engine*)handle); }

DPUF_EXPORT int32_t dpuf_engine_set_slot(void* handle, int32_t slot_id) {
  Engine* e = (Engine*)handle;
  if (!e || slot_id < 0 || slot_id >= e->n_slots) return -1;
  cudaSetDevice(e->device);
  if (dpuf::slot_alloc(e, slot_id) != cudaSuccess) return -2;
  e->active = slot_id;
  return 0;
}

DPUF_EXPORT int32_t dpuf_engine_get_slot(void* handle) { return handle ? ((Engine*)handle)->active : 0; }

DPUF_EXPORT int32_t dpuf_engine_num_slots(void* handle) { return handle ? ((Engine*)handle)->n_slots : 1; }

DPUF_EXPORT void dpuf_engine_reset_slot(void* handle, int32_t slot_id) {
  Engine* e = (Engine*)handle;
  if (!e || slot_id < 0 || slot_id >= e->n_slots || !e->slots[slot_id].k) return;
  cudaSetDevice(e->device);
  const size_t n = (size_t)e->L * e->S * e->nkv * e->kv_row;
  cudaMemsetAsync(e->slots[slot_id].k, 0, n, e->stream);
  cudaMemsetAsync(e->slots[slot_id].v, 0, n, e->stream);
  cudaStreamSynchronize(e->stream);
}

DPUF_EXPORT void dpuf_engine_reset_cache(void* handle) {
  Engine* e = (Engine*)handle;
  if (e) dpuf_engine_reset_slot(handle, e->active);
}

DPUF_EXPORT size_t dpuf_engine_slot_memory(void* handle) {
  Engine* e = (Engine*)handle;
  return e ? 2 * (size_t)e->L * e->S * e->nkv * e->kv_row : 0;
}

// Freeze / apply copy [L][n_kv][len][hd] between the active slot and a prefix store with one
// strided device copy (dpuf_engine.c:1509-1594).
DPUF_EXPORT int32_t dpuf_engine_freeze_prefix(void* handle, int32_t pfx_id, int32_t prefix_len) {
  Engine* e = (Engine*)handle;
  if (!e || pfx_id < 0 || pfx_id >= dpuf::kMaxPrefixes || prefix_len <= 0 || prefix_len > e->S) return 0;
  cudaSetDevice(e->device);
  dpuf::Prefix& p = e->prefixes[pfx_id];
  const size_t rows = (size_t)e->L * e->nkv;
  if (p.cap < prefix_len || !p.k) {
    cudaFree(p.k);
    cudaFree(p.v);
    p = dpuf::Prefix();
    if (cudaMalloc(&p.k, rows * prefix_len * e->kv_row) != cudaSuccess) { p.k = nullptr; return 0; }
    if (cudaMalloc(&p.v, rows * prefix_len * e->kv_row) != cudaSuccess) { cudaFree(p.k); p.k = nullptr; p.v = nullptr; return 0; }
    p.cap = prefix_len;
  }
  const dpuf::Slot& s = e->slots[e->active];
  if (!s.k) return 0;
  const size_t w = (size_t)prefix_len * e->kv_row;
  if (cudaMemcpy2DAsync(p.k, w, s.k, (size_t)e->S * e->kv_row, w, rows, cudaMemcpyDeviceToDevice, e->stream) ||
      cudaMemcpy2DAsync(p.v, w, s.v, (size_t)e->S * e->kv_row, w, rows, cudaMemcpyDeviceToDevice, e->stream) ||
      cudaStreamSynchronize(e->stream))
    return 0;
  p.len = prefix_len;
  p.valid = true;
  return 1;
}

DPUF_EXPORT int32_t dpuf_engine_apply_prefix(void* handle, int32_t slot_id, int32_t pfx_id) {
  Engine* e = (Engine*)handle;
  if (!e || slot_id < 0 || slot_id >= e->n_slots || pfx_id < 0 || pfx_id >= dpuf::kMaxPrefixes) return 0;
  dpuf::Prefix& p = e->prefixes[pfx_id];
  if (!p.valid || p.len <= 0) return 0;
  cudaSetDevice(e->device);
  if (dpuf::slot_alloc(e, slot_id) != cudaSuccess) return 0;
  const dpuf::Slot& s = e->slots[slot_id];
  const size_t rows = (size_t)e->L * e->nkv, w = (size_t)p.len * e->kv_row;
  if (cudaMemcpy2DAsync(s.k, (size_t)e->S * e->kv_row, p.k, w, w, rows, cudaMemcpyDeviceToDevice, e->stream) ||
      cudaMemcpy2DAsync(s.v, (size_t)e->S * e->kv_row, p.v, w, w, rows, cudaMemcpyDeviceToDevice, e->stream) ||
      cudaStreamSynchronize(e->stream))
    return 0;
  return p.len;
}

DPUF_EXPORT int32_t dpuf_engine_get_prefix_len(void* handle, int32_t pfx_id) {
  Engine* e = (Engine*)handle;
  if (!e || pfx_id < 0 || pfx_id >= dpuf::kMaxPrefixes) return 0;
  return e->prefixes[pfx_id].valid ? e->prefixes[pfx_id].len : 0;
}

DPUF_EXPORT int32_t dpuf_engine_forward_batch_ex(void* handle, int32_t n_tokens, const int32_t* token_ids,
                                                 int32_t pos0, const float* embeds_in, const int32_t* pos_t,
                                                 const int32_t* pos_h, const int32_t* pos_w,
                                                 const float* const* deepstack_in, int32_t only_last_logits,
                                                 float* logits_out) {
  return dpuf::forward_common((Engine*)handle, n_tokens, token_ids, pos0, embeds_in, pos_t, pos_h, pos_w,
                              deepstack_in, only_last_logits, logits_out, true);
}

DPUF_EXPORT int32_t dpuf_engine_forward_batch(void* handle, int32_t n_tokens, const int32_t* token_ids, int32_t pos0,
                                              int32_t only_last_logits, float* logits_out) {
  return dpuf::forward_common((Engine*)handle, n_tokens, token_ids, pos0, nullptr, nullptr, nullptr, nullptr,
                              nullptr, only_last_logits, logits_out, true);
}

DPUF_EXPORT int32_t dpuf_engine_forward_token(void* handle, int32_t token_id, int32_t pos, float* logits_out) {
  const int32_t id = token_id;
  return dpuf_engine_forward_batch(handle, 1, &id, pos, 1, logits_out);
}

DPUF_EXPORT int32_t dpuf_cuda_forward_greedy(void* handle, int32_t n_tokens, const int32_t* token_ids, int32_t pos0,
                                             int32_t* next_id) {
  Engine* e = (Engine*)handle;
  if (!e || !next_id) return -1;
  const int32_t rc = dpuf::forward_common(e, n_tokens, token_ids, pos0, nullptr, nullptr, nullptr, nullptr, nullptr,
                                          1, nullptr, false);
  if (rc != 0) return rc;
  const dpuf::Launch Lc{e->stream, false};
  if (dpuf::launch_argmax(Lc, e->logits, e->V, e->d_part, e->d_counter + 1, e->d_argmax) != cudaSuccess ||
      cudaMemcpyAsync(next_id, e->d_argmax, 4, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess ||
      cudaStreamSynchronize(e->stream) != cudaSuccess)
    return -4;
  return 0;
}

// n_steps greedy decode steps at batch 1 with the token fed back on the device.  The step
// kernels are the same as dpuf_engine_forward_token's; only the id hand-off differs.
DPUF_EXPORT int32_t dpuf_cuda_decode_greedy(void* handle, int32_t first_id, int32_t pos0, int32_t n_steps,
                                            int32_t* ids_out, float* device_ms) {
  Engine* e = (Engine*)handle;
  if (!e || !ids_out) return -1;
  if (n_steps <= 0) return -2;
  if (pos0 < 0 || pos0 + n_steps > e->S) return -3;
  if (first_id < 0 || first_id >= e->tok.rows) return -1;
  if (cudaSetDevice(e->device) != cudaSuccess) return -4;
  dpuf::StepParams P = dpuf::step_params(e, 1, 1);
  P.greedy_loop = true;
  e->stage->ids[0] = first_id;
  e->stage->pos0 = pos0;
  const int32_t zero = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  if (cudaMemcpyAsync(e->d_ids, e->stage, sizeof(dpuf::Staging), cudaMemcpyHostToDevice, e->stream) ||
      cudaMemcpyAsync(e->d_hist_step, &zero, 4, cudaMemcpyHostToDevice, e->stream) ||
      cudaStreamSynchronize(e->stream) || cudaEventCreate(&ev0) || cudaEventCreate(&ev1))
    return -4;
  const bool persistent = dpuf::persistent_step(e, P);
  cudaEventRecord(ev0, e->stream);
  if (persistent) {
    if (dpuf::run_decode(e, first_id, pos0, n_steps, true, P.keep) != cudaSuccess) {
      cudaEventDestroy(ev0);
      cudaEventDestroy(ev1);
      return -4;
    }
  } else {
    for (int i = 0; i < n_steps; i++)
      if (dpuf::run_step(e, P) != cudaSuccess) { cudaEventDestroy(ev0); cudaEventDestroy(ev1); return -4; }
  }
  cudaEventRecord(ev1, e->stream);
  int32_t rc = 0;
  if (cudaMemcpyAsync(ids_out, e->d_hist, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, e->stream) ||
      cudaStreamSynchronize(e->stream))
    rc = -4;
  float ms = 0.0f;
  if (rc == 0 && cudaEventElapsedTime(&ms, ev0, ev1) != cudaSuccess) rc = -4;
  if (rc == 0 && persistent) rc = dpuf::decode_status(e);
  if (device_ms) *device_ms = ms;
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  e->last_rows = 1;
  e->last_zone_used = 0;
  e->last_logits = persistent ? e->dec.logits : e->logits;
  return rc;
}

// One greedy step of n independent sequences (batched serving): row i is sequence slots[i] at
// position pos[i] with input ids[i].  Every row is computed as that sequence's own batch-1 step
// (same kernels as an M-row step, with the reference's per-step vector/scalar SwiGLU split of
// one row), so each row's logits and id equal dpuf_engine_forward_token's on that slot.
DPUF_EXPORT int32_t dpuf_cuda_decode_batch(void* handle, int32_t n, const int32_t* slots, const int32_t* ids,
                                           const int32_t* pos, int32_t* next_ids, float* logits_out) {
  Engine* e = (Engine*)handle;
  if (!e || !slots || !ids || !pos || !next_ids) return -1;
  if (n <= 0 || n > dpuf::kMaxBatch) return -2;
  std::vector<char> seen(e->n_slots, 0);
  for (int i = 0; i < n; i++) {
    if (slots[i] < 0 || slots[i] >= e->n_slots || seen[slots[i]]) {
      dpuf::set_error("decode_batch: slot ids must be valid and distinct");
      return -1;
    }
    seen[slots[i]] = 1;
    if (ids[i] < 0 || ids[i] >= e->tok.rows) {
      dpuf::set_error("token id out of range");
      return -1;
    }
    if (pos[i] < 0 || pos[i] >= e->S) return -3;
  }
  if (cudaSetDevice(e->device) != cudaSuccess) return -4;
  for (int i = 0; i < n; i++) {
    if (dpuf::slot_alloc(e, slots[i]) != cudaSuccess) return -2;
    e->stage->ids[i] = ids[i];
    e->bstage->pos[i] = pos[i];
    e->bstage->k[i] = e->slots[slots[i]].k;
    e->bstage->v[i] = e->slots[slots[i]].v;
  }
  // each row is a batch-1 step: the decode knob DPUF_GEN_KEEP_TILES, no Zone A (the reference
  // tests lm_M == 1 per call; a batched call has lm_M == n)
  dpuf::StepParams P = dpuf::step_params(e, 1, 1);
  P.M = n;
  P.only_last = 0;
  P.za = 0;
  P.batch = true;
  if (dpuf::run_step(e, P) != cudaSuccess) return -4;
  if (cudaMemcpyAsync(next_ids, e->d_next, (size_t)n * 4, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
    return -4;
  if (logits_out &&
      cudaMemcpyAsync(logits_out, e->logits, (size_t)n * e->V * 4, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
    return -4;
  if (!sync_ok(e)) return -4;
  e->last_rows = n;
  e->last_zone_used = 0;
  e->last_logits = e->logits;
  return 0;
}

DPUF_EXPORT int32_t dpuf_cuda_read_logits(void* handle, int32_t row, float* out) {
  Engine* e = (Engine*)handle;
  if (!e || !out || row < 0 || row >= e->last_rows) return -1;
  cudaSetDevice(e->device);
  const float* src = e->last_logits ? e->last_logits : e->logits;
  if (cudaMemcpy(out, src + (size_t)row * e->V, (size_t)e->V * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -4;
  return 0;
}

DPUF_EXPORT int32_t dpuf_cuda_set_option(void* handle, const char* name, int64_t value) {
  Engine* e = (Engine*)handle;
  if (!e || !name) return -1;
  if (!strcmp(name, "pdl")) { e->use_pdl = value != 0; dpuf::drop_graphs(e); return 0; }
  if (!strcmp(name, "graphs")) { e->use_graphs = value != 0; dpuf::drop_graphs(e); return 0; }
  if (!strcmp(name, "persistent")) { e->use_persistent = value != 0; return 0; }
  if (!strcmp(name, "tc_gemm")) { e->use_tc_gemm = value != 0; dpuf::drop_graphs(e); return 0; }
  if (!strcmp(name, "wait_ms")) {
    if (value <= 0) return -1;
    e->dec.wait_ns = (unsigned long long)value * 1000000ull;
    return 0;
  }
  if (!strcmp(name, "test_stall_unit")) {
    // failure-detection test hook: in the next persistent launch, the CTA that computes q/k/v
    // unit `value` (8 rows of layer 0, q rows first) withholds its outputs of the first step,
    // so every wait on them runs into the wait limit
    if (value < 0 || value >= (int64_t)(e->dec.qd + 2 * e->dec.kvd) / 8) return -1;
    e->dec_stall_next = (int)value;
    return 0;
  }
  return -1;
}

DPUF_EXPORT int32_t dpuf_cuda_decode_trace(void* handle, int32_t* n_ctas, int32_t* per_cta, uint64_t* out,
                                           int64_t max_values) {
  Engine* e = (Engine*)handle;
  if (!e || !e->dec.trace) return -1;
  if (n_ctas) *n_ctas = e->dec.grid;
  if (per_cta) *per_cta = e->dec.trace_per_cta;
  const int64_t n = (int64_t)e->dec.grid * e->dec.trace_per_cta;
  if (!out) return 0;
  if (max_values < n) return -2;
  cudaSetDevice(e->device);
  return cudaMemcpy(out, e->dec.trace, (size_t)n * 8, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -4;
}

DPUF_EXPORT int32_t dpuf_cuda_persistent_decode(void* handle, const char** why) {
  Engine* e = (Engine*)handle;
  if (!e) return -1;
  if (why) *why = e->dec_ok ? "" : e->dec_why.c_str();
  return e->dec_ok && e->use_persistent ? 1 : 0;
}

DPUF_EXPORT int32_t dpuf_cuda_tp_handle(void* handle, int32_t rank, int32_t world, uint8_t* blob_out) {
  Engine* e = (Engine*)handle;
  if (!e || !blob_out || world < 2 || world > dpuf::kMaxTp || rank < 0 || rank >= world) return -1;
  if (e->tp_world > 1 || e->tp_buf) {
    dpuf::set_error("tensor parallelism is already set up on this engine");
    return -1;
  }
  if (!e->dec_ok) {
    dpuf::set_error("tensor parallelism needs the persistent decode kernel: " + e->dec_why);
    return -5;
  }
  // every rank must own units of the q/k/v, o and gate/up projections (see take_range)
  if ((e->qd + 2 * e->kvd) / 16 < world || e->H / 16 < world || e->I / 16 < world) {
    dpuf::set_error("tensor parallelism: the model has fewer 16-row tiles per projection than ranks");
    return -1;
  }
  if (cudaSetDevice(e->device) != cudaSuccess) return -4;
  const dpuf::DecLayout t = dpuf::dec_layout(e, world, e->dec.grid);
  dpuf::TpBlob b{};
  if (cudaDeviceGetPCIBusId(b.pci, (int)sizeof(b.pci) - 1, e->device) != cudaSuccess) return -4;
  if (cudaMalloc(&e->tp_buf, t.total) != cudaSuccess || cudaMemset(e->tp_buf, 0, t.total) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&b.handle, e->tp_buf) != cudaSuccess) {
    cudaFree(e->tp_buf);
    e->tp_buf = nullptr;
    dpuf::set_error("tensor parallelism: exchange buffer allocation or export failed");
    return -4;
  }
  e->tp_bytes = t.total;
  e->tp_rank = rank;
  e->tp_pending = world;
  memcpy(b.magic, dpuf::kTpMagic, 8);
  b.rank = rank; b.world = world; b.grid = e->dec.grid; b.L = e->L; b.H = e->H; b.I = e->I; b.V = e->V;
  b.qd = e->qd; b.kvd = e->kvd; b.S = e->S; b.bytes = t.total;
  memset(blob_out, 0, DPUF_CUDA_TP_BLOB_BYTES);
  memcpy(blob_out, &b, sizeof(b));
  return 0;
}

DPUF_EXPORT int32_t dpuf_cuda_tp_attach(void* handle, const uint8_t* blobs) {
  Engine* e = (Engine*)handle;
  if (!e || !blobs) return -1;
  if (!e->tp_buf || e->tp_world > 1) {
    dpuf::set_error("tensor parallelism: call dpuf_cuda_tp_handle once before dpuf_cuda_tp_attach");
    return -1;
  }
  const int world = e->tp_pending;
  for (int r = 0; r < world; r++) {
    dpuf::TpBlob b;
    memcpy(&b, blobs + (size_t)r * DPUF_CUDA_TP_BLOB_BYTES, sizeof(b));
    if (memcmp(b.magic, dpuf::kTpMagic, 8) || b.rank != r || b.world != world || b.grid != e->dec.grid ||
        b.L != e->L || b.H != e->H || b.I != e->I || b.V != e->V || b.qd != e->qd || b.kvd != e->kvd ||
        b.S != e->S || b.bytes != e->tp_bytes) {
      dpuf::set_error("tensor parallelism: rank " + std::to_string(r) +
                      " published a different model, grid or rank order");
      return -1;
    }
    for (int r2 = 0; r2 < r; r2++) {
      dpuf::TpBlob b2;
      memcpy(&b2, blobs + (size_t)r2 * DPUF_CUDA_TP_BLOB_BYTES, sizeof(b2));
      if (!strncmp(b.pci, b2.pci, sizeof(b.pci))) {
        dpuf::set_error("tensor parallelism: ranks " + std::to_string(r2) + " and " + std::to_string(r) +
                        " are on the same GPU; every rank needs its own");
        return -1;
      }
    }
  }
  if (cudaSetDevice(e->device) != cudaSuccess) return -4;
  void* peer[dpuf::kMaxTp] = {};
  for (int r = 0; r < world; r++) {
    if (r == e->tp_rank) continue;
    dpuf::TpBlob b;
    memcpy(&b, blobs + (size_t)r * DPUF_CUDA_TP_BLOB_BYTES, sizeof(b));
    if (cudaIpcOpenMemHandle(&peer[r], b.handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      for (void* p : peer)
        if (p) cudaIpcCloseMemHandle(p);
      cudaGetLastError();
      dpuf::set_error("tensor parallelism: cannot map rank " + std::to_string(r) + "'s exchange buffer");
      return -4;
    }
  }
  const dpuf::DecLayout t = dpuf::dec_layout(e, world, e->dec.grid);
  dpuf::DecodeArgs& A = e->dec;
  unsigned char* base = e->tp_buf;
  for (int r = 0; r < world; r++) {
    e->tp_peer[r] = peer[r];
    A.tp_delta[r] = r == e->tp_rank ? 0 : (long long)((unsigned char*)peer[r] - base);
  }
  A.tp_rank = e->tp_rank;
  A.tp_world = world;
  dpuf::dec_bind(A, base, t);
  e->tp_world = world;
  e->dec_gen = 1;  // every rank starts at the same generation over zeroed buffers and counters
  return 0;
}

DPUF_EXPORT int32_t dpuf_cuda_zone_info(void* handle, int32_t* used, int32_t* exited, float* b1, float* b2) {
  Engine* e = (Engine*)handle;
  if (!e) return -1;
  int flag = 0;
  float b[2] = {0, 0};
  cudaSetDevice(e->device);
  if (cudaMemcpy(&flag, e->d_flag, 4, cudaMemcpyDeviceToHost) || cudaMemcpy(b, e->d_b12, 8, cudaMemcpyDeviceToHost))
    return -4;
  if (used) *used = e->last_zone_used;
  if (exited) *exited = e->last_zone_used ? flag : 0;
  if (b1) *b1 = b[0];
  if (b2) *b2 = b[1];
  return 0;
}

}  // extern "C"
