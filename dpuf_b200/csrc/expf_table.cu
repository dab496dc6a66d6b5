// expf_table.cu - exception table that makes the GPU's expf bit-identical to the host glibc.
//
// The reference evaluates some exponentials with libm expf (the softmax tail,
// dpuf_engine.c:406-409, and the scalar SwiGLU tail, :990-996).  The device evaluates
// dpuf_exp_d (common.cuh, identical bits on host and device) rounded to float; the table lists
// every finite input in [-160, 100] where that differs from this machine's expf, with expf's
// result.  It is built once per process from the host libm (multi-threaded scan of ~2.3e9
// inputs) and cached next to the library; a cached file is accepted only after spot checks
// against the running libm.
#include <dlfcn.h>
#include <unistd.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "engine_internal.h"

namespace dpuf {

namespace {

uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

bool differs(uint32_t bits, uint32_t* glibc_out) {
  const float x = u2f(bits);
  const float a = expf(x);
  const float b = (float)dpuf_exp_d((double)x);
  if (f2u(a) == f2u(b)) return false;
  *glibc_out = f2u(a);
  return true;
}

// Bit-pattern ranges scanned: [+0, 100.0] and [-0, -160.0].
constexpr uint32_t kPosEnd = 0x42C80000u;  // 100.0f
constexpr uint32_t kNegBeg = 0x80000000u;
constexpr uint32_t kNegEnd = 0xC3200000u;  // -160.0f

void scan(std::vector<uint32_t>& keys, std::vector<uint32_t>& vals) {
  unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  nt = std::min(nt, 128u);
  const uint64_t n_pos = (uint64_t)kPosEnd + 1, n_neg = (uint64_t)(kNegEnd - kNegBeg) + 1;
  const uint64_t total = n_pos + n_neg;
  std::vector<std::vector<std::pair<uint32_t, uint32_t>>> parts(nt);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++) {
    th.emplace_back([&, t]() {
      const uint64_t b = total * t / nt, e = total * (t + 1) / nt;
      for (uint64_t i = b; i < e; i++) {
        const uint32_t bits = i < n_pos ? (uint32_t)i : (uint32_t)(kNegBeg + (i - n_pos));
        uint32_t g;
        if (differs(bits, &g)) parts[t].push_back({bits, g});
      }
    });
  }
  for (auto& x : th) x.join();
  std::vector<std::pair<uint32_t, uint32_t>> all;
  for (auto& p : parts) all.insert(all.end(), p.begin(), p.end());
  std::sort(all.begin(), all.end());
  keys.resize(all.size());
  vals.resize(all.size());
  for (size_t i = 0; i < all.size(); i++) {
    keys[i] = all[i].first;
    vals[i] = all[i].second;
  }
}

std::string cache_path() {
  Dl_info info;
  if (dladdr((void*)&scan, &info) && info.dli_fname) {
    std::string p(info.dli_fname);
    size_t s = p.rfind('/');
    return (s == std::string::npos ? std::string(".") : p.substr(0, s)) + "/_expf_exceptions.bin";
  }
  return "_expf_exceptions.bin";
}

// Spot checks of a cached table against the running libm: listed entries must still be
// exceptions with the same value, and unlisted inputs must agree.
bool validate(const std::vector<uint32_t>& keys, const std::vector<uint32_t>& vals) {
  if (keys.empty() || keys.size() != vals.size()) return false;
  if (!std::is_sorted(keys.begin(), keys.end())) return false;
  const size_t step = std::max<size_t>(1, keys.size() / 257);
  for (size_t i = 0; i < keys.size(); i += step) {
    uint32_t g;
    if (!differs(keys[i], &g) || g != vals[i]) return false;
  }
  uint64_t s = 0x9E3779B97F4A7C15ull;
  for (int i = 0; i < 4096; i++) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    const uint32_t bits = (i & 1) ? (uint32_t)((s >> 33) % (kPosEnd + 1))
                                  : (uint32_t)(kNegBeg + (s >> 33) % (kNegEnd - kNegBeg + 1));
    uint32_t g;
    const bool d = differs(bits, &g);
    const bool listed = std::binary_search(keys.begin(), keys.end(), bits);
    if (d != listed) return false;
  }
  return true;
}

bool load(const std::string& path, std::vector<uint32_t>& keys, std::vector<uint32_t>& vals) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  uint32_t magic = 0, n = 0;
  bool ok = fread(&magic, 4, 1, f) == 1 && magic == 0x45585046u && fread(&n, 4, 1, f) == 1 && n < (1u << 24);
  if (ok) {
    keys.resize(n);
    vals.resize(n);
    ok = fread(keys.data(), 4, n, f) == n && fread(vals.data(), 4, n, f) == n;
  }
  fclose(f);
  return ok && validate(keys, vals);
}

void save(const std::string& path, const std::vector<uint32_t>& keys, const std::vector<uint32_t>& vals) {
  const std::string tmp = path + ".tmp" + std::to_string((unsigned long)getpid());
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return;
  const uint32_t magic = 0x45585046u, n = (uint32_t)keys.size();
  bool ok = fwrite(&magic, 4, 1, f) == 1 && fwrite(&n, 4, 1, f) == 1 && fwrite(keys.data(), 4, n, f) == n &&
            fwrite(vals.data(), 4, n, f) == n;
  ok = (fclose(f) == 0) && ok;
  if (ok) rename(tmp.c_str(), path.c_str());
  else remove(tmp.c_str());
}

std::once_flag g_once;
std::vector<uint32_t> g_keys, g_vals;

}  // namespace

const std::vector<uint32_t>& expf_exception_keys() {
  std::call_once(g_once, []() {
    const std::string p = cache_path();
    if (!load(p, g_keys, g_vals)) {
      scan(g_keys, g_vals);
      save(p, g_keys, g_vals);
    }
  });
  return g_keys;
}

const std::vector<uint32_t>& expf_exception_vals() {
  expf_exception_keys();
  return g_vals;
}

void expf_exception_hash(std::vector<uint2>& slots, uint32_t* mask, int* max_probe) {
  const auto& keys = expf_exception_keys();
  const auto& vals = expf_exception_vals();
  size_t cap = 1024;
  while (cap < keys.size() * 3) cap <<= 1;  // load factor <= 1/3
  slots.assign(cap, make_uint2(kExpfEmpty, 0u));
  *mask = (uint32_t)(cap - 1);
  int longest = 1;
  for (size_t k = 0; k < keys.size(); k++) {
    uint32_t i = expf_hash(keys[k]) & *mask;
    int probe = 1;
    while (slots[i].x != kExpfEmpty) {
      i = (i + 1) & *mask;
      probe++;
    }
    slots[i] = make_uint2(keys[k], vals[k]);
    longest = std::max(longest, probe);
  }
  *max_probe = longest;
}

}  // namespace dpuf

// Builds (or validates) the cached table; returns the number of exceptions.  Called by the
// package build so that the scan runs once per machine image, not once per process.
extern "C" __attribute__((visibility("default"))) int64_t dpuf_cuda_prepare_expf_table(void) {
  return (int64_t)dpuf::expf_exception_keys().size();
}

namespace dpuf {
namespace {

__global__ void expf_eval_kernel(uint32_t bits0, long long n, float* out, ExpfTable t) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = glibc_expf(__uint_as_float(bits0 + (uint32_t)i), t);
}

}  // namespace
}  // namespace dpuf

// The device's glibc-compatible expf (the function the softmax and SwiGLU tails use), evaluated
// for the `count` consecutive float bit patterns starting at bits_begin into out_dev (device,
// `count` floats), so that a test can compare it with the host libm over whole input ranges.
// Uploads the exception table for the call (allocates and frees it); synchronous.  Returns 0,
// -1 for bad arguments (the range must not pass 0xFFFFFFFF), -4 for a CUDA error.
extern "C" __attribute__((visibility("default"))) int32_t dpuf_cuda_expf_eval(uint32_t bits_begin, int64_t count,
                                                                           float* out_dev) {
  if (!out_dev || count <= 0 || (uint64_t)bits_begin + (uint64_t)count > (1ull << 32)) return -1;
  std::vector<uint2> slots;
  dpuf::ExpfTable t{};
  dpuf::expf_exception_hash(slots, &t.mask, &t.max_probe);
  uint2* d = nullptr;
  if (cudaMalloc(&d, slots.size() * sizeof(uint2)) != cudaSuccess) return -4;
  cudaError_t e = cudaMemcpy(d, slots.data(), slots.size() * sizeof(uint2), cudaMemcpyHostToDevice);
  t.slots = d;
  if (e == cudaSuccess) {
    dpuf::expf_eval_kernel<<<1184, 256>>>(bits_begin, (long long)count, out_dev, t);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(d);
  return e == cudaSuccess ? 0 : -4;
}
