// noalloc.cu - the standalone mode-12 matmul for callers that cannot allocate device memory.
//
// Who needs this: hosts that reserve the GPU's memory for their own pool when they start (an
// inference server sizing its KV pool to "all free memory", a framework with a caching
// allocator), where any further cudaMalloc either fails or escapes the host's accounting; and
// latency-critical loops where cudaMalloc/cudaFree are unacceptable because they can
// synchronise the device.  dpuf_cuda_matmul_noalloc takes the weight, the input and the output
// as device buffers the caller already owns and allocates nothing: its only scratch, the
// quantised activation (int8 codes, block scales, block sums), lives in a fixed array compiled
// into this library's device image.
//
// Limits and sharing rules:
//   * M * cols <= 1,048,576 activation values per call (1.25 MiB of scratch); larger calls are
//     rejected with -2 and an error text.  Every GPU that loads the library holds the array
//     until the process exits.
//   * All calls share the one array and it keeps the last call's contents.  Nothing in it needs
//     to start at zero: every call rewrites the codes, scales and sums it reads.  Calls whose
//     kernels overlap on the GPU (different streams, or different host threads on one device)
//     race on the array and give wrong results; serialise them.
//   * Every call resolves the array's device address on the current device
//     (cudaGetSymbolAddress, which allocates nothing), so a module reloaded after
//     cudaDeviceReset is picked up; the first call on each device also sets the kernels'
//     shared-memory limits - make that first call before any stream capture.
//   * Tile offsets must be multiples of 16 bytes (as the container writes them); the offsets
//     live in device memory and are not read back, so a misaligned offset gives undefined
//     results instead of an error code.
#include <algorithm>
#include <mutex>
#include <string>

#include "dpuf_cuda.h"
#include "engine_internal.h"
#include "kernels.cuh"

namespace dpuf {
namespace {

constexpr size_t kNoAllocMaxValues = size_t(1) << 20;
constexpr size_t kNoAllocBlocks = kNoAllocMaxValues / 32;
constexpr size_t kNoAllocBytes = kNoAllocMaxValues + kNoAllocBlocks * sizeof(float) + kNoAllocBlocks * sizeof(int32_t);

// Codes [kNoAllocMaxValues] int8, then block scales [kNoAllocBlocks] float, then block sums
// [kNoAllocBlocks] int32.  In host code this name is only a stand-in for the symbol; the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
bool g_configured[kMaxDevices] = {};

// With device `dev` current: the scratch array's device address (looked up on every call), and
// once per device the kernels' shared-memory limits.  Neither allocates.
cudaError_t setup_device(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  if (!g_configured[dev]) {
    e = configure_kernels();
    if (e != cudaSuccess) return e;
    g_configured[dev] = true;
  }
  *out = (unsigned char*)p;
  return cudaSuccess;
}

}  // namespace
}  // namespace dpuf

extern "C" {

DPUF_EXPORT int32_t dpuf_cuda_matmul_noalloc(int32_t M, int32_t rows, int32_t cols, int32_t n_tiles,
                                             const float* x_dev, const uint8_t* tiles_dev,
                                             const uint64_t* tile_offsets_dev, const uint8_t* sign_bits_dev,
                                             float* y_dev, void* stream) {
  dpuf::set_error("");
  if (!x_dev || !tiles_dev || !tile_offsets_dev || !y_dev) {
    dpuf::set_error("dpuf_cuda_matmul_noalloc: null device pointer");
    return -1;
  }
  if (((uintptr_t)tiles_dev & 15) != 0) {
    dpuf::set_error("dpuf_cuda_matmul_noalloc: tiles_dev must be 16-byte aligned");
    return -1;
  }
  if (rows <= 0 || cols <= 0 || cols % 64 != 0 || n_tiles != (rows + dpuf::kTileRows - 1) / dpuf::kTileRows) {
    dpuf::set_error("dpuf_cuda_matmul_noalloc: need rows > 0, cols % 64 == 0, n_tiles == ceil(rows / 16)");
    return -1;
  }
  if (M <= 0 || (size_t)M * (size_t)cols > dpuf::kNoAllocMaxValues) {
    dpuf::set_error("dpuf_cuda_matmul_noalloc: M * cols = " + std::to_string((long long)M * cols) +
                    " is outside [1, " + std::to_string(dpuf::kNoAllocMaxValues) +
                    "], the size of the fixed scratch array");
    return -2;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && (dev < 0 || dev >= dpuf::kMaxDevices)) e = cudaErrorInvalidDevice;
  unsigned char* base = nullptr;
  if (e == cudaSuccess) e = dpuf::setup_device(dev, &base);
  if (e != cudaSuccess) {
    dpuf::set_error(std::string("dpuf_cuda_matmul_noalloc: setup: ") + cudaGetErrorString(e));
    return -4;
  }
  int8_t* q8 = (int8_t*)base;
  float* xs = (float*)(base + dpuf::kNoAllocMaxValues);
  int32_t* xm = (int32_t*)(base + dpuf::kNoAllocMaxValues + dpuf::kNoAllocBlocks * sizeof(float));
  const dpuf::W12 w{tiles_dev, tile_offsets_dev, sign_bits_dev, rows, cols, n_tiles};
  const dpuf::Launch L{(cudaStream_t)stream, false};
  // the whole input is prepped into the array once, then the tokens go through the matmul in
  // chunks of at most kMaxBatch (256), as the allocating entry point splits them
  e = dpuf::launch_prep(L, x_dev, cols, M, cols, sign_bits_dev, dpuf::Act{q8, xs, xm, cols});
  for (int c0 = 0; e == cudaSuccess && c0 < M; c0 += dpuf::kMaxBatch) {
    const int mc = std::min(dpuf::kMaxBatch, M - c0);
    const size_t o = (size_t)c0 * cols;
    const dpuf::Act a{q8 + o, xs + o / 32, xm + o / 32, cols};
    dpuf::LinJobs J = {};
    J.n = 1;
    J.j[0] = {w, a, y_dev + (size_t)c0 * rows, rows, 0, n_tiles};
    J.tile_prefix[1] = n_tiles;
    e = mc == 1 ? dpuf::launch_gemv(L, J, nullptr, nullptr) : dpuf::launch_gemm_exact(L, J, mc);
  }
  if (e == cudaErrorInvalidValue) {
    dpuf::set_error("dpuf_cuda_matmul_noalloc: shape not supported by the matmul kernels (cols too large)");
    return -1;
  }
  if (e != cudaSuccess) {
    dpuf::set_error(std::string("dpuf_cuda_matmul_noalloc: launch: ") + cudaGetErrorString(e));
    return -4;
  }
  return 0;
}

}  // extern "C"
