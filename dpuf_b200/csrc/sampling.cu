// Token sampling of the reference's callers (host code).
//
// The engine returns logits; the reference's callers pick the next token with
// `sample_token` (dpuf-cli.c:1997-2027) and its generator `rand_f32` (dpuf-cli.c:1987-1995),
// host code that every caller of the engine (CLI turns, bench, HTTP server) runs.  Greedy
// selection also runs on the device (the persistent decode kernel and argmax_blocks_kernel);
// temperature sampling stays on the host, as in the reference: its probability sum is a
// sequential double-precision chain over the whole vocabulary whose rounding decides the
// chosen id, and glibc's expf produces the probabilities, so the host's own libm is the
// exact match.
//
//   greedy (temp <= 0): the first index of the maximum (strict '>');
//   temp > 0: m = max, p_i = expf((l_i - m) * (1/temp)) in fp32, S = sequential double sum,
//             r = (double)u * S with u from xorshift64*, the first i whose sequential double
//             prefix reaches r (else V - 1).
#include <math.h>
#include <stdint.h>

#include <vector>

#include "dpuf_cuda.h"

namespace {

// rand_f32 (dpuf-cli.c:1988-1995): xorshift64 step, then the top 24 bits of the
// multiplied state as a fraction of 2^24.
float next_uniform(uint64_t* state) {
  uint64_t x = *state;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *state = x;
  return (float)((x * 2685821657736338717ULL) >> 40) / 16777216.0f;
}

}  // namespace

extern "C" DPUF_EXPORT uint64_t dpuf_cuda_sample_seed(void) { return 88172645463325252ULL; }

extern "C" DPUF_EXPORT int32_t dpuf_cuda_sample_token(const float* logits, int32_t V, float temp, uint64_t* rng) {
  if (!logits || V <= 0) return -1;
  if (temp <= 0.0f) {
    int32_t best = 0;
    float best_v = logits[0];
    for (int32_t i = 1; i < V; i++)
      if (logits[i] > best_v) {
        best_v = logits[i];
        best = i;
      }
    return best;
  }
  if (!rng) return -1;
  float max_l = logits[0];
  for (int32_t i = 1; i < V; i++)
    if (logits[i] > max_l) max_l = logits[i];
  const float inv_t = 1.0f / temp;
  thread_local std::vector<float> probs;
  probs.resize((size_t)V);
  double sum = 0.0;
  for (int32_t i = 0; i < V; i++) {
    const float p = expf((logits[i] - max_l) * inv_t);
    probs[(size_t)i] = p;
    sum += (double)p;
  }
  const double r = (double)next_uniform(rng) * sum;
  double cdf = 0.0;
  for (int32_t i = 0; i < V; i++) {
    cdf += (double)probs[(size_t)i];
    if (cdf >= r) return i;
  }
  return V - 1;
}
