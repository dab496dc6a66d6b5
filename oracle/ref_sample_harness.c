/*
 * ref_sample_harness.c - exposes the reference CLI's own token sampler for parity tests.
 *
 * TEST INFRASTRUCTURE ONLY (built by oracle/build_ref.sh into oracle/_ref/, never linked by
 * the product).  The reference's `sample_token` and `rand_f32` (dpuf-cli.c:1987-2027) are
 * file-static inside the CLI, so this file compiles the CLI source where it lies (found on
 * the include path, not copied) with its `main` renamed, and exports one wrapper that runs the
 * sampler from a caller-given generator state and returns the state it leaves.
 */
#define main dpuf_cli_main_unused
#include "dpuf-cli.c"

__attribute__((visibility("default"))) int32_t ref_sample_token(const float* logits, int32_t V, float temp,
                                                                uint64_t* rng) {
  g_rng = *rng;
  const int32_t r = sample_token(logits, V, temp);
  *rng = g_rng;
  return r;
}
