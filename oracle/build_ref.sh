#!/usr/bin/env bash
# Builds the UNMODIFIED reference engine (libdpuf_avx2.so) out of tree, for use as the
# parity checker and the timed CPU baseline.  Test infrastructure only: nothing in the
# product links or loads this library.
#
#   usage: oracle/build_ref.sh REF_DIR     (or env DPUF_REFERENCE_DIR; there is no default)
#
# Outputs go only to oracle/_ref/ (git-ignored; it still travels with the repository
# snapshot to the GPU box).  The reference sources are read where they lie; the only
# file written outside the compiler's objects is a patched temporary copy of
# dpuf_engine.c under oracle/_ref/src/, needed because GCC rejects one OpenMP construct
# in it (dpuf_engine.c:1891-1893, `omp atomic capture` with a cast).  That single
# statement is replaced by the equivalent __atomic_fetch_add.  Everything else is
# handled without touching the sources:
#   * dpuf_avx2.c:12 includes MSVC's <intrin.h>  -> shim/intrin.h on the include path;
#   * dpuf_kernels.h:13 defines __forceinline as "static inline ..." which doubles the
#     `static` keyword                          -> pre-defined on the command line;
#   * dpuf_engine.c:1216 calloc()s a struct with 64-byte aligned members; GCC -O3 emits
#     aligned AVX stores into it and glibc calloc only guarantees 16 bytes -> the
#     pre-include maps calloc to a 64-byte aligned allocation (freeable with free()).
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${DPUF_REFERENCE_DIR:-}}"
if [ -z "$REF" ]; then
  echo "build_ref: give the reference source directory (argument or DPUF_REFERENCE_DIR)" >&2
  exit 2
fi
OUT="$HERE/_ref"
if [ ! -f "$REF/dpuf_engine.c" ]; then
  echo "build_ref: reference sources not found at $REF" >&2
  exit 2
fi
mkdir -p "$OUT/src" "$OUT/shim"

cat > "$OUT/shim/intrin.h" <<'EOF'
#pragma once
#include <x86intrin.h>
static inline unsigned char _BitScanForward(unsigned long* idx, unsigned long mask) {
    if (!mask) return 0;
    *idx = (unsigned long)__builtin_ctzl(mask);
    return 1;
}
EOF

cat > "$OUT/shim/pre.h" <<'EOF'
#pragma once
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#include <sys/select.h>
static inline void* dpuf_ref_calloc64(size_t n, size_t sz) {
    size_t total = n * sz;
    void* p = NULL;
    if (total == 0) total = 64;
    if (posix_memalign(&p, 64, (total + 63) & ~(size_t)63) != 0) return NULL;
    memset(p, 0, total);
    return p;
}
#define calloc(n, s) dpuf_ref_calloc64((n), (s))
#define _strtoi64 strtoll
EOF

# dpuf_engine.c: replace the GCC-rejected atomic capture by an equivalent builtin.
python3 - "$REF/dpuf_engine.c" "$OUT/src/dpuf_engine.c" <<'EOF'
import sys
src = open(sys.argv[1]).read()
old = "#pragma omp atomic capture\n                    { task = (int32_t)(*a_ctr); (*a_ctr)++; }"
new = "task = (int32_t)__atomic_fetch_add((long*)a_ctr, 1L, __ATOMIC_SEQ_CST);"
if src.count(old) != 1:
    sys.exit("build_ref: patch site not found exactly once in dpuf_engine.c")
open(sys.argv[2], "w").write(src.replace(old, new))
EOF

CFLAGS=(-O3 -mavx2 -mfma -mf16c -fopenmp -std=gnu11 -fPIC -w
        "-D__forceinline=inline __attribute__((always_inline))"
        -I"$OUT/shim" -I"$REF" -include "$OUT/shim/pre.h")
gcc "${CFLAGS[@]}" -c "$REF/dpuf_avx2.c"      -o "$OUT/dpuf_avx2.o"
gcc "${CFLAGS[@]}" -c "$OUT/src/dpuf_engine.c" -o "$OUT/dpuf_engine.o"
gcc "${CFLAGS[@]}" -c "$REF/dpuf_vision.c"    -o "$OUT/dpuf_vision.o"
gcc -shared -fopenmp -o "$OUT/libdpuf_avx2.so" \
    "$OUT/dpuf_avx2.o" "$OUT/dpuf_engine.o" "$OUT/dpuf_vision.o" -lm
echo "build_ref: built $OUT/libdpuf_avx2.so"

# The reference's own C host (dpuf-cli.c, unmodified): once over the reference engine, and once
# linked as its Makefile would be with this repository's libdpuf_cuda.so providing every
# dpuf_engine_* symbol (the CLI's load-time helpers - tile CRC checks, vision - stay the
# reference's objects).  The second binary is the drop-in demonstration the GPU tests run.
gcc "${CFLAGS[@]}" -c "$REF/dpuf-cli.c" -o "$OUT/dpuf-cli.o"
gcc -fopenmp -o "$OUT/dpuf-cli" "$OUT/dpuf-cli.o" -L"$OUT" -ldpuf_avx2 -Wl,-rpath,'$ORIGIN' -lm
echo "build_ref: built $OUT/dpuf-cli"
CUDA_LIB_DIR="$HERE/../dpuf_b200"
if [ -f "$CUDA_LIB_DIR/libdpuf_cuda.so" ]; then
  gcc -fopenmp -o "$OUT/dpuf-cli-cuda" "$OUT/dpuf-cli.o" "$OUT/dpuf_avx2.o" "$OUT/dpuf_vision.o" \
      -L"$CUDA_LIB_DIR" -ldpuf_cuda -Wl,-rpath,'$ORIGIN/../../dpuf_b200' -lm
  echo "build_ref: built $OUT/dpuf-cli-cuda"
fi
rm -f "$OUT"/*.o

# The CLI's token sampler (file-static in dpuf-cli.c), exported by oracle/ref_sample_harness.c.
gcc "${CFLAGS[@]}" -shared "$HERE/ref_sample_harness.c" -o "$OUT/libdpuf_ref_sample.so" \
    -L"$OUT" -ldpuf_avx2 -Wl,-rpath,'$ORIGIN' -lm
echo "build_ref: built $OUT/libdpuf_ref_sample.so"
