// engine_internal.h - host-side declarations shared by the engine's translation units.
#pragma once
#include <stdint.h>
#include <vector_types.h>

#include <string>
#include <vector>

namespace dpuf {

// glibc expf exception table (expf_table.cu): sorted input bits and glibc output bits.
const std::vector<uint32_t>& expf_exception_keys();
const std::vector<uint32_t>& expf_exception_vals();
// The same table as an open-addressing hash (see ExpfTable in common.cuh).
void expf_exception_hash(std::vector<uint2>& slots, uint32_t* mask, int* max_probe);

// Per-thread text of the last error (engine.cu).
void set_error(const std::string& msg);

}  // namespace dpuf
