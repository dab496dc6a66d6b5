// engine_internal.h - host-side declarations shared by the engine's translation units.
#pragma once
#include <stdint.h>

#include <string>
#include <vector>

namespace dpuf {

// glibc expf exception table (expf_table.cu): sorted input bits and glibc output bits.
const std::vector<uint32_t>& expf_exception_keys();
const std::vector<uint32_t>& expf_exception_vals();

// Per-thread text of the last error (engine.cu).
void set_error(const std::string& msg);

}  // namespace dpuf
