// GGUF v2/v3 header reader (tensor infos with absolute file offsets).
//
// The reference engine never parses the header: it maps tensors through a generated
// table of absolute offsets (src/model.cpp:78-133, include/minicpm_metadata.h).  This
// reader resolves the same tensors by name from the file itself, so any file with the
// MiniCPM5 tensor set (Q4_K_M mix or another supported mix) loads.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mcpm {

struct GGUFTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;   // dims[0] = columns (input), dims[1] = rows
    uint64_t offset = 0;          // absolute file offset
    uint64_t nbytes = 0;
};

struct GGUFFile {
    uint64_t file_size = 0;
    uint64_t data_start = 0;
    uint32_t alignment = 32;
    std::map<std::string, uint64_t> u64_kv;   // integer metadata (u8..u64, i8..i64)
    std::map<std::string, double> f_kv;       // float metadata
    std::vector<GGUFTensor> tensors;
};

// Returns an empty string on success, otherwise a description of the problem.
std::string gguf_read(const std::string& path, GGUFFile& out);
// Bytes of a tensor of `type` with `n` elements, 0 for unsupported types.
uint64_t ggml_nbytes(uint32_t type, uint64_t n);

}  // namespace mcpm
