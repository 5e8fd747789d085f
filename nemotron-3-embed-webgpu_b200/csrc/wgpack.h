// .wgpack (WGPACK02) container parser: a C++ restatement of
// parsePrepackedModel (src/prepacked/format.ts:146-169) with the same checks
// and error messages.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace nemo {

enum GgmlType { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_K = 12, kQ6_K = 14 };

struct PackTensor {
  std::string name;
  std::vector<int64_t> dims;  // GGUF order: dims[0] = k (contiguous), dims[1] = n (rows)
  int type = -1;
  bool compact = false;       // storage "q4_0-tile32-compact"
  uint64_t offset = 0;        // relative to the data section
  uint64_t byte_length = 0;
  uint64_t byte_offset = 0;   // absolute offset in the file
};

struct Pack {
  int version = 0;
  std::string source_sha256;
  std::map<std::string, PackTensor> tensors;
  uint64_t data_offset = 0;
};

// Parses and validates the header; tensor payloads stay in the caller's buffer.
// Returns false with `err` set on any format error.
bool parse_wgpack(const uint8_t* data, size_t bytes, Pack* out, std::string* err);

}  // namespace nemo
