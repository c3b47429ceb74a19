// Byte-level fallback tokenizer used by the CLIs when no token ids are given
// (same behaviour as the reference's ByteTokenizer, src/csrc/lib/tokenizer.cpp:7-26).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace minimind {

class ByteTokenizer {
 public:
  std::vector<int32_t> encode(const std::string& text) const;
  std::string decode(const std::vector<int32_t>& tokens) const;
};

}  // namespace minimind
