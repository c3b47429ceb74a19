#include "tokenizer.h"

#include <stdexcept>

namespace minimind {

std::vector<int32_t> ByteTokenizer::encode(const std::string& text) const {
  return std::vector<int32_t>(reinterpret_cast<const unsigned char*>(text.data()),
                              reinterpret_cast<const unsigned char*>(text.data()) + text.size());
}

std::string ByteTokenizer::decode(const std::vector<int32_t>& tokens) const {
  std::string out;
  out.reserve(tokens.size());
  for (int32_t t : tokens) {
    if (t < 0 || t > 255) throw std::invalid_argument("ByteTokenizer can only decode tokens in [0, 255]");
    out.push_back(static_cast<char>(t));
  }
  return out;
}

}  // namespace minimind
