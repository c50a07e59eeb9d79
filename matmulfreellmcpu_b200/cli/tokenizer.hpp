// tokenizer.hpp -- text <-> token ids for the CLI's text mode, from a tokenizer.mmtok file.
//
// The file is the reference's packed LLaMA SentencePiece-BPE tokenizer (matmulfreellmCPU
// tools/provision.py:171-219): magic "MMTOK1\n\0", u32 vocab size, u32 merge count, i32
// bos / eos / unk ids, then every piece and every merge ("left right", in rank order) as a
// u32 byte length + UTF-8 bytes. The algorithm is that of the reference's Tokenizer
// (cpp/include/mmfree/tokenizer.hpp, cpp/src/io/tokenizer.cpp:83-182):
//   encode: optional BOS; the text with U+2581 prepended and every ' ' replaced by U+2581,
//           split into UTF-8 code points; then repeatedly the adjacent pair with the lowest
//           merge rank (the leftmost on ties) is merged; final pieces that are not in the
//           vocabulary fall back to their bytes' <0xNN> tokens.
//   decode: specials skipped (optional), <0xNN> tokens as raw bytes, U+2581 as ' ', one
//           leading space removed.
// This is host code of the CLI (no GPU).
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace mmfree_cli {

class Tokenizer {
 public:
  explicit Tokenizer(const std::string& path);
  std::vector<std::int64_t> encode(const std::string& text, bool add_bos = true) const;
  std::string decode(const std::vector<std::int64_t>& ids, bool skip_special = true) const;
  std::int64_t bos_id() const { return bos_; }
  std::int64_t eos_id() const { return eos_; }
  std::int64_t unk_id() const { return unk_; }
  std::size_t vocab_size() const { return pieces_.size(); }

 private:
  int rank(const std::string& left, const std::string& right) const;
  std::vector<std::string> pieces_;
  std::unordered_map<std::string, int> ids_;
  std::unordered_map<std::string, int> ranks_;  // "left right" -> merge rank
  int byte_ids_[256];                           // <0xNN> -> id, -1 when absent
  std::int64_t bos_ = 1, eos_ = 2, unk_ = 0;
};

}  // namespace mmfree_cli
