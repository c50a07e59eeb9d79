// tokenizer.cpp -- see tokenizer.hpp.
#include "tokenizer.hpp"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <stdexcept>

namespace mmfree_cli {

namespace {

const char kMagic[8] = {'M', 'M', 'T', 'O', 'K', '1', '\n', '\0'};
const char kSpace[] = "\xE2\x96\x81";  // U+2581, the SentencePiece word boundary

struct Reader {
  std::ifstream in;
  std::string path;
  std::uint32_t u32() {
    unsigned char b[4];
    in.read(reinterpret_cast<char*>(b), 4);
    return b[0] | (b[1] << 8) | (b[2] << 16) | (static_cast<std::uint32_t>(b[3]) << 24);
  }
  std::string str() {
    const std::uint32_t n = u32();
    if (!in || n > (1u << 20)) throw std::runtime_error("tokenizer: malformed " + path);
    std::string s(n, '\0');
    if (n) in.read(&s[0], n);
    return s;
  }
};

// Byte length of the UTF-8 code point starting with byte c (1 for continuation / invalid
// lead bytes, which then fall back to byte tokens).
std::size_t cp_len(unsigned char c) {
  if (c >= 0xF0) return 4;
  if (c >= 0xE0) return 3;
  if (c >= 0xC0) return 2;
  return 1;
}

}  // namespace

Tokenizer::Tokenizer(const std::string& path) {
  Reader r{std::ifstream(path, std::ios::binary), path};
  if (!r.in) throw std::runtime_error("tokenizer: cannot open " + path);
  char magic[8];
  r.in.read(magic, 8);
  if (!r.in || std::memcmp(magic, kMagic, 8) != 0)
    throw std::runtime_error("tokenizer: not a tokenizer.mmtok file: " + path);
  const std::uint32_t n_pieces = r.u32(), n_merges = r.u32();
  bos_ = static_cast<std::int32_t>(r.u32());
  eos_ = static_cast<std::int32_t>(r.u32());
  unk_ = static_cast<std::int32_t>(r.u32());
  pieces_.reserve(n_pieces);
  for (std::uint32_t i = 0; i < n_pieces; ++i) {
    pieces_.push_back(r.str());
    ids_.emplace(pieces_.back(), static_cast<int>(i));
  }
  for (std::uint32_t i = 0; i < n_merges; ++i) ranks_.emplace(r.str(), static_cast<int>(i));
  if (!r.in) throw std::runtime_error("tokenizer: truncated " + path);
  for (int b = 0; b < 256; ++b) {
    char name[8];
    std::snprintf(name, sizeof(name), "<0x%02X>", b);
    auto it = ids_.find(name);
    byte_ids_[b] = it == ids_.end() ? -1 : it->second;
  }
}

int Tokenizer::rank(const std::string& left, const std::string& right) const {
  auto it = ranks_.find(left + " " + right);
  return it == ranks_.end() ? std::numeric_limits<int>::max() : it->second;
}

std::vector<std::int64_t> Tokenizer::encode(const std::string& text, bool add_bos) const {
  std::vector<std::int64_t> out;
  if (add_bos) out.push_back(bos_);
  if (text.empty()) return out;
  std::string norm = kSpace;
  for (char c : text) {
    if (c == ' ') norm += kSpace;
    else norm += c;
  }
  std::vector<std::string> sym;  // current pieces, left to right
  for (std::size_t i = 0; i < norm.size();) {
    std::size_t n = cp_len(static_cast<unsigned char>(norm[i]));
    if (i + n > norm.size()) n = 1;
    sym.push_back(norm.substr(i, n));
    i += n;
  }
  // pr[i]: merge rank of the pair (sym[i], sym[i + 1]); merge the lowest, leftmost first
  const int none = std::numeric_limits<int>::max();
  std::vector<int> pr(sym.size() > 1 ? sym.size() - 1 : 0);
  for (std::size_t i = 0; i + 1 < sym.size(); ++i) pr[i] = rank(sym[i], sym[i + 1]);
  while (!pr.empty()) {
    std::size_t best = 0;
    for (std::size_t i = 1; i < pr.size(); ++i)
      if (pr[i] < pr[best]) best = i;
    if (pr[best] == none) break;
    sym[best] += sym[best + 1];
    sym.erase(sym.begin() + static_cast<std::ptrdiff_t>(best) + 1);
    pr.erase(pr.begin() + static_cast<std::ptrdiff_t>(best));
    if (best > 0) pr[best - 1] = rank(sym[best - 1], sym[best]);
    if (best < pr.size()) pr[best] = rank(sym[best], sym[best + 1]);
  }
  for (const std::string& s : sym) {
    auto it = ids_.find(s);
    if (it != ids_.end()) {
      out.push_back(it->second);
    } else {
      for (unsigned char c : s) out.push_back(byte_ids_[c]);
    }
  }
  return out;
}

std::string Tokenizer::decode(const std::vector<std::int64_t>& ids, bool skip_special) const {
  std::string out;
  const std::size_t sp = std::strlen(kSpace);
  for (std::int64_t id : ids) {
    if (id < 0 || static_cast<std::size_t>(id) >= pieces_.size()) continue;
    if (skip_special && (id == bos_ || id == eos_ || id == unk_)) continue;
    const std::string& p = pieces_[static_cast<std::size_t>(id)];
    if (p.size() == 6 && p.compare(0, 3, "<0x") == 0 && p[5] == '>') {  // a byte token
      out.push_back(static_cast<char>(std::strtol(p.substr(3, 2).c_str(), nullptr, 16)));
      continue;
    }
    for (std::size_t i = 0; i < p.size();) {
      if (p.compare(i, sp, kSpace) == 0) {
        out.push_back(' ');
        i += sp;
      } else {
        out.push_back(p[i++]);
      }
    }
  }
  if (!out.empty() && out[0] == ' ') out.erase(0, 1);
  return out;
}

}  // namespace mmfree_cli
