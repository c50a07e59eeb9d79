// blob.cpp -- model.mmfree reader: mmap + a small recursive-descent JSON parser.
#include "blob.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace mmfree_cuda {
namespace {

struct JValue {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<JValue> items;
  std::vector<std::pair<std::string, JValue>> members;

  const JValue* member(const char* key) const {
    for (const auto& kv : members)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JReader {
 public:
  JReader(const char* p, const char* end) : p_(p), end_(end) {}
  JValue document() {
    JValue v = value();
    skip();
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("weights: bad header json (") + what + ")");
  }
  void skip() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool eat(char c) {
    skip();
    if (p_ < end_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  void expect(char c) {
    if (!eat(c)) fail("unexpected character");
  }
  JValue value() {
    skip();
    if (p_ >= end_) fail("truncated");
    const char c = *p_;
    if (c == '{') return object();
    if (c == '[') return array();
    if (c == '"') {
      JValue v;
      v.kind = JValue::String;
      v.str = string();
      return v;
    }
    if (c == 't' || c == 'f' || c == 'n') return literal();
    return number();
  }
  JValue object() {
    JValue v;
    v.kind = JValue::Object;
    expect('{');
    if (eat('}')) return v;
    do {
      skip();
      std::string k = string();
      expect(':');
      v.members.emplace_back(std::move(k), value());
    } while (eat(','));
    expect('}');
    return v;
  }
  JValue array() {
    JValue v;
    v.kind = JValue::Array;
    expect('[');
    if (eat(']')) return v;
    do v.items.push_back(value());
    while (eat(','));
    expect(']');
    return v;
  }
  std::string string() {
    if (p_ >= end_ || *p_ != '"') fail("expected string");
    ++p_;
    std::string s;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= end_) fail("truncated escape");
        char e = *p_++;
        switch (e) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u':
            if (end_ - p_ < 4) fail("truncated \\u");
            s += '?';  // tensor names and config keys are ASCII
            p_ += 4;
            break;
          default: s += e;
        }
      } else {
        s += c;
      }
    }
    if (p_ >= end_) fail("unterminated string");
    ++p_;
    return s;
  }
  JValue literal() {
    JValue v;
    auto match = [&](const char* w) {
      size_t n = std::strlen(w);
      if (static_cast<size_t>(end_ - p_) >= n && std::strncmp(p_, w, n) == 0) {
        p_ += n;
        return true;
      }
      return false;
    };
    if (match("true")) { v.kind = JValue::Bool; v.b = true; }
    else if (match("false")) { v.kind = JValue::Bool; v.b = false; }
    else if (match("null")) { v.kind = JValue::Null; }
    else fail("bad literal");
    return v;
  }
  JValue number() {
    const char* s = p_;
    while (p_ < end_ && (std::strchr("+-0123456789.eE", *p_) != nullptr)) ++p_;
    if (p_ == s) fail("bad value");
    JValue v;
    v.kind = JValue::Number;
    v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
    return v;
  }
};

constexpr size_t kAlign = 64;
size_t align_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

}  // namespace

Blob::Blob(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("weights: cannot open " + path);
  struct stat st {};
  if (::fstat(fd_, &st) != 0) {
    ::close(fd_);
    throw std::runtime_error("weights: fstat failed for " + path);
  }
  size_ = static_cast<size_t>(st.st_size);
  if (size_ < 16) {
    ::close(fd_);
    throw std::runtime_error("weights: bad magic in " + path);
  }
  base_ = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (base_ == MAP_FAILED) {
    base_ = nullptr;
    ::close(fd_);
    throw std::runtime_error("weights: mmap failed for " + path);
  }
  try {
    const char* bytes = static_cast<const char*>(base_);
    const bool v2 = std::strncmp(bytes, "MMFREE2\n", 8) == 0;
    if (!v2 && std::strncmp(bytes, "MMFREE1\n", 8) != 0)
      throw std::runtime_error("weights: bad magic in " + path);
    uint64_t hl = 0;
    std::memcpy(&hl, bytes + 8, 8);
    if (hl > size_ - 16) throw std::runtime_error("weights: truncated header in " + path);
    JValue root = JReader(bytes + 16, bytes + 16 + hl).document();
    const JValue* c = root.member("config");
    if (!c || c->kind != JValue::Object) throw std::runtime_error("weights: no config in header");
    auto num = [&](const char* k, size_t def) {
      const JValue* j = c->member(k);
      return j && j->kind == JValue::Number ? static_cast<size_t>(j->num) : def;
    };
    auto flag = [&](const char* k, bool def) {
      const JValue* j = c->member(k);
      return j && j->kind == JValue::Bool ? j->b : def;
    };
    cfg_.vocab_size = num("vocab_size", cfg_.vocab_size);
    cfg_.hidden_size = num("hidden_size", cfg_.hidden_size);
    cfg_.num_hidden_layers = num("num_hidden_layers", cfg_.num_hidden_layers);
    cfg_.num_heads = num("num_heads", cfg_.num_heads);
    cfg_.expand_ratio = num("expand_ratio", cfg_.expand_ratio);
    cfg_.intermediate_size = num("intermediate_size", cfg_.intermediate_size);
    cfg_.use_lower_bound = flag("use_lower_bound", cfg_.use_lower_bound);
    cfg_.use_short_conv = flag("use_short_conv", cfg_.use_short_conv);
    if (const JValue* e = c->member("rms_norm_eps"))
      if (e->kind == JValue::Number) cfg_.rms_norm_eps = static_cast<float>(e->num);

    const size_t data_start = align_up(16 + hl);
    const JValue* ts = root.member("tensors");
    if (!ts || ts->kind != JValue::Object) throw std::runtime_error("weights: no tensors in header");
    for (const auto& kv : ts->members) {
      const JValue& m = kv.second;
      BlobTensor t;
      const JValue* dt = m.member("dtype");
      t.is_int8 = dt && dt->kind == JValue::String && dt->str == "i8";
      t.is_packed = v2 && dt && dt->kind == JValue::String && dt->str == "t2";
      if (const JValue* sh = m.member("shape"))
        for (const auto& d : sh->items) t.shape.push_back(static_cast<size_t>(d.num));
      const JValue* off = m.member("offset");
      if (!off) throw std::runtime_error("weights: tensor without offset: " + kv.first);
      t.offset = data_start + static_cast<size_t>(off->num);
      if (t.is_packed) {
        if (t.shape.size() != 2) throw std::runtime_error("weights: t2 tensor must be 2-D: " + kv.first);
        // tiled 2-bit: 32-row groups x 64-column chunks of 512 bytes (common.cuh)
        t.nbytes = (t.shape[0] + 31) / 32 * ((t.shape[1] + 63) / 64) * 512;
      } else {
        t.nbytes = t.numel() * (t.is_int8 ? 1 : 4);
      }
      if (t.offset + t.nbytes > size_)
        throw std::runtime_error("weights: tensor past end of file: " + kv.first);
      tensors_.emplace(kv.first, std::move(t));
    }
  } catch (...) {
    ::munmap(base_, size_);
    ::close(fd_);
    base_ = nullptr;
    fd_ = -1;
    throw;
  }
}

Blob::~Blob() {
  if (base_) ::munmap(base_, size_);
  if (fd_ >= 0) ::close(fd_);
}

const BlobTensor& Blob::get(const std::string& name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw std::runtime_error("weights: missing tensor " + name);
  return it->second;
}

}  // namespace mmfree_cuda
