#include "gguf.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace lfm {

bool ggml_block_info(uint32_t type, uint64_t& block, uint64_t& bytes) {
  switch (type) {
    case 0: block = 1; bytes = 4; return true;      // F32
    case 1: block = 1; bytes = 2; return true;      // F16
    case 2: block = 32; bytes = 18; return true;    // Q4_0
    case 3: block = 32; bytes = 20; return true;    // Q4_1
    case 6: block = 32; bytes = 22; return true;    // Q5_0
    case 7: block = 32; bytes = 24; return true;    // Q5_1
    case 8: block = 32; bytes = 34; return true;    // Q8_0
    case 9: block = 32; bytes = 36; return true;    // Q8_1
    case 10: block = 256; bytes = 84; return true;  // Q2_K
    case 11: block = 256; bytes = 112; return true; // Q3_K
    case 12: block = 256; bytes = 144; return true; // Q4_K
    case 13: block = 256; bytes = 176; return true; // Q5_K
    case 14: block = 256; bytes = 210; return true; // Q6_K
    case 15: block = 256; bytes = 288; return true; // Q8_K
    default: return false;
  }
}

namespace {

// Well-formed UTF-8 (RFC 3629): no overlong forms, no surrogates, nothing
// above U+10FFFF; the check Rust's String::from_utf8 makes.
bool valid_utf8(const std::string& s) {
  const unsigned char* p = (const unsigned char*)s.data();
  size_t i = 0, n = s.size();
  while (i < n) {
    unsigned c = p[i];
    if (c < 0x80) { i++; continue; }
    int len;
    unsigned cp;
    if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; k++) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
    if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// Buffered sequential reader over the header region.
class Reader {
 public:
  Reader(int fd, uint64_t len) : fd_(fd), len_(len) {}
  bool bytes(void* dst, size_t n) {
    uint8_t* d = (uint8_t*)dst;
    while (n) {
      if (pos_ == fill_) {
        if (!refill()) return false;
      }
      size_t take = std::min(n, fill_ - pos_);
      memcpy(d, buf_.data() + pos_, take);
      pos_ += take;
      d += take;
      n -= take;
      consumed_ += take;
    }
    return true;
  }
  template <class T> bool get(T& v) { return bytes(&v, sizeof(T)); }
  // GGUF string: u64 length, then UTF-8 bytes (gguf.rs read_string). A
  // violation other than running out of file leaves its message in `err`.
  bool str(std::string& s, std::string& err) {
    uint64_t n;
    if (!get(n)) return false;
    if (n > (1ull << 30)) {
      err = "String length " + std::to_string(n) + " exceeds maximum (1 GiB)";
      return false;
    }
    if (n > len_) return false;  // longer than the file: truncated
    s.resize(n);
    if (n && !bytes(&s[0], n)) return false;
    if (!valid_utf8(s)) {
      err = "Invalid UTF-8 in string";
      return false;
    }
    return true;
  }
  uint64_t position() const { return consumed_; }

 private:
  bool refill() {
    buf_.resize(1 << 20);
    ssize_t r = pread(fd_, buf_.data(), buf_.size(), (off_t)file_pos_);
    if (r <= 0) return false;
    file_pos_ += (uint64_t)r;
    fill_ = (size_t)r;
    pos_ = 0;
    return true;
  }
  int fd_;
  uint64_t len_;
  std::vector<uint8_t> buf_;
  size_t pos_ = 0, fill_ = 0;
  uint64_t file_pos_ = 0, consumed_ = 0;
};

bool read_value(Reader& r, uint32_t t, GgufValue& v, std::string& err, int depth) {
  v.gtype = t;
  switch (t) {
    case 0: { uint8_t x; if (!r.get(x)) return false; v.kind = GgufValue::UINT; v.u = x; v.i = x; return true; }
    case 1: { int8_t x; if (!r.get(x)) return false; v.kind = GgufValue::INT; v.i = x; v.u = (uint64_t)x; return true; }
    case 2: { uint16_t x; if (!r.get(x)) return false; v.kind = GgufValue::UINT; v.u = x; v.i = x; return true; }
    case 3: { int16_t x; if (!r.get(x)) return false; v.kind = GgufValue::INT; v.i = x; v.u = (uint64_t)x; return true; }
    case 4: { uint32_t x; if (!r.get(x)) return false; v.kind = GgufValue::UINT; v.u = x; v.i = x; return true; }
    case 5: { int32_t x; if (!r.get(x)) return false; v.kind = GgufValue::INT; v.i = x; v.u = (uint64_t)x; return true; }
    case 6: { float x; if (!r.get(x)) return false; v.kind = GgufValue::FLOAT; v.f = x; return true; }
    case 7: {
      uint8_t x;
      if (!r.get(x)) return false;
      if (x > 1) { err = "Invalid BOOL value: " + std::to_string(x); return false; }
      v.kind = GgufValue::BOOL;
      v.u = x;
      return true;
    }
    case 8: v.kind = GgufValue::STRING; return r.str(v.s, err);
    case 9: {
      uint32_t et;
      uint64_t n;
      if (!r.get(et) || !r.get(n)) return false;
      if (n > 10000000ull) { err = "Array length " + std::to_string(n) + " exceeds maximum (10 M)"; return false; }
      if (depth > 4) { err = "nested arrays too deep"; return false; }
      v.kind = GgufValue::ARRAY;
      v.arr.resize(n);
      for (uint64_t i = 0; i < n; i++)
        if (!read_value(r, et, v.arr[i], err, depth + 1)) return false;
      return true;
    }
    case 10: { uint64_t x; if (!r.get(x)) return false; v.kind = GgufValue::UINT; v.u = x; v.i = (int64_t)x; return true; }
    case 11: { int64_t x; if (!r.get(x)) return false; v.kind = GgufValue::INT; v.i = x; v.u = (uint64_t)x; return true; }
    case 12: { double x; if (!r.get(x)) return false; v.kind = GgufValue::FLOAT; v.f = x; return true; }
    default: err = "Unknown metadata value type: " + std::to_string(t); return false;
  }
}

}  // namespace

GgufFile::~GgufFile() {
  if (fd_ >= 0) close(fd_);
}

bool GgufFile::open(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) { err_ = "open model file " + path; return false; }
  struct stat st;
  if (fstat(fd_, &st) != 0) { err_ = "stat model file"; return false; }
  file_len_ = (uint64_t)st.st_size;
  Reader r(fd_, file_len_);
  const std::string trunc = "Unexpected end of file (truncated input)";
  char magic[4];
  if (!r.bytes(magic, 4)) { err_ = trunc; return false; }
  if (memcmp(magic, "GGUF", 4) != 0) { err_ = "Invalid magic (expected \"GGUF\")"; return false; }
  uint32_t version;
  uint64_t tensor_count, kv_count;
  if (!r.get(version)) { err_ = trunc; return false; }
  if (version != 3) { err_ = "Unsupported GGUF version: " + std::to_string(version) + " (expected 3)"; return false; }
  if (!r.get(tensor_count) || !r.get(kv_count)) { err_ = trunc; return false; }
  const uint64_t MAX_COUNT = 100000;
  if (tensor_count > MAX_COUNT) {
    err_ = "Tensor count " + std::to_string(tensor_count) + " exceeds maximum (100000)";
    return false;
  }
  if (kv_count > MAX_COUNT) {
    err_ = "KV count " + std::to_string(kv_count) + " exceeds maximum (100000)";
    return false;
  }
  for (uint64_t i = 0; i < kv_count; i++) {
    std::string key, e;
    uint32_t vt;
    if (!r.str(key, e) || !r.get(vt)) { err_ = e.empty() ? trunc : e; return false; }
    GgufValue v;
    if (!read_value(r, vt, v, e, 0)) { err_ = e.empty() ? trunc : e; return false; }
    if (meta_.count(key)) { err_ = "Duplicate metadata key: " + key; return false; }
    meta_[key] = std::move(v);
  }
  auto al = meta_.find("general.alignment");
  alignment_ = (al != meta_.end() && al->second.gtype == 4) ? (uint32_t)al->second.u : 32u;
  if (alignment_ == 0 || (alignment_ & (alignment_ - 1)) != 0) {
    err_ = "Invalid alignment: " + std::to_string(alignment_) + " (must be a power of two)";
    return false;
  }
  for (uint64_t i = 0; i < tensor_count; i++) {
    GgufTensor t;
    uint32_t nd;
    std::string e;
    if (!r.str(t.name, e) || !r.get(nd)) { err_ = e.empty() ? trunc : e; return false; }
    if (nd > 8) { err_ = "Too many dimensions: " + std::to_string(nd) + " (max 8)"; return false; }
    t.ne.resize(nd);
    for (uint32_t d = 0; d < nd; d++)
      if (!r.get(t.ne[d])) { err_ = trunc; return false; }
    if (!r.get(t.type) || !r.get(t.offset)) { err_ = trunc; return false; }
    uint64_t block, bpb;
    if (!ggml_block_info(t.type, block, bpb)) { err_ = "Unknown GGML type: " + std::to_string(t.type); return false; }
    uint64_t n = 1;
    bool empty = false;
    for (auto d : t.ne) {
      if (d == 0) { empty = true; break; }
      if (n > UINT64_MAX / d) { err_ = "Dimension product overflow"; return false; }
      n *= d;
    }
    if (empty) {
      t.nbytes = 0;
    } else {
      if (block > 1 && n % block != 0) {
        err_ = "Tensor has " + std::to_string(n) + " elements, not a multiple of block size " +
               std::to_string(block) + " for GGML type " + std::to_string(t.type);
        return false;
      }
      if (n / block > UINT64_MAX / bpb) { err_ = "Tensor size overflow"; return false; }
      t.nbytes = n / block * bpb;
    }
    if (by_name_.count(t.name)) { err_ = "Duplicate tensor name: " + t.name; return false; }
    by_name_[t.name] = tensors_.size();
    tensors_.push_back(std::move(t));
  }
  uint64_t pos = r.position();
  data_offset_ = (pos + alignment_ - 1) / alignment_ * alignment_;
  if (data_offset_ > file_len_) {
    err_ = "Data offset " + std::to_string(data_offset_) + " exceeds file length " + std::to_string(file_len_);
    return false;
  }
  uint64_t data_size = file_len_ - data_offset_;
  for (auto& t : tensors_) {
    if (t.offset > data_size) {
      err_ = "Tensor \"" + t.name + "\" offset " + std::to_string(t.offset) + " exceeds data size " +
             std::to_string(data_size);
      return false;
    }
    if (t.offset + t.nbytes < t.offset) { err_ = "Tensor \"" + t.name + "\" offset+nbytes overflow"; return false; }
    if (t.offset + t.nbytes > data_size) {
      err_ = "Tensor \"" + t.name + "\" end " + std::to_string(t.offset + t.nbytes) + " exceeds data size " +
             std::to_string(data_size);
      return false;
    }
    t.offset += data_offset_;
  }
  return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = by_name_.find(name);
  return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

bool GgufFile::meta_u32(const std::string& key, uint32_t& out) const {
  auto it = meta_.find(key);
  if (it == meta_.end()) return false;
  const GgufValue& v = it->second;
  // model_file.rs:131-140 accepts U32, U64, I32, I64, U8.
  switch (v.gtype) {
    case 4: case 10: case 0: out = (uint32_t)v.u; return true;
    case 5: case 11: out = (uint32_t)v.i; return true;
    default: return false;
  }
}

uint32_t GgufFile::meta_u32_default(const std::string& key, uint32_t def) const {
  uint32_t v;
  return meta_u32(key, v) ? v : def;
}

bool GgufFile::meta_f32(const std::string& key, float& out) const {
  auto it = meta_.find(key);
  if (it == meta_.end() || it->second.kind != GgufValue::FLOAT) return false;
  out = (float)it->second.f;
  return true;
}

bool GgufFile::meta_u32_array(const std::string& key, std::vector<uint32_t>& out) const {
  auto it = meta_.find(key);
  if (it == meta_.end() || it->second.kind != GgufValue::ARRAY) return false;
  out.clear();
  for (auto& v : it->second.arr) {
    // model_file.rs:166-182: U32, I32, U16, I16, U8, I8 elements.
    switch (v.gtype) {
      case 4: case 2: case 0: out.push_back((uint32_t)v.u); break;
      case 5: case 3: case 1: out.push_back((uint32_t)v.i); break;
      default: return false;
    }
  }
  return true;
}

bool GgufFile::meta_str(const std::string& key, std::string& out) const {
  auto it = meta_.find(key);
  if (it == meta_.end() || it->second.kind != GgufValue::STRING) return false;
  out = it->second.s;
  return true;
}

bool GgufFile::read(const GgufTensor& t, uint64_t off, uint64_t len, void* dst) const {
  if (off + len > t.nbytes) return false;
  uint8_t* d = (uint8_t*)dst;
  uint64_t pos = t.offset + off;
  while (len) {
    ssize_t r = pread(fd_, d, len > (1ull << 30) ? (1ull << 30) : len, (off_t)pos);
    if (r <= 0) return false;
    d += r;
    pos += (uint64_t)r;
    len -= (uint64_t)r;
  }
  return true;
}

}  // namespace lfm
