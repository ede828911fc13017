// GGUF v3 reader for the engine's weight load.
//
// Validation follows the reference parser (parser/src/gguf.rs:304-440): magic
// "GGUF", version 3, tensor/KV counts <= 100000, no duplicate keys or tensor
// names, power-of-two general.alignment (default 32), at most 8 dimensions,
// known GGML block sizes (gguf.rs:174-192), element counts that are a multiple
// of the block size, arrays of at most 10M elements stored as (type, count),
// BOOL values 0/1, and every tensor range inside the file.
// Typed metadata access mirrors engine/src/model_file.rs:131-182.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace lfm {

struct GgufValue {
  enum Kind { UINT, INT, FLOAT, BOOL, STRING, ARRAY } kind = UINT;
  uint32_t gtype = 0;  // GGUF value type id
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  std::vector<GgufValue> arr;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> ne;  // ne[0] fastest
  uint32_t type = 0;         // 0 = F32, 14 = Q6_K
  uint64_t offset = 0;       // absolute file offset of the payload
  uint64_t nbytes = 0;
};

class GgufFile {
 public:
  // Parses the header; returns false and sets err() on any violation.
  bool open(const std::string& path);
  ~GgufFile();

  const std::string& err() const { return err_; }
  const GgufTensor* tensor(const std::string& name) const;
  const std::vector<GgufTensor>& tensors() const { return tensors_; }

  // model_file.rs:131-182
  bool meta_u32(const std::string& key, uint32_t& out) const;
  uint32_t meta_u32_default(const std::string& key, uint32_t def) const;
  bool meta_f32(const std::string& key, float& out) const;
  bool meta_u32_array(const std::string& key, std::vector<uint32_t>& out) const;
  bool meta_str(const std::string& key, std::string& out) const;

  // pread of a payload range (model_file.rs:100-109)
  bool read(const GgufTensor& t, uint64_t off, uint64_t len, void* dst) const;

  uint64_t data_offset() const { return data_offset_; }
  uint32_t alignment() const { return alignment_; }

 private:
  int fd_ = -1;
  uint64_t file_len_ = 0, data_offset_ = 0;
  uint32_t alignment_ = 32;
  std::string err_;
  std::map<std::string, GgufValue> meta_;
  std::vector<GgufTensor> tensors_;
  std::map<std::string, size_t> by_name_;
};

// (block_size, bytes_per_block) for a GGML type (parser/src/gguf.rs:174-192).
bool ggml_block_info(uint32_t type, uint64_t& block, uint64_t& bytes);

}  // namespace lfm
