// GGUF v3 reader of the host engine: a C++ restatement of the reference
// loader Gguf::open (src/gguf.rs:95-180) over a read-only mapping
// (src/io.rs:56-97).  Tensor bytes stay in the mapping until they are
// transcoded and uploaded to HBM.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace laya {

struct MetaValue {
  uint32_t type = 0;
  double num = 0;   // scalars (and array length for arrays)
  std::string str;  // strings
};

struct TensorInfo {
  std::vector<uint64_t> dims;
  uint32_t kind = 0;
  uint64_t offset = 0;  // absolute, from the start of the file
  uint64_t len = 0;     // bytes
  uint64_t count() const {
    uint64_t c = 1;
    for (auto d : dims) c *= d;
    return c;
  }
};

// (block elements, block bytes) per GGML type (src/gguf.rs:81-93); false if unsupported.
bool ggml_layout(uint32_t kind, int* block, int* size);

class Gguf {
 public:
  ~Gguf();
  // Maps a file read-only; "" on success, else the error message.
  std::string open_file(const std::string& path);
  // Parses an image the caller keeps alive while this object is used.
  std::string open_memory(const uint8_t* b, size_t n);

  const uint8_t* bytes() const { return b_; }
  size_t size() const { return n_; }
  const MetaValue* meta(const std::string& k) const {
    auto it = meta_.find(k);
    return it == meta_.end() ? nullptr : &it->second;
  }
  double num(const std::string& k, double def) const {
    auto m = meta(k);
    return m ? m->num : def;
  }
  std::string str(const std::string& k) const {
    auto m = meta(k);
    return m ? m->str : std::string();
  }
  const TensorInfo* tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
  }
  const uint8_t* data(const TensorInfo& t) const { return b_ + t.offset; }
  const std::map<std::string, TensorInfo>& tensors() const { return tensors_; }

 private:
  std::string parse();
  const uint8_t* b_ = nullptr;
  size_t n_ = 0;
  void* map_ = nullptr;
  size_t map_len_ = 0;
  std::map<std::string, MetaValue> meta_;
  std::map<std::string, TensorInfo> tensors_;
};

}  // namespace laya
