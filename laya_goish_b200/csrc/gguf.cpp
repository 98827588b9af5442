// GGUF v3 reader (restates src/gguf.rs:22-180 and src/io.rs:56-97).
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace laya {

bool ggml_layout(uint32_t kind, int* block, int* size) {
  switch (kind) {
    case 0: *block = 1; *size = 4; return true;
    case 1: *block = 1; *size = 2; return true;
    case 2: *block = 32; *size = 18; return true;
    case 8: *block = 32; *size = 34; return true;
    case 12: *block = 256; *size = 144; return true;
    case 14: *block = 256; *size = 210; return true;
  }
  return false;
}

Gguf::~Gguf() {
  if (map_) munmap(map_, map_len_);
}

// Mapping::open (src/io.rs:65-88): read-only private mapping of the whole file.
std::string Gguf::open_file(const std::string& path) {
  if (path.find('\0') != std::string::npos) return "NUL in path";
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return "open " + path + ": " + std::strerror(errno);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    ::close(fd);
    return "empty/unreadable model";
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) return "mmap failed";
  map_ = p;
  map_len_ = (size_t)st.st_size;
  b_ = static_cast<const uint8_t*>(p);
  n_ = map_len_;
  return parse();
}

std::string Gguf::open_memory(const uint8_t* b, size_t n) {
  b_ = b;
  n_ = n;
  return parse();
}

namespace {
struct Reader {
  const uint8_t* b;
  size_t n, p = 0;
  std::string err;
  // Reader::take (src/gguf.rs:27-32)
  const uint8_t* take(size_t k) {
    if (!err.empty()) return nullptr;
    if (p + k < p) {
      err = "GGUF length overflow";
      return nullptr;
    }
    if (p + k > n) {
      err = "truncated GGUF";
      return nullptr;
    }
    const uint8_t* s = b + p;
    p += k;
    return s;
  }
  bool u32(uint32_t* v) {
    auto s = take(4);
    if (!s) return false;
    std::memcpy(v, s, 4);
    return true;
  }
  bool u64(uint64_t* v) {
    auto s = take(8);
    if (!s) return false;
    std::memcpy(v, s, 8);
    return true;
  }
  static bool utf8(const uint8_t* s, size_t n) {
    size_t i = 0;
    while (i < n) {
      uint8_t c = s[i];
      size_t k;
      uint32_t cp;
      if (c < 0x80) {
        i++;
        continue;
      }
      if ((c & 0xe0) == 0xc0) { k = 1; cp = c & 0x1f; }
      else if ((c & 0xf0) == 0xe0) { k = 2; cp = c & 0x0f; }
      else if ((c & 0xf8) == 0xf0) { k = 3; cp = c & 0x07; }
      else return false;
      if (i + k >= n) return false;
      for (size_t j = 1; j <= k; j++) {
        if ((s[i + j] & 0xc0) != 0x80) return false;
        cp = (cp << 6) | (s[i + j] & 0x3f);
      }
      if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) || cp > 0x10ffff ||
          (cp >= 0xd800 && cp <= 0xdfff))
        return false;
      i += k + 1;
    }
    return true;
  }
  // Reader::string (src/gguf.rs:39-47)
  bool string(std::string* out) {
    uint64_t k;
    if (!u64(&k)) return false;
    if (k > 32ull * 1024 * 1024) {
      err = "GGUF string too large";
      return false;
    }
    auto s = take((size_t)k);
    if (!s) return false;
    if (!utf8(s, (size_t)k)) {
      err = "invalid GGUF UTF-8";
      return false;
    }
    if (out) out->assign(reinterpret_cast<const char*>(s), (size_t)k);
    return true;
  }
  // Reader::value (src/gguf.rs:48-79)
  bool value(uint32_t t, int depth, MetaValue* v) {
    if (depth > 4) {
      err = "GGUF metadata nesting too deep";
      return false;
    }
    v->type = t;
    const uint8_t* s;
    switch (t) {
      case 0: if (!(s = take(1))) return false; v->num = s[0]; return true;
      case 1: if (!(s = take(1))) return false; v->num = (int8_t)s[0]; return true;
      case 2: { uint16_t x; if (!(s = take(2))) return false; std::memcpy(&x, s, 2); v->num = x; return true; }
      case 3: { int16_t x; if (!(s = take(2))) return false; std::memcpy(&x, s, 2); v->num = x; return true; }
      case 4: { uint32_t x; if (!u32(&x)) return false; v->num = x; return true; }
      case 5: { uint32_t x; if (!u32(&x)) return false; v->num = (int32_t)x; return true; }
      case 6: { uint32_t x; float f; if (!u32(&x)) return false; std::memcpy(&f, &x, 4); v->num = f; return true; }
      case 7: if (!(s = take(1))) return false; v->num = s[0] != 0; return true;
      case 8: return string(&v->str);
      case 9: {
        uint32_t et;
        uint64_t k;
        if (!u32(&et) || !u64(&k)) return false;
        if (k > 1000000) {
          err = "GGUF array too large";
          return false;
        }
        for (uint64_t i = 0; i < k; i++) {
          MetaValue e;
          if (!value(et, depth + 1, &e)) return false;
        }
        v->num = (double)k;
        return true;
      }
      case 10: { uint64_t x; if (!u64(&x)) return false; v->num = (double)x; return true; }
      case 11: { uint64_t x; if (!u64(&x)) return false; v->num = (double)(int64_t)x; return true; }
      case 12: { uint64_t x; double d; if (!u64(&x)) return false; std::memcpy(&d, &x, 8); v->num = d; return true; }
    }
    err = "unsupported GGUF metadata type " + std::to_string(t);
    return false;
  }
};
}  // namespace

std::string Gguf::parse() {
  Reader r{b_, n_};
  auto magic = r.take(4);
  if (!magic) return r.err;
  if (std::memcmp(magic, "GGUF", 4)) return "not a GGUF file";
  uint32_t ver;
  if (!r.u32(&ver)) return r.err;
  if (ver != 3) return "expected GGUF version 3";
  uint64_t nt, nk;
  if (!r.u64(&nt) || !r.u64(&nk)) return r.err;
  if (nt > 100000 || nk > 100000) return "GGUF table too large";
  for (uint64_t i = 0; i < nk; i++) {
    std::string k;
    uint32_t t;
    MetaValue v;
    if (!r.string(&k) || !r.u32(&t) || !r.value(t, 0, &v)) return r.err;
    if (!meta_.emplace(k, v).second) return "duplicate GGUF metadata key";
  }
  for (uint64_t i = 0; i < nt; i++) {
    std::string name;
    uint32_t nd;
    if (!r.string(&name) || !r.u32(&nd)) return r.err;
    if (nd < 1 || nd > 4) return "invalid tensor rank";
    TensorInfo t;
    uint64_t count = 1;
    for (uint32_t j = 0; j < nd; j++) {
      uint64_t d;
      if (!r.u64(&d)) return r.err;
      if (d == 0) return "empty tensor";
      if (count > UINT64_MAX / d) return "tensor size overflow";
      count *= d;
      t.dims.push_back(d);
    }
    if (!r.u32(&t.kind) || !r.u64(&t.offset)) return r.err;
    int block, size;
    if (!ggml_layout(t.kind, &block, &size))
      return "unsupported GGML tensor type " + std::to_string(t.kind) + "; supported F32/F16/Q4_0/Q8_0/Q4_K/Q6_K";
    if (t.dims[0] % (uint64_t)block) return "invalid quantized row alignment";
    if (count / (uint64_t)block > UINT64_MAX / (uint64_t)size) return "tensor byte size overflow";
    t.len = count / (uint64_t)block * (uint64_t)size;
    if (!tensors_.emplace(name, t).second) return "duplicate tensor";
  }
  uint64_t align = 32;
  if (auto a = meta("general.alignment")) align = (uint64_t)a->num;
  if (align == 0 || (align & (align - 1)) || align > 4096) return "invalid GGUF alignment";
  const uint64_t base = ((uint64_t)r.p + align - 1) & ~(align - 1);
  for (auto& kv : tensors_) {
    TensorInfo& t = kv.second;
    if (t.offset % align) return "unaligned GGUF tensor";
    if (t.offset + base < t.offset) return "offset overflow";
    t.offset += base;
    if (t.offset + t.len < t.offset) return "length overflow";
    if (t.offset + t.len > n_) return "truncated tensor data";
  }
  return "";
}

}  // namespace laya
