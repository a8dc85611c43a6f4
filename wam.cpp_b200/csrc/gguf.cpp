#include "gguf.h"

#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

namespace wamb {

namespace {

enum : uint32_t {
  GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6,
  GT_BOOL = 7, GT_STR = 8, GT_ARR = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12,
};

class Cursor {
 public:
  explicit Cursor(FILE* f) : f_(f) {}
  bool bytes(void* dst, size_t n) {
    if (n && std::fread(dst, 1, n, f_) != n) return false;
    pos_ += n;
    return true;
  }
  template <class T>
  bool pod(T* v) {
    return bytes(v, sizeof(T));
  }
  bool str(std::string* s) {
    uint64_t n = 0;
    if (!pod(&n) || n > (1ull << 30)) return false;
    s->resize(n);
    return bytes(&(*s)[0], n);
  }
  bool skip(uint64_t n) {
    if (std::fseek(f_, static_cast<long>(n), SEEK_CUR) != 0) return false;
    pos_ += n;
    return true;
  }
  uint64_t pos() const { return pos_; }

 private:
  FILE* f_;
  uint64_t pos_ = 0;
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t t, GgufValue* v) {
  uint8_t b[8] = {0};
  const size_t n = scalar_size(t);
  if (!n || !c.bytes(b, n)) return false;
  switch (t) {
    case GT_U8: case GT_BOOL: v->u = b[0]; v->i = b[0]; v->f = b[0]; break;
    case GT_I8: v->i = static_cast<int8_t>(b[0]); v->u = v->i; v->f = v->i; break;
    case GT_U16: { uint16_t x; std::memcpy(&x, b, 2); v->u = x; v->i = x; v->f = x; break; }
    case GT_I16: { int16_t x; std::memcpy(&x, b, 2); v->i = x; v->u = x; v->f = x; break; }
    case GT_U32: { uint32_t x; std::memcpy(&x, b, 4); v->u = x; v->i = x; v->f = x; break; }
    case GT_I32: { int32_t x; std::memcpy(&x, b, 4); v->i = x; v->u = x; v->f = x; break; }
    case GT_F32: { float x; std::memcpy(&x, b, 4); v->f = x; break; }
    case GT_U64: { uint64_t x; std::memcpy(&x, b, 8); v->u = x; v->i = static_cast<int64_t>(x); v->f = static_cast<double>(x); break; }
    case GT_I64: { int64_t x; std::memcpy(&x, b, 8); v->i = x; v->u = x; v->f = static_cast<double>(x); break; }
    case GT_F64: { double x; std::memcpy(&x, b, 8); v->f = x; break; }
    default: return false;
  }
  return true;
}

}  // namespace

uint64_t ggml_type_bytes(uint32_t type, uint64_t n) {
  switch (type) {
    case GGML_F32: return n * 4;
    case GGML_F16: case GGML_BF16: return n * 2;
    case GGML_Q8_0: return (n % 32) ? 0 : (n / 32) * 34;
    default: return 0;
  }
}

bool GgufFile::open(const std::string& path, std::string* error) {
  path_ = path;
  struct stat st;
  if (::stat(path.c_str(), &st) != 0) {
    *error = "cannot stat artifact " + path;
    return false;
  }
  file_size_ = static_cast<uint64_t>(st.st_size);
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    *error = "cannot open artifact " + path;
    return false;
  }
  Cursor c(f);
  auto fail = [&](const std::string& m) {
    std::fclose(f);
    *error = "GGUF " + path + ": " + m;
    return false;
  };
  char magic[4];
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!c.bytes(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return fail("bad magic");
  if (!c.pod(&version) || (version != 2 && version != 3)) return fail("unsupported version");
  if (!c.pod(&n_tensors) || !c.pod(&n_kv) || n_tensors > (1u << 24) || n_kv > (1u << 24))
    return fail("truncated header");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    GgufValue v;
    if (!c.str(&key) || !c.pod(&v.type)) return fail("truncated metadata");
    if (v.type == GT_STR) {
      if (!c.str(&v.s)) return fail("truncated string value");
    } else if (v.type == GT_ARR) {
      uint32_t et = 0;
      uint64_t n = 0;
      if (!c.pod(&et) || !c.pod(&n)) return fail("truncated array");
      if (et == GT_STR) {
        for (uint64_t j = 0; j < n; ++j) {
          std::string s;
          if (!c.str(&s)) return fail("truncated string array");
        }
      } else {
        const size_t es = scalar_size(et);
        if (!es) return fail("bad array element type");
        if (n <= 4096) {
          for (uint64_t j = 0; j < n; ++j) {
            GgufValue e;
            if (!read_scalar(c, et, &e)) return fail("truncated array");
            v.arr.push_back(e.f);
          }
        } else if (!c.skip(n * es)) {
          return fail("truncated array");
        }
      }
    } else if (!read_scalar(c, v.type, &v)) {
      return fail("bad metadata value for " + key);
    }
    kv_[key] = v;
  }
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    uint32_t nd = 0;
    if (!c.str(&t.name) || !c.pod(&nd) || nd == 0 || nd > 4) return fail("bad tensor descriptor");
    t.ne.resize(nd);
    for (uint32_t d = 0; d < nd; ++d)
      if (!c.pod(&t.ne[d])) return fail("truncated tensor descriptor");
    if (!c.pod(&t.type) || !c.pod(&t.offset)) return fail("truncated tensor descriptor");
    t.bytes = ggml_type_bytes(t.type, t.elements());
    index_[t.name] = tensors_.size();
    tensors_.push_back(t);
  }
  uint64_t align = 32;
  if (has("general.alignment")) align = kv_["general.alignment"].u;
  if (align == 0 || (align & (align - 1))) return fail("bad alignment");
  const uint64_t data = (c.pos() + align - 1) / align * align;
  for (GgufTensor& t : tensors_) {
    t.offset += data;
    if (t.bytes && t.offset + t.bytes > file_size_) return fail("tensor " + t.name + " is truncated");
  }
  std::fclose(f);
  return true;
}

bool GgufFile::get_u32(const std::string& key, uint32_t* out) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return false;
  *out = static_cast<uint32_t>(it->second.u);
  return true;
}

bool GgufFile::get_f32(const std::string& key, float* out) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return false;
  *out = static_cast<float>(it->second.f);
  return true;
}

bool GgufFile::get_f32_array(const std::string& key, std::vector<float>* out) const {
  auto it = kv_.find(key);
  if (it == kv_.end() || it->second.type != GT_ARR) return false;
  out->assign(it->second.arr.begin(), it->second.arr.end());
  return true;
}

bool GgufFile::get_str(const std::string& key, std::string* out) const {
  auto it = kv_.find(key);
  if (it == kv_.end() || it->second.type != GT_STR) return false;
  *out = it->second.s;
  return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

bool GgufFile::read(const GgufTensor& t, uint64_t start, void* dst, uint64_t bytes) const {
  if (start + bytes > t.bytes) return false;
  const int fd = ::open(path_.c_str(), O_RDONLY);
  if (fd < 0) return false;
  uint8_t* p = static_cast<uint8_t*>(dst);
  uint64_t off = t.offset + start, left = bytes;
  while (left) {
    const ssize_t r = ::pread(fd, p, left > (1u << 30) ? (1u << 30) : left, static_cast<off_t>(off));
    if (r <= 0) {
      ::close(fd);
      return false;
    }
    p += r;
    off += static_cast<uint64_t>(r);
    left -= static_cast<uint64_t>(r);
  }
  ::close(fd);
  return true;
}

}  // namespace wamb
