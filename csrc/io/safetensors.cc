#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace mbio {

// ------------------------------------------------------------------ mmap
class Mapping {
 public:
  explicit Mapping(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("safetensors: cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) throw std::runtime_error("safetensors: cannot stat " + path);
    size_ = (size_t)st.st_size;
    if (size_ > 0) {
      base_ = ::mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd_, 0);
      if (base_ == MAP_FAILED) {
        base_ = nullptr;
        throw std::runtime_error("safetensors: mmap failed for " + path);
      }
      ::madvise(base_, size_, MADV_WILLNEED);
    }
  }
  ~Mapping() {
    if (base_) ::munmap(base_, size_);
    if (fd_ >= 0) ::close(fd_);
  }
  const uint8_t* data() const { return static_cast<const uint8_t*>(base_); }
  size_t size() const { return size_; }

 private:
  int fd_ = -1;
  void* base_ = nullptr;
  size_t size_ = 0;
};

// ------------------------------------------------------------------ JSON
// Recursive-descent parser for the subset a header uses: objects, arrays,
// strings (with escapes) and integers.  Anything else is rejected.
struct J {
  enum K { OBJ, ARR, STR, NUM } k = NUM;
  std::map<std::string, J> o;
  std::vector<J> a;
  std::string s;
  int64_t n = 0;
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), e_(p + n) {}
  J parse() {
    J v = value(0);
    ws();
    if (p_ != e_) fail("trailing data");
    return v;
  }

 private:
  const char *p_, *e_;
  [[noreturn]] void fail(const char* m) { throw std::runtime_error(std::string("safetensors header: ") + m); }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  char peek() {
    ws();
    if (p_ >= e_) fail("unexpected end");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) fail("unexpected character");
    ++p_;
  }
  J value(int depth) {
    if (depth > 16) fail("nesting too deep");
    char c = peek();
    if (c == '{') return object(depth);
    if (c == '[') return array(depth);
    if (c == '"') {
      J j;
      j.k = J::STR;
      j.s = str();
      return j;
    }
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    fail("unsupported value");
  }
  std::string str() {
    expect('"');
    std::string out;
    while (true) {
      if (p_ >= e_) fail("unterminated string");
      char c = *p_++;
      if (c == '"') break;
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= e_) fail("bad escape");
      char x = *p_++;
      switch (x) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'n': out += '\n'; break;
        case 't': out += '\t'; break;
        case 'r': out += '\r'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'u': {
          if (e_ - p_ < 4) fail("bad unicode escape");
          unsigned cp = 0;
          for (int i = 0; i < 4; ++i) {
            char h = p_[i];
            cp <<= 4;
            if (h >= '0' && h <= '9') cp |= h - '0';
            else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
            else fail("bad unicode escape");
          }
          p_ += 4;
          if (cp < 0x80) out += (char)cp;
          else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
          else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  J number() {
    J j;
    j.k = J::NUM;
    const char* s = p_;
    if (*p_ == '-') ++p_;
    const char* digits = p_;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    if (p_ == digits || p_ - digits > 18) fail("bad integer");
    if (p_ < e_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) fail("non-integer number");
    j.n = std::stoll(std::string(s, p_ - s));
    return j;
  }
  J object(int depth) {
    J j;
    j.k = J::OBJ;
    expect('{');
    if (peek() == '}') { ++p_; return j; }
    while (true) {
      std::string key = str();
      expect(':');
      j.o.emplace(key, value(depth + 1));
      char c = peek();
      ++p_;
      if (c == '}') break;
      if (c != ',') fail("expected , or }");
    }
    return j;
  }
  J array(int depth) {
    J j;
    j.k = J::ARR;
    expect('[');
    if (peek() == ']') { ++p_; return j; }
    while (true) {
      j.a.push_back(value(depth + 1));
      char c = peek();
      ++p_;
      if (c == ']') break;
      if (c != ',') fail("expected , or ]");
    }
    return j;
  }
};

static int64_t dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  throw std::runtime_error("safetensors: unsupported dtype " + d);
}

static at::ScalarType to_torch(const std::string& d) {
  if (d == "F64") return at::kDouble;
  if (d == "F32") return at::kFloat;
  if (d == "F16") return at::kHalf;
  if (d == "BF16") return at::kBFloat16;
  if (d == "I64") return at::kLong;
  if (d == "I32") return at::kInt;
  if (d == "I16") return at::kShort;
  if (d == "I8") return at::kChar;
  if (d == "U8") return at::kByte;
  if (d == "BOOL") return at::kBool;
  if (d == "F8_E4M3") return at::kFloat8_e4m3fn;
  if (d == "F8_E5M2") return at::kFloat8_e5m2;
  throw std::runtime_error("safetensors: unsupported dtype " + d);
}

[[maybe_unused]] static std::string from_torch(at::ScalarType t) {
  switch (t) {
    case at::kDouble: return "F64";
    case at::kFloat: return "F32";
    case at::kHalf: return "F16";
    case at::kBFloat16: return "BF16";
    case at::kLong: return "I64";
    case at::kInt: return "I32";
    case at::kShort: return "I16";
    case at::kChar: return "I8";
    case at::kByte: return "U8";
    case at::kBool: return "BOOL";
    case at::kFloat8_e4m3fn: return "F8_E4M3";
    case at::kFloat8_e5m2: return "F8_E5M2";
    default: throw std::runtime_error("safetensors: unsupported torch dtype");
  }
}

static void parse_header(const char* p, size_t n, size_t data_bytes, std::map<std::string, TensorInfo>& out,
                         std::map<std::string, std::string>& meta) {
  J root = Parser(p, n).parse();
  if (root.k != J::OBJ) throw std::runtime_error("safetensors header: not an object");
  for (auto& kv : root.o) {
    if (kv.first == "__metadata__") {
      if (kv.second.k != J::OBJ) throw std::runtime_error("safetensors header: bad __metadata__");
      for (auto& m : kv.second.o) {
        if (m.second.k != J::STR) throw std::runtime_error("safetensors header: metadata values must be strings");
        meta[m.first] = m.second.s;
      }
      continue;
    }
    const J& t = kv.second;
    if (t.k != J::OBJ || !t.o.count("dtype") || !t.o.count("shape") || !t.o.count("data_offsets") ||
        t.o.at("dtype").k != J::STR || t.o.at("shape").k != J::ARR || t.o.at("data_offsets").k != J::ARR)
      throw std::runtime_error("safetensors header: incomplete entry " + kv.first);
    TensorInfo info;
    info.dtype = t.o.at("dtype").s;
    int64_t numel = 1;
    for (auto& d : t.o.at("shape").a) {
      if (d.k != J::NUM || d.n < 0) throw std::runtime_error("safetensors header: bad shape for " + kv.first);
      info.shape.push_back(d.n);
      numel *= d.n;
    }
    const auto& off = t.o.at("data_offsets").a;
    if (off.size() != 2 || off[0].k != J::NUM || off[1].k != J::NUM)
      throw std::runtime_error("safetensors header: bad data_offsets for " + kv.first);
    info.begin = off[0].n;
    info.end = off[1].n;
    if (info.begin < 0 || info.end < info.begin || (size_t)info.end > data_bytes)
      throw std::runtime_error("safetensors: data_offsets out of range for " + kv.first);
    if (info.end - info.begin != numel * dtype_size(info.dtype))
      throw std::runtime_error("safetensors: byte size does not match shape for " + kv.first);
    out[kv.first] = info;
  }
}

SafeTensorsFile::SafeTensorsFile(const std::string& path) : path_(path), map_(std::make_shared<Mapping>(path)) {
  if (map_->size() < 8) throw std::runtime_error("safetensors: file too small: " + path);
  uint64_t n = 0;
  std::memcpy(&n, map_->data(), 8);
  if (n > map_->size() - 8 || n > (100ull << 20)) throw std::runtime_error("safetensors: bad header length in " + path);
  data_start_ = 8 + n;
  parse_header(reinterpret_cast<const char*>(map_->data() + 8), n, map_->size() - data_start_, tensors_, meta_);
}

std::vector<std::string> SafeTensorsFile::keys() const {
  std::vector<std::string> k;
  for (auto& kv : tensors_) k.push_back(kv.first);
  return k;
}

const TensorInfo& SafeTensorsFile::info(const std::string& name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw std::out_of_range("safetensors: no tensor named " + name);
  return it->second;
}

at::Tensor SafeTensorsFile::get(const std::string& name) const {
  const TensorInfo& ti = info(name);
  void* ptr = const_cast<uint8_t*>(map_->data() + data_start_ + ti.begin);
  auto keep = map_;  // the view keeps the mapping alive
  return torch::from_blob(ptr, ti.shape, [keep](void*) {}, at::TensorOptions().dtype(to_torch(ti.dtype)));
}

at::Tensor SafeTensorsFile::get_slice(const std::string& name, int64_t dim, int64_t rank, int64_t world) const {
  at::Tensor t = get(name);
  if (world <= 1) return t;
  if (dim < 0) dim += t.dim();
  TORCH_CHECK(dim >= 0 && dim < t.dim(), "get_slice: bad dim");
  TORCH_CHECK(rank >= 0 && rank < world, "get_slice: bad rank");
  const int64_t n = t.size(dim);
  if (n % world != 0)
    throw std::invalid_argument("get_slice: dim " + std::to_string(dim) + " of " + name + " (" + std::to_string(n) +
                                ") is not divisible by " + std::to_string(world));
  const int64_t part = n / world;
  at::Tensor s = t.narrow(dim, rank * part, part);
  return dim == 0 ? s : s.contiguous();
}

std::map<std::string, TensorInfo> read_header(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("safetensors: cannot open " + path);
  f.seekg(0, std::ios::end);
  const size_t size = f.tellg();
  f.seekg(0);
  uint64_t n = 0;
  if (size < 8 || !f.read(reinterpret_cast<char*>(&n), 8)) throw std::runtime_error("safetensors: file too small");
  if (n > size - 8 || n > (100ull << 20)) throw std::runtime_error("safetensors: bad header length");
  std::string hdr(n, '\0');
  f.read(&hdr[0], n);
  std::map<std::string, TensorInfo> out;
  std::map<std::string, std::string> meta;
  parse_header(hdr.data(), n, size - 8 - n, out, meta);
  return out;
}

void bind(pybind11::module& m) {
  namespace py = pybind11;
  py::class_<SafeTensorsFile>(m, "SafeTensorsFile")
      .def(py::init<const std::string&>())
      .def("keys", &SafeTensorsFile::keys)
      .def("metadata", &SafeTensorsFile::metadata)
      .def("get", &SafeTensorsFile::get)
      .def("get_slice", &SafeTensorsFile::get_slice)
      .def("shape", [](const SafeTensorsFile& f, const std::string& n) { return f.info(n).shape; })
      .def("dtype", [](const SafeTensorsFile& f, const std::string& n) { return f.info(n).dtype; })
      .def_property_readonly("path", &SafeTensorsFile::path);
  m.def("read_header", [](const std::string& p) {
    py::dict d;
    for (auto& kv : read_header(p)) {
      py::dict e;
      e["dtype"] = kv.second.dtype;
      e["shape"] = kv.second.shape;
      e["data_offsets"] = py::make_tuple(kv.second.begin, kv.second.end);
      d[py::str(kv.first)] = e;
    }
    return d;
  });
}

}  // namespace mbio
