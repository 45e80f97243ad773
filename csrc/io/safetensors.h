// safetensors reader/writer.
//
// File format (public spec): 8-byte little-endian header length N, then N
// bytes of JSON mapping tensor name -> {"dtype", "shape", "data_offsets":
// [begin, end]} (offsets relative to the end of the header), plus an optional
// "__metadata__" object of string pairs; then the raw tensor bytes.
//
// Writing is done in Python (mod_b200/io/safetensors.py).  The reader mmaps the file and returns zero-copy torch views that keep the
// mapping alive; shard slicing (dim, rank, world) returns a view for dim 0 and
// a contiguous copy otherwise, so a tensor-/expert-parallel rank touches only
// its slice.  The reference's loader (pio/plugins/cpu/c_src/safetensors_loader.c)
// finds names with strstr, decodes BF16 as F16 and has no shape checks.
#pragma once
#include <torch/extension.h>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace mbio {

struct TensorInfo {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
};

class Mapping;

class SafeTensorsFile {
 public:
  explicit SafeTensorsFile(const std::string& path);
  std::vector<std::string> keys() const;
  std::map<std::string, std::string> metadata() const { return meta_; }
  const TensorInfo& info(const std::string& name) const;
  at::Tensor get(const std::string& name) const;
  at::Tensor get_slice(const std::string& name, int64_t dim, int64_t rank, int64_t world) const;
  std::string path() const { return path_; }

 private:
  std::string path_;
  std::shared_ptr<Mapping> map_;
  std::map<std::string, TensorInfo> tensors_;
  std::map<std::string, std::string> meta_;
  size_t data_start_ = 0;
};

std::map<std::string, TensorInfo> read_header(const std::string& path);

void bind(pybind11::module& m);

}  // namespace mbio
