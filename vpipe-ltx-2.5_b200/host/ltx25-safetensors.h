// ltx25-safetensors.h -- the on-disk checkpoint reader: a safetensors file
// mapped read-only, its JSON header parsed once.  The reference reads the
// same files through its WeightSet (src/ltx25-dit-weights.cc:230-403,
// src/ltx25-lora.cc:180-300); the format is: u64 little-endian header length,
// the JSON header {name: {"dtype", "shape", "data_offsets": [begin, end]},
// "__metadata__": {key: string}}, then the data, offsets relative to it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ltx25 {

enum StDtype : int {
  ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2, ST_U32 = 3, ST_I32 = 4, ST_U8 = 5,
  ST_I8 = 6, ST_F64 = 7, ST_I64 = 8, ST_U16 = 9, ST_I16 = 10, ST_BOOL = 11,
};

// A header whose tensor has more dimensions than this is refused (the C
// ABI's ltx_st_info hands a shape back in 8 slots).
constexpr int kStMaxDims = 8;

struct StTensor {
  std::string name;
  int dtype = 0;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  uint64_t bytes = 0;
};

class SafeTensors {
public:
  ~SafeTensors();
  // Map and parse `path`.  Refuses a header that is not the format's
  // (unknown dtype, offsets outside the data or disagreeing with the
  // shape, a truncated file) rather than binding part of it.
  bool open(const std::string& path, std::string* err);
  // Parse an in-memory image of a file (the same checks).
  bool parse(const uint8_t* base, size_t size, std::string* err);

  int count() const { return (int)_tensors.size(); }
  const StTensor& at(int i) const { return _tensors[(size_t)i]; }
  // index of `name`, or -1
  int find(const std::string& name) const;
  // a __metadata__ value, or nullptr
  const std::string* metadata(const std::string& key) const;

  // Element size of a dtype, 0 if unknown.
  static size_t elem_size(int dtype);
  // A float tensor (F32 / F16 / BF16) as f32, `n` elements from element
  // `off`; false for other dtypes or a range past the tensor.
  static bool to_f32(const StTensor& t, size_t off, size_t n, float* out);
  // The same as bf16 bits (f32 rounded to nearest even; F16 through f32).
  static bool to_bf16(const StTensor& t, size_t off, size_t n, uint16_t* out);

private:
  std::vector<StTensor> _tensors;
  std::map<std::string, int> _index;
  std::map<std::string, std::string> _meta;
  void* _map = nullptr;
  size_t _map_bytes = 0;
};

}  // namespace ltx25
