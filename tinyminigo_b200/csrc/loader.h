// Host-side parsing helpers (no CUDA).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <utility>
#include <vector>

#include "../../include/tmg_cuda.h"

namespace tmg {

struct Json {
  enum Type { Null, Bool, Num, Str, Arr, Obj } type = Null;
  bool b = false;
  double num = 0.0;
  bool is_uint = false;  // a non-negative integer literal (serde_json's as_u64)
  uint64_t u = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const;
};

bool json_parse(const char* text, size_t n, Json& out, std::string& err);
bool config_from_json(const Json& cfg, tmg_config* out, std::string& err);
bool read_file(const std::string& path, std::string& out, std::string& err);

struct StTensor {
  std::string name;
  int dtype = 0;  // 0 F32, 1 BF16, 2 F16
  std::vector<int64_t> shape;
  int64_t offset = 0;  // absolute file offset of the data
  int64_t nbytes = 0;
};

bool safetensors_parse(const uint8_t* bytes, size_t n, std::vector<StTensor>& out,
                       std::string& err);

// One tensor of a TMB1 file: where its bytes lie in the file (TensorRef,
// src/tmb.rs:28-35).
struct TmbTensor {
  std::string name;
  int64_t offset = 0;  // absolute file offset of the data
  int64_t nbytes = 0;
};

// parse_tmb_header, src/tmb.rs:80-121: magic "TMB1", u64 config length, u32
// tensor count, the config JSON (ModelConfig::from_json), the weights section
// (u64 length, zero padding to 8 bytes, the tensors), then per tensor
// (u32 name length, name, u64 offset, u64 length).  Ranges that fall outside
// the file are errors here (the reference panics on a short header and checks
// tensor ranges when it borrows them, TensorRef::bytes, src/tmb.rs:39-44).
bool tmb_parse(const uint8_t* bytes, size_t n, tmg_config* cfg, std::vector<TmbTensor>& out,
               std::string& err);

struct MappedFile {
  int fd = -1;
  void* base = nullptr;
  size_t size = 0;
  ~MappedFile();
  bool open(const std::string& path, std::string& err);
  const uint8_t* data() const { return static_cast<const uint8_t*>(base); }
};

float f16_to_f32(uint16_t h);

// StdRng restatement (rand 0.10.2: ChaCha12, seed_from_u64 via PCG32;
// StandardUniform f32 = (next_u32 >> 8) * 2^-24): the `r` of
// src/tensor.rs:1204.
void stdrng_uniforms(uint64_t seed, int64_t n, float* out);

}  // namespace tmg
