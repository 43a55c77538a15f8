// PGW1 container parsing for the CUDA backend (engine/weights.js:5-40).
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mllm {

struct PgwTensor {
  std::string name;
  std::vector<int64_t> shape;
  std::string storage;  // "q4", "f32", ...
  int group = 32;
  int64_t offset = 0, nbytes = 0, scale_offset = 0, scale_nbytes = 0;
};

struct PgwModel {
  int arch = 0;  // 0 llama, 1 gpt2 (header byte 5; engine/weights.js:15-16, 36-38)
  std::string kind;
  int vocab = 0, n_layers = 0, d_model = 0, n_heads = 0, n_kv_heads = 0, d_ff = 0, max_seq = 0, q_group = 32;
  double rope_theta = 10000.0, rope_pct = 1.0;
  int64_t payload_off = 0;
  std::map<std::string, PgwTensor> tensors;
};

// Parses the header and JSON tensor table of `buf`; returns false with a message in `err`.
bool parse_pgw(const uint8_t* buf, size_t len, PgwModel* out, std::string* err);

}  // namespace mllm
