// Host-side readers for the formats the runtime consumes: config.json,
// safetensors checkpoints (single or sharded), .qpack containers and the
// synthetic checkpoint description. No CUDA here.
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace swl {

// ---------------------------------------------------------------- JSON ----
struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  static Json parse(const std::string& text);
  const Json* find(const std::string& k) const;
  bool is_int() const;
};

std::string read_text_file(const std::string& path);
bool path_exists(const std::string& path);

// -------------------------------------------------------------- config ----
// Mirrors QwenConfig (Sources/SwiftletCore/QwenConfig.swift:51-115) field for
// field, including its defaults and the qwen3_5 / qwen3_next layout rule.
struct ModelConfig {
  std::string model_type;
  int hidden = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0;
  double partial_rotary = 0.25, rope_theta = 1e7, eps = 1e-6;
  int vocab = 0;
  bool tie_embed = false;
  int full_attn_interval = 4;
  int nv = 0, nk = 0, dk = 0, dv = 0, conv_k = 4;
  int experts = 0, topk = 0, moe_inter = 0, shared_inter = 0;
  bool norm_topk = false;
  bool split_layout = false;  // qwen3_5 in_proj_qkv/z/b/a vs qwen3_next in_proj_qkvz/ba
  std::string prefix;         // "" or "language_model."

  bool is_linear(int i) const { return (i + 1) % full_attn_interval != 0; }
  int key_dim() const { return nk * dk; }
  int value_dim() const { return nv * dv; }
  int conv_dim() const { return 2 * key_dim() + value_dim(); }
  int rot_dims() const { return int(double(head_dim) * partial_rotary); }

  void parse(const Json& top);
};

// Default quantisation + per-module overrides, matched by suffix in either
// direction (Checkpoint.swift:31-49, :126-133). Overrides are tried in key
// order so the choice is deterministic.
struct QuantTable {
  bool has_default = false;
  int def_bits = 0, def_gs = 0;
  std::vector<std::pair<std::string, std::pair<int, int>>> overrides;  // key -> (bits, gs)
  void parse(const Json& top);
  bool lookup(const std::string& path, int& bits, int& gs) const;
};

// ---------------------------------------------------------- safetensors ----
struct TensorMeta {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t numel() const { int64_t n = 1; for (auto d : shape) n *= d; return n; }
};

struct MappedFile {
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t size = 0;
  explicit MappedFile(const std::string& path);
  ~MappedFile();
};

struct SafetensorsFile {
  std::unique_ptr<MappedFile> map;
  size_t data_start = 0;
  std::map<std::string, std::pair<TensorMeta, std::pair<int64_t, int64_t>>> tensors;
  explicit SafetensorsFile(const std::string& path);
};

// A checkpoint directory (mlx-lm layout, single or sharded) with the
// "language_model." prefix resolution of Checkpoint.swift:75-79.
struct CheckpointFiles {
  std::vector<std::unique_ptr<SafetensorsFile>> files;
  std::map<std::string, int> where;
  explicit CheckpointFiles(const std::string& dir);
  std::string resolve(const std::string& name) const;
  bool has(const std::string& name) const { return where.count(resolve(name)) > 0; }
  TensorMeta meta(const std::string& name) const;
  const uint8_t* data(const std::string& name, size_t* nbytes) const;
};

// ---------------------------------------------------------------- qpack ----
// packed_experts/layout.json of a .qpack container (Qpack.swift:22-46).
struct QpackSection {
  std::string name, dtype;
  std::vector<int64_t> shape;
  int64_t offset = 0, size = 0;
};
struct QpackLayout {
  int expert_count = 0, layer_count = 0;
  int64_t stride = 0;
  std::vector<QpackSection> sections;
  int quant_bits = 0, quant_group = 0;  // from manifest.json
  void load(const std::string& container_dir);
  const QpackSection* find(const std::string& name) const;
};

int dtype_code(const std::string& dt);         // F32/BF16/F16 -> DType
int64_t dtype_size(const std::string& dt);

}  // namespace swl
