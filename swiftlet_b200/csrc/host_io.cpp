// Host-side format readers (config.json, safetensors, .qpack layout).
#include "host_io.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

namespace swl {

// ---------------------------------------------------------------- JSON ----
namespace {
struct Reader {
  const char* p;
  const char* end;
  [[noreturn]] void bad() { throw Error(ERR_FORMAT, "malformed JSON"); }
  void skip() { while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p; }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(end - p) >= n && memcmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  std::string string_body() {
    std::string out;
    ++p;  // opening quote
    while (p < end && *p != '"') {
      char c = *p++;
      if (c != '\\') { out.push_back(c); continue; }
      if (p >= end) bad();
      char esc = *p++;
      if (esc == 'u') {
        if (end - p < 4) bad();
        unsigned cp = (unsigned)strtoul(std::string(p, 4).c_str(), nullptr, 16);
        p += 4;
        if (cp < 0x80) out.push_back(char(cp));
        else if (cp < 0x800) { out.push_back(char(0xC0 | (cp >> 6))); out.push_back(char(0x80 | (cp & 0x3F))); }
        else { out.push_back(char(0xE0 | (cp >> 12))); out.push_back(char(0x80 | ((cp >> 6) & 0x3F))); out.push_back(char(0x80 | (cp & 0x3F))); }
      } else {
        static const char from[] = "nrtbf", to[] = "\n\r\t\b\f";
        const char* hit = strchr(from, esc);
        out.push_back(hit && esc ? to[hit - from] : esc);
      }
    }
    if (p >= end) bad();
    ++p;
    return out;
  }
  Json value() {
    skip();
    if (p >= end) bad();
    Json j;
    if (*p == '{') {
      j.kind = Json::OBJ; ++p; skip();
      if (p < end && *p == '}') { ++p; return j; }
      while (true) {
        skip();
        if (p >= end || *p != '"') bad();
        std::string key = string_body();
        skip();
        if (p >= end || *p != ':') bad();
        ++p;
        j.obj[key] = value();
        skip();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; return j; }
        bad();
      }
    }
    if (*p == '[') {
      j.kind = Json::ARR; ++p; skip();
      if (p < end && *p == ']') { ++p; return j; }
      while (true) {
        j.arr.push_back(value());
        skip();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; return j; }
        bad();
      }
    }
    if (*p == '"') { j.kind = Json::STR; j.str = string_body(); return j; }
    if (lit("true")) { j.kind = Json::BOOL; j.b = true; return j; }
    if (lit("false")) { j.kind = Json::BOOL; j.b = false; return j; }
    if (lit("null")) return j;
    char* stop = nullptr;
    j.num = strtod(p, &stop);
    if (stop == p) bad();
    j.kind = Json::NUM;
    p = stop;
    return j;
  }
};
}  // namespace

Json Json::parse(const std::string& text) {
  Reader r{text.data(), text.data() + text.size()};
  return r.value();
}
const Json* Json::find(const std::string& k) const {
  if (kind != OBJ) return nullptr;
  auto it = obj.find(k);
  return it == obj.end() ? nullptr : &it->second;
}
bool Json::is_int() const { return kind == NUM && std::floor(num) == num && std::fabs(num) < 9.0e15; }

std::string read_text_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(ERR_IO, "cannot read " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}
bool path_exists(const std::string& path) { struct stat st; return stat(path.c_str(), &st) == 0; }

// -------------------------------------------------------------- config ----
void ModelConfig::parse(const Json& top) {
  const Json* tc = top.find("text_config");
  const Json& t = tc ? *tc : top;
  auto need_int = [&](const char* k) {
    const Json* v = t.find(k);
    if (!v || !v->is_int()) throw Error(ERR_FORMAT, std::string("config.json: missing field ") + k);
    return int(v->num);
  };
  auto num_or = [&](const Json& o, const char* k, double def, bool required) {
    const Json* v = o.find(k);
    if (v && v->kind == Json::NUM) return v->num;
    if (required) throw Error(ERR_FORMAT, std::string("config.json: missing field ") + k);
    return def;
  };
  const Json* mt = t.find("model_type");
  const Json* mt_top = top.find("model_type");
  model_type = (mt && mt->kind == Json::STR) ? mt->str : (mt_top && mt_top->kind == Json::STR) ? mt_top->str : "qwen3_next";
  hidden = need_int("hidden_size");
  layers = need_int("num_hidden_layers");
  heads = need_int("num_attention_heads");
  kv_heads = need_int("num_key_value_heads");
  head_dim = need_int("head_dim");
  eps = num_or(t, "rms_norm_eps", 1e-6, false);
  vocab = need_int("vocab_size");
  const Json* tw = t.find("tie_word_embeddings");
  const Json* tw_top = top.find("tie_word_embeddings");
  tie_embed = (tw && tw->kind == Json::BOOL) ? tw->b : (tw_top && tw_top->kind == Json::BOOL) ? tw_top->b : false;
  const Json* fai = t.find("full_attention_interval");
  full_attn_interval = (fai && fai->is_int()) ? int(fai->num) : 4;
  if (const Json* rp = t.find("rope_parameters"); rp && rp->kind == Json::OBJ) {
    rope_theta = num_or(*rp, "rope_theta", 10000000.0, false);
    const Json* pr = rp->find("partial_rotary_factor");
    // QwenConfig reads it with `as? Double`, so an integral literal is ignored.
    partial_rotary = (pr && pr->kind == Json::NUM && !pr->is_int()) ? pr->num : 0.25;
  } else {
    rope_theta = num_or(t, "rope_theta", 0, true);
    partial_rotary = num_or(t, "partial_rotary_factor", 0.25, false);
  }
  nv = need_int("linear_num_value_heads");
  nk = need_int("linear_num_key_heads");
  dk = need_int("linear_key_head_dim");
  dv = need_int("linear_value_head_dim");
  conv_k = need_int("linear_conv_kernel_dim");
  experts = need_int("num_experts");
  topk = need_int("num_experts_per_tok");
  moe_inter = need_int("moe_intermediate_size");
  shared_inter = need_int("shared_expert_intermediate_size");
  const Json* nt = t.find("norm_topk_prob");
  norm_topk = nt && nt->kind == Json::BOOL && nt->b;
  bool nested = tc != nullptr;
  split_layout = model_type.rfind("qwen3_5", 0) == 0 || model_type.rfind("qwen3_6", 0) == 0 || nested;
  prefix = nested ? "language_model." : "";
}

void QuantTable::parse(const Json& top) {
  const Json* q = top.find("quantization");
  if (!q || q->kind != Json::OBJ) return;
  const Json* g = q->find("group_size");
  const Json* b = q->find("bits");
  if (g && b && g->is_int() && b->is_int()) { has_default = true; def_gs = int(g->num); def_bits = int(b->num); }
  for (auto& kv : q->obj) {
    if (kv.second.kind != Json::OBJ) continue;
    const Json* sg = kv.second.find("group_size");
    const Json* sb = kv.second.find("bits");
    if (sg && sb && sg->is_int() && sb->is_int()) overrides.push_back({kv.first, {int(sb->num), int(sg->num)}});
  }
  std::sort(overrides.begin(), overrides.end());
}

bool QuantTable::lookup(const std::string& path, int& bits, int& gs) const {
  auto ends = [](const std::string& a, const std::string& s) {
    return a.size() >= s.size() && a.compare(a.size() - s.size(), s.size(), s) == 0;
  };
  for (auto& kv : overrides)
    if (ends(path, kv.first) || ends(kv.first, path)) { bits = kv.second.first; gs = kv.second.second; return true; }
  if (!has_default) return false;
  bits = def_bits; gs = def_gs;
  return true;
}

// ---------------------------------------------------------- safetensors ----
MappedFile::MappedFile(const std::string& path) {
  fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error(ERR_IO, "cannot open " + path);
  struct stat st;
  fstat(fd, &st);
  size = size_t(st.st_size);
  if (size) {
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) throw Error(ERR_IO, "mmap failed: " + path);
    base = static_cast<const uint8_t*>(m);
  }
}
MappedFile::~MappedFile() {
  if (base) munmap(const_cast<uint8_t*>(base), size);
  if (fd >= 0) close(fd);
}

SafetensorsFile::SafetensorsFile(const std::string& path) : map(new MappedFile(path)) {
  if (map->size < 8) throw Error(ERR_FORMAT, "malformed safetensors header: " + path);
  uint64_t hl;
  memcpy(&hl, map->base, 8);
  data_start = 8 + hl;
  if (data_start > map->size) throw Error(ERR_FORMAT, "malformed safetensors header: " + path);
  Json h = Json::parse(std::string(reinterpret_cast<const char*>(map->base) + 8, hl));
  if (h.kind != Json::OBJ) throw Error(ERR_FORMAT, "malformed safetensors header: " + path);
  for (auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const Json* dt = kv.second.find("dtype");
    const Json* sh = kv.second.find("shape");
    const Json* off = kv.second.find("data_offsets");
    if (!dt || !sh || !off || off->arr.size() != 2) throw Error(ERR_FORMAT, "malformed safetensors entry " + kv.first);
    TensorMeta m;
    m.dtype = dt->str;
    for (auto& d : sh->arr) m.shape.push_back(int64_t(d.num));
    int64_t a = int64_t(off->arr[0].num), b = int64_t(off->arr[1].num);
    if (b < a || data_start + size_t(b) > map->size) throw Error(ERR_FORMAT, "tensor outside file: " + kv.first);
    tensors[kv.first] = {m, {a, b}};
  }
}

CheckpointFiles::CheckpointFiles(const std::string& dir) {
  std::string idx = dir + "/model.safetensors.index.json";
  if (path_exists(idx)) {
    Json j = Json::parse(read_text_file(idx));
    const Json* wm = j.find("weight_map");
    if (!wm || wm->kind != Json::OBJ) throw Error(ERR_FORMAT, "index without weight_map: " + idx);
    std::map<std::string, int> file_id;
    for (auto& kv : wm->obj) {
      auto it = file_id.find(kv.second.str);
      if (it == file_id.end()) {
        files.emplace_back(new SafetensorsFile(dir + "/" + kv.second.str));
        it = file_id.emplace(kv.second.str, int(files.size()) - 1).first;
      }
      where[kv.first] = it->second;
    }
  } else {
    files.emplace_back(new SafetensorsFile(dir + "/model.safetensors"));
    for (auto& kv : files[0]->tensors) where[kv.first] = 0;
  }
}
std::string CheckpointFiles::resolve(const std::string& name) const {
  if (where.count(name)) return name;
  std::string p = "language_model." + name;
  return where.count(p) ? p : name;
}
TensorMeta CheckpointFiles::meta(const std::string& name) const {
  std::string r = resolve(name);
  auto it = where.find(r);
  if (it == where.end()) throw Error(ERR_FORMAT, "missing tensor " + name);
  return files[it->second]->tensors.at(r).first;
}
const uint8_t* CheckpointFiles::data(const std::string& name, size_t* nbytes) const {
  std::string r = resolve(name);
  auto it = where.find(r);
  if (it == where.end()) throw Error(ERR_FORMAT, "missing tensor " + name);
  const SafetensorsFile& f = *files[it->second];
  auto& e = f.tensors.at(r);
  if (nbytes) *nbytes = size_t(e.second.second - e.second.first);
  return f.map->base + f.data_start + e.second.first;
}

// ---------------------------------------------------------------- qpack ----
void QpackLayout::load(const std::string& dir) {
  Json lay = Json::parse(read_text_file(dir + "/packed_experts/layout.json"));
  auto geti = [&](const Json& o, const char* k) {
    const Json* v = o.find(k);
    if (!v || !v->is_int()) throw Error(ERR_FORMAT, std::string("layout.json: missing ") + k);
    return int64_t(v->num);
  };
  expert_count = int(geti(lay, "expertCount"));
  layer_count = int(geti(lay, "layerCount"));
  stride = geti(lay, "expertStride");
  const Json* secs = lay.find("sections");
  if (!secs || secs->kind != Json::ARR || secs->arr.empty() || stride <= 0)
    throw Error(ERR_FORMAT, "corrupt container: empty expert layout");
  for (auto& s : secs->arr) {
    QpackSection q;
    q.name = s.find("name") ? s.find("name")->str : "";
    q.dtype = s.find("dtype") ? s.find("dtype")->str : "";
    if (const Json* sh = s.find("shape")) for (auto& d : sh->arr) q.shape.push_back(int64_t(d.num));
    q.offset = geti(s, "offset");
    q.size = geti(s, "size");
    if (q.offset < 0 || q.offset + q.size > stride) throw Error(ERR_FORMAT, "qpack section outside the expert stride: " + q.name);
    sections.push_back(q);
  }
  if (path_exists(dir + "/manifest.json")) {
    Json man = Json::parse(read_text_file(dir + "/manifest.json"));
    if (const Json* b = man.find("quantBits"); b && b->is_int()) quant_bits = int(b->num);
    if (const Json* g = man.find("quantGroupSize"); g && g->is_int()) quant_group = int(g->num);
  }
}
const QpackSection* QpackLayout::find(const std::string& name) const {
  for (auto& s : sections) if (s.name == name) return &s;
  return nullptr;
}

int dtype_code(const std::string& dt) {
  if (dt == "F32") return DT_F32;
  if (dt == "BF16") return DT_BF16;
  if (dt == "F16") return DT_F16;
  throw Error(ERR_UNSUPPORTED, "unsupported floating dtype " + dt);
}
int64_t dtype_size(const std::string& dt) {
  if (dt == "F32" || dt == "U32" || dt == "I32") return 4;
  if (dt == "BF16" || dt == "F16" || dt == "U16" || dt == "I16") return 2;
  if (dt == "F64" || dt == "I64" || dt == "U64") return 8;
  if (dt == "U8" || dt == "I8") return 1;
  throw Error(ERR_UNSUPPORTED, "unsupported dtype " + dt);
}

}  // namespace swl
