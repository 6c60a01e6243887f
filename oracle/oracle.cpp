// Swiftlet CPU oracle — TEST INFRASTRUCTURE ONLY.
//
// A C++17 restatement of Swiftlet's float32 CPU reference forward pass
// (Sources/SwiftletCore/QwenCPUModel.swift), its checkpoint reader and MLX
// affine dequantiser (Checkpoint.swift), the safetensors parser
// (Safetensors.swift) and the config decoder (QwenConfig.swift). It is the
// checker for the CUDA product in swiftlet_b200/ and the timed CPU baseline
// of bench.py; nothing in the product links, loads or calls it.
//
// Parity is pinned against the reference's own mlx-generated fixtures
// (fixtures/tiny_forward*.safetensors + greedy ids), with the tolerances of
// Tests/SwiftletCoreTests/FixtureForwardTests.swift:29-102; see
// tests/test_oracle_fixtures.py.
//
// Op order and constants follow the reference line by line (cited below):
// f32 accumulation, max-subtracted softmax, insertion top-k with ties keeping
// the lower expert id, softplus pass-through above 20, q/k RMSNorm eps 1e-6
// scaled by 1/dk and 1/sqrt(dk), (i+1) % interval layer typing. Compile with
// -ffp-contract=off so `scale * q + bias` rounds twice, as Swift does.
//
// A second weight source, "synthetic", generates checkpoint bytes from a
// counter-based hash (splitmix64 finaliser over (tensor name, element
// index)); the CUDA product implements the same published generator on the
// device so that 35B-shaped models need no files. Its byte-level agreement
// is checked by tests/test_gpu_synth.py.

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace orc {

using std::string;
using std::vector;

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---------------------------------------------------------------------------
// Minimal JSON (objects, arrays, numbers, strings, bools, null).
// ---------------------------------------------------------------------------
struct JVal {
  enum T { Null, Bool, Num, Str, Arr, Obj } t = Null;
  bool b = false;
  double n = 0;
  string s;
  vector<JVal> a;
  std::map<string, JVal> o;
  const JVal* get(const string& k) const {
    if (t != Obj) return nullptr;
    auto it = o.find(k);
    return it == o.end() ? nullptr : &it->second;
  }
  // Swift `as? Int` on a JSONSerialization number: integral values only.
  bool isInt() const { return t == Num && std::floor(n) == n && std::fabs(n) < 9e15; }
};

struct JParser {
  const char* p;
  const char* e;
  void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  [[noreturn]] void fail() { throw Error("malformed JSON"); }
  JVal parse() {
    ws();
    if (p >= e) fail();
    JVal v;
    char c = *p;
    if (c == '{') {
      v.t = JVal::Obj; ++p; ws();
      if (p < e && *p == '}') { ++p; return v; }
      for (;;) {
        ws(); if (p >= e || *p != '"') fail();
        string k = str(); ws();
        if (p >= e || *p != ':') fail();
        ++p;
        v.o[k] = parse(); ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; break; }
        fail();
      }
    } else if (c == '[') {
      v.t = JVal::Arr; ++p; ws();
      if (p < e && *p == ']') { ++p; return v; }
      for (;;) {
        v.a.push_back(parse()); ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; break; }
        fail();
      }
    } else if (c == '"') {
      v.t = JVal::Str; v.s = str();
    } else if (!strncmp(p, "true", 4)) { v.t = JVal::Bool; v.b = true; p += 4; }
    else if (!strncmp(p, "false", 5)) { v.t = JVal::Bool; v.b = false; p += 5; }
    else if (!strncmp(p, "null", 4)) { v.t = JVal::Null; p += 4; }
    else {
      char* end = nullptr;
      v.t = JVal::Num; v.n = strtod(p, &end);
      if (end == p) fail();
      p = end;
    }
    return v;
  }
  string str() {
    string r; ++p;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p; if (p >= e) fail();
        char c = *p++;
        switch (c) {
          case 'n': r += '\n'; break; case 't': r += '\t'; break;
          case 'r': r += '\r'; break; case 'b': r += '\b'; break; case 'f': r += '\f'; break;
          case 'u': { if (e - p < 4) fail(); unsigned cp = std::stoul(string(p, 4), nullptr, 16); p += 4;
                      if (cp < 0x80) r += char(cp); else if (cp < 0x800) { r += char(0xC0 | (cp >> 6)); r += char(0x80 | (cp & 63)); }
                      else { r += char(0xE0 | (cp >> 12)); r += char(0x80 | ((cp >> 6) & 63)); r += char(0x80 | (cp & 63)); } break; }
          default: r += c;
        }
      } else r += *p++;
    }
    if (p >= e) fail();
    ++p;
    return r;
  }
};

static JVal parseJSON(const string& text) {
  JParser jp{text.data(), text.data() + text.size()};
  return jp.parse();
}

static bool readFile(const string& path, string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END); long n = ftell(f); fseek(f, 0, SEEK_SET);
  out.resize(n);
  size_t got = n ? fread(&out[0], 1, n, f) : 0;
  fclose(f);
  return got == (size_t)n;
}

static bool fileExists(const string& p) { struct stat st; return stat(p.c_str(), &st) == 0; }

// ---------------------------------------------------------------------------
// Numeric helpers (Safetensors.swift:117-133, Checkpoint.swift:228-244).
// ---------------------------------------------------------------------------
static inline float bf16ToF32(uint16_t u) { uint32_t v = uint32_t(u) << 16; float f; memcpy(&f, &v, 4); return f; }
static inline float f16ToF32(uint16_t h) {
  uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023, out;
  if (e == 0) {
    if (m == 0) out = s << 31;
    else { int k = -1; do { m <<= 1; ++k; } while (!(m & 1024)); m &= 1023; out = (s << 31) | uint32_t(127 - 15 - k) << 23 | (m << 13); }
  } else if (e == 31) out = (s << 31) | 0x7F800000u | (m << 13);
  else out = (s << 31) | (e + 112) << 23 | (m << 13);
  float f; memcpy(&f, &out, 4); return f;
}
static inline uint16_t f32ToBF16RN(float f) {
  uint32_t u; memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
static size_t dtypeBytes(const string& d) {
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "I8" || d == "U8") return 1;
  throw Error("unsupported dtype " + d);
}

struct TensorInfo {
  string dtype;
  vector<int64_t> shape;
  int64_t numel() const { int64_t n = 1; for (auto s : shape) n *= s; return n; }
};

// ---------------------------------------------------------------------------
// Weight sources: safetensors files or the counter-based synthetic generator.
// ---------------------------------------------------------------------------
struct Source {
  virtual ~Source() = default;
  virtual bool has(const string& name) const = 0;
  virtual TensorInfo info(const string& name) const = 0;
  // Raw little-endian element bytes for elements [e0, e1).
  virtual void bytes(const string& name, int64_t e0, int64_t e1, uint8_t* dst) const = 0;
  virtual vector<string> names() const = 0;
};

// One mmapped safetensors file (Safetensors.swift:22-52).
struct STFile {
  int fd = -1; uint8_t* base = nullptr; size_t size = 0; size_t dataStart = 0;
  std::map<string, std::pair<TensorInfo, std::pair<int64_t, int64_t>>> tensors;
  explicit STFile(const string& path) {
    fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error("cannot open " + path);
    struct stat st; fstat(fd, &st); size = st.st_size;
    if (size < 8) throw Error("malformed safetensors header: " + path);
    base = (uint8_t*)mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (base == MAP_FAILED) throw Error("mmap failed: " + path);
    uint64_t hl; memcpy(&hl, base, 8);
    dataStart = 8 + hl;
    if (size < dataStart) throw Error("malformed safetensors header: " + path);
    JVal h = parseJSON(string((const char*)base + 8, hl));
    if (h.t != JVal::Obj) throw Error("malformed safetensors header");
    for (auto& kv : h.o) {
      if (kv.first == "__metadata__") continue;
      const JVal* dt = kv.second.get("dtype"); const JVal* sh = kv.second.get("shape"); const JVal* off = kv.second.get("data_offsets");
      if (!dt || !sh || !off || off->a.size() != 2) throw Error("malformed safetensors entry " + kv.first);
      TensorInfo ti; ti.dtype = dt->s;
      for (auto& d : sh->a) ti.shape.push_back((int64_t)d.n);
      tensors[kv.first] = {ti, {(int64_t)off->a[0].n, (int64_t)off->a[1].n}};
    }
  }
  ~STFile() { if (base && base != MAP_FAILED) munmap(base, size); if (fd >= 0) close(fd); }
};

// Checkpoint directory: single model.safetensors or sharded with an index
// (Checkpoint.swift:51-70).
struct FileSource : Source {
  vector<std::unique_ptr<STFile>> files;
  std::map<string, int> t2f;
  explicit FileSource(const string& dir) {
    string idx = dir + "/model.safetensors.index.json", text;
    if (fileExists(idx) && readFile(idx, text)) {
      JVal j = parseJSON(text);
      const JVal* wm = j.get("weight_map");
      if (!wm) throw Error("index without weight_map");
      std::map<string, int> fileIndex;
      for (auto& kv : wm->o) {
        auto it = fileIndex.find(kv.second.s);
        if (it == fileIndex.end()) {
          files.emplace_back(new STFile(dir + "/" + kv.second.s));
          it = fileIndex.emplace(kv.second.s, (int)files.size() - 1).first;
        }
        t2f[kv.first] = it->second;
      }
    } else {
      files.emplace_back(new STFile(dir + "/model.safetensors"));
      for (auto& kv : files[0]->tensors) t2f[kv.first] = 0;
    }
  }
  bool has(const string& n) const override { return t2f.count(n) > 0; }
  TensorInfo info(const string& n) const override {
    auto it = t2f.find(n); if (it == t2f.end()) throw Error("missing tensor " + n);
    return files[it->second]->tensors.at(n).first;
  }
  void bytes(const string& n, int64_t e0, int64_t e1, uint8_t* dst) const override {
    auto it = t2f.find(n); if (it == t2f.end()) throw Error("missing tensor " + n);
    const STFile& f = *files[it->second];
    auto& ent = f.tensors.at(n);
    size_t eb = dtypeBytes(ent.first.dtype);
    size_t off = f.dataStart + ent.second.first + e0 * eb, len = (e1 - e0) * eb;
    if (off + len > f.size || ent.second.first + (int64_t)((e1) * eb) > ent.second.second) throw Error("tensor range out of bounds: " + n);
    memcpy(dst, f.base + off, len);
  }
  vector<string> names() const override { vector<string> r; for (auto& kv : t2f) r.push_back(kv.first); return r; }
};

// --- Synthetic generator "swl-synth-v1" ------------------------------------
// Element i of tensor `name` draws h = mix64(key + (i+1)*GAMMA) with
// key = fnv1a64(name) ^ (seed * GAMMA) and mix64 the splitmix64 finaliser
// (Steele, Lea, Flood, "Fast splittable pseudorandom number generators",
// OOPSLA 2014). Every float op below is a single IEEE operation (no fused
// multiply-add), so host and device produce identical bytes.
static const uint64_t GAMMA = 0x9E3779B97F4A7C15ull;
static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t fnv1a64(const string& s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char c : s) { h ^= c; h *= 0x100000001b3ull; }
  return h;
}
static inline uint64_t synthHash(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * GAMMA); }
static inline float synthU(uint64_t h) { return float(h >> 40) * 5.9604644775390625e-08f; }  // [0,1), 24 bits
static inline float synthN(uint64_t h) {  // Irwin-Hall(4) standardised, ~N(0,1)
  int s = int(h & 0xFFFF) + int((h >> 16) & 0xFFFF) + int((h >> 32) & 0xFFFF) + int((h >> 48) & 0xFFFF);
  return float(s - 131070) * 2.6429039e-05f;
}

struct SynthSpec {
  uint64_t seed = 0;
  float weightStd = 0.02f;
  string scaleDtype = "BF16";   // scales / biases
  string plainDtype = "BF16";   // norms, conv, A_log, dt_bias
};

// The synthetic checkpoint exposes the tensor set of an mlx-lm qwen3_next /
// qwen3_5 checkpoint (stacked experts under switch_mlp) with every linear
// module quantised per the config's quantization block.
struct SynthSource : Source {
  SynthSpec sp;
  std::map<string, TensorInfo> infos;
  std::map<string, int> bitsOf;      // quantised module path -> bits
  std::map<string, int> groupOf;     // quantised module path -> group size
  std::map<string, int> roleOf;      // plain tensor -> role
  enum Role { NormW = 1, ALog = 2, DtBias = 3, Conv = 4, Other = 5 };

  void addQuant(const string& path, vector<int64_t> lead, int64_t out, int64_t in, int bits, int gs) {
    int pw = 32 / bits;
    TensorInfo w; w.dtype = "U32"; w.shape = lead; w.shape.push_back(out); w.shape.push_back(in / pw);
    TensorInfo s; s.dtype = sp.scaleDtype; s.shape = lead; s.shape.push_back(out); s.shape.push_back(in / gs);
    infos[path + ".weight"] = w; infos[path + ".scales"] = s; infos[path + ".biases"] = s;
    bitsOf[path] = bits; groupOf[path] = gs;
  }
  void addPlain(const string& name, vector<int64_t> shape, int role) {
    TensorInfo t; t.dtype = sp.plainDtype; t.shape = shape; infos[name] = t; roleOf[name] = role;
  }
  bool has(const string& n) const override { return infos.count(n) > 0; }
  TensorInfo info(const string& n) const override {
    auto it = infos.find(n); if (it == infos.end()) throw Error("missing tensor " + n); return it->second;
  }
  vector<string> names() const override { vector<string> r; for (auto& kv : infos) r.push_back(kv.first); return r; }

  static float scaleValue(uint64_t key, uint64_t i, float s0) {
    float u = synthU(synthHash(key, i));
    float t = u * 0.5f;
    t = t + 0.75f;
    return t * s0;
  }
  void bytes(const string& n, int64_t e0, int64_t e1, uint8_t* dst) const override {
    const TensorInfo& ti = info(n);
    uint64_t key = fnv1a64(n) ^ (sp.seed * GAMMA);
    if (ti.dtype == "U32") {
      uint32_t* o = (uint32_t*)dst;
      for (int64_t i = e0; i < e1; ++i) o[i - e0] = uint32_t(synthHash(key, i));
      return;
    }
    bool bf = ti.dtype == "BF16";
    if (!bf && ti.dtype != "F32") throw Error("synthetic dtype unsupported");
    auto put = [&](int64_t i, float v) {
      if (bf) { uint16_t b = f32ToBF16RN(v); memcpy(dst + (i - e0) * 2, &b, 2); }
      else memcpy(dst + (i - e0) * 4, &v, 4);
    };
    auto endsWith = [](const string& a, const string& b) { return a.size() >= b.size() && a.compare(a.size() - b.size(), b.size(), b) == 0; };
    if (endsWith(n, ".scales") || endsWith(n, ".biases")) {
      string path = n.substr(0, n.size() - 7);
      int bits = bitsOf.at(path);
      float qstd = bits == 4 ? 4.6097722286464435f : 73.90027063549903f;    // std of uniform q in [0, 2^bits)
      float s0 = float(double(sp.weightStd) / double(qstd));
      float mid = bits == 4 ? 7.5f : 127.5f;
      float nb = float(0.1 * double(sp.weightStd));
      uint64_t skey = fnv1a64(path + ".scales") ^ (sp.seed * GAMMA);
      bool isScale = endsWith(n, ".scales");
      for (int64_t i = e0; i < e1; ++i) {
        float s = scaleValue(skey, i, s0);
        float sq = bf ? bf16ToF32(f32ToBF16RN(s)) : s;   // the stored scale
        if (isScale) { put(i, s); continue; }
        float m1 = sq * (-mid);
        float m2 = synthN(synthHash(key, i)) * nb;
        put(i, m1 + m2);
      }
      return;
    }
    int role = roleOf.at(n);
    for (int64_t i = e0; i < e1; ++i) {
      uint64_t h = synthHash(key, i);
      float v;
      switch (role) {
        case NormW: { float m = synthN(h) * 0.05f; v = 1.0f + m; break; }
        case ALog: v = synthU(h); break;
        case DtBias: v = synthN(h) * 0.5f; break;
        case Conv: v = synthN(h) * 0.3f; break;
        default: v = synthN(h) * sp.weightStd;
      }
      put(i, v);
    }
  }
};

// ---------------------------------------------------------------------------
// QwenConfig (QwenConfig.swift:51-115).
// ---------------------------------------------------------------------------
struct Config {
  string modelType;
  int hiddenSize, numHiddenLayers, numAttentionHeads, numKeyValueHeads, headDim;
  double partialRotaryFactor, ropeTheta, rmsNormEps;
  int vocabSize; bool tieWordEmbeddings; int fullAttentionInterval;
  int linearNumValueHeads, linearNumKeyHeads, linearKeyHeadDim, linearValueHeadDim, linearConvKernelDim;
  int numExperts, numExpertsPerTok, moeIntermediateSize, sharedExpertIntermediateSize;
  bool normTopkProb;
  bool splitLayout;      // DeltaProjectionLayout.split (qwen3_5) vs fusedInterleaved
  string weightPrefix;

  bool isLinearLayer(int i) const { return (i + 1) % fullAttentionInterval != 0; }
  int keyDim() const { return linearNumKeyHeads * linearKeyHeadDim; }
  int valueDim() const { return linearNumValueHeads * linearValueHeadDim; }
  int convDim() const { return 2 * keyDim() + valueDim(); }
  int rotaryDims() const { return int(double(headDim) * partialRotaryFactor); }

  void parse(const JVal& top) {
    const JVal* tc = top.get("text_config");
    const JVal& text = tc ? *tc : top;
    bool nested = tc != nullptr;
    auto I = [&](const char* k) -> int {
      const JVal* v = text.get(k);
      if (!v || !v->isInt()) throw Error(string("missing config field ") + k);
      return (int)v->n;
    };
    auto D = [&](const char* k, const double* fb) -> double {
      const JVal* v = text.get(k);
      if (v && v->t == JVal::Num) return v->n;
      if (fb) return *fb;
      throw Error(string("missing config field ") + k);
    };
    const JVal* mt = text.get("model_type"); const JVal* mt2 = top.get("model_type");
    modelType = (mt && mt->t == JVal::Str) ? mt->s : (mt2 && mt2->t == JVal::Str) ? mt2->s : "qwen3_next";
    hiddenSize = I("hidden_size"); numHiddenLayers = I("num_hidden_layers");
    numAttentionHeads = I("num_attention_heads"); numKeyValueHeads = I("num_key_value_heads");
    headDim = I("head_dim");
    double epsDef = 1e-6; rmsNormEps = D("rms_norm_eps", &epsDef);
    vocabSize = I("vocab_size");
    const JVal* tw = text.get("tie_word_embeddings"); const JVal* tw2 = top.get("tie_word_embeddings");
    tieWordEmbeddings = (tw && tw->t == JVal::Bool) ? tw->b : (tw2 && tw2->t == JVal::Bool) ? tw2->b : false;
    const JVal* fai = text.get("full_attention_interval");
    fullAttentionInterval = (fai && fai->isInt()) ? (int)fai->n : 4;
    const JVal* rp = text.get("rope_parameters");
    if (rp && rp->t == JVal::Obj) {
      const JVal* th = rp->get("rope_theta"); const JVal* pr = rp->get("partial_rotary_factor");
      ropeTheta = (th && th->t == JVal::Num) ? th->n : 10000000.0;
      partialRotaryFactor = (pr && pr->t == JVal::Num && !pr->isInt()) ? pr->n : 0.25;
    } else {
      ropeTheta = D("rope_theta", nullptr);
      double prDef = 0.25; partialRotaryFactor = D("partial_rotary_factor", &prDef);
    }
    linearNumValueHeads = I("linear_num_value_heads"); linearNumKeyHeads = I("linear_num_key_heads");
    linearKeyHeadDim = I("linear_key_head_dim"); linearValueHeadDim = I("linear_value_head_dim");
    linearConvKernelDim = I("linear_conv_kernel_dim");
    numExperts = I("num_experts"); numExpertsPerTok = I("num_experts_per_tok");
    moeIntermediateSize = I("moe_intermediate_size"); sharedExpertIntermediateSize = I("shared_expert_intermediate_size");
    const JVal* nt = text.get("norm_topk_prob");
    normTopkProb = (nt && nt->t == JVal::Bool) ? nt->b : false;
    bool q35 = modelType.rfind("qwen3_5", 0) == 0 || modelType.rfind("qwen3_6", 0) == 0 || nested;
    splitLayout = q35;
    weightPrefix = nested ? "language_model." : "";
  }
};

// ---------------------------------------------------------------------------
// Checkpoint: quant spec resolution + MLX affine dequant (Checkpoint.swift).
// ---------------------------------------------------------------------------
struct QuantSpec { int groupSize = 0, bits = 0; };

struct Checkpoint {
  std::unique_ptr<Source> src;
  bool hasDefault = false; QuantSpec defQuant;
  vector<std::pair<string, QuantSpec>> overrides;   // sorted by key

  string resolve(const string& name) const {                         // Checkpoint.swift:75-79
    if (src->has(name)) return name;
    string p = "language_model." + name;
    return src->has(p) ? p : name;
  }
  bool contains(const string& n) const { return src->has(resolve(n)); }
  bool isQuantized(const string& path) const { return contains(path + ".scales"); }   // :122-124
  bool quantSpec(const string& path, QuantSpec& out) const {                          // :126-133
    if (!isQuantized(path)) return false;
    auto sfx = [](const string& a, const string& b) { return a.size() >= b.size() && a.compare(a.size() - b.size(), b.size(), b) == 0; };
    for (auto& kv : overrides)
      if (sfx(path, kv.first) || sfx(kv.first, path)) { out = kv.second; return true; }
    if (!hasDefault) return false;
    out = defQuant; return true;
  }
  TensorInfo info(const string& n) const { return src->info(resolve(n)); }

  vector<float> floats(const string& name, int64_t e0 = 0, int64_t e1 = -1) const {  // :228-244
    string r = resolve(name);
    TensorInfo ti = src->info(r);
    if (e1 < 0) e1 = ti.numel();
    vector<float> out(e1 - e0);
    if (ti.dtype == "F32") { src->bytes(r, e0, e1, (uint8_t*)out.data()); return out; }
    vector<uint16_t> tmp(e1 - e0);
    if (ti.dtype != "BF16" && ti.dtype != "F16") throw Error("unsupported dtype " + ti.dtype + " for " + name);
    src->bytes(r, e0, e1, (uint8_t*)tmp.data());
    bool bf = ti.dtype == "BF16";
    for (size_t i = 0; i < tmp.size(); ++i) out[i] = bf ? bf16ToF32(tmp[i]) : f16ToF32(tmp[i]);
    return out;
  }
  vector<uint32_t> u32s(const string& name, int64_t e0, int64_t e1) const {
    string r = resolve(name);
    TensorInfo ti = src->info(r);
    if (ti.dtype != "U32" && ti.dtype != "I32") throw Error("unsupported dtype " + ti.dtype + " for " + name);
    vector<uint32_t> out(e1 - e0);
    src->bytes(r, e0, e1, (uint8_t*)out.data());
    return out;
  }

  // MLX affine dequant, w[i] = scale[g]*q[i] + bias[g] (Checkpoint.swift:168-209).
  vector<float> dequantized(const string& path, int64_t r0, int64_t r1) const {
    QuantSpec spec;
    if (!quantSpec(path, spec)) throw Error("missing tensor " + path + ".scales");
    if (spec.bits != 4 && spec.bits != 8) throw Error("unsupported bits " + std::to_string(spec.bits));
    int perWord = 32 / spec.bits;
    uint32_t mask = (1u << spec.bits) - 1;
    TensorInfo wi = info(path + ".weight");
    int64_t packedCols = wi.shape.back(), logicalCols = packedCols * perWord;
    int64_t totalRows = 1; for (size_t i = 0; i + 1 < wi.shape.size(); ++i) totalRows *= wi.shape[i];
    if (r1 < 0) { r0 = 0; r1 = totalRows; }
    int64_t gpr = logicalCols / spec.groupSize;
    vector<uint32_t> packed = u32s(path + ".weight", r0 * packedCols, r1 * packedCols);
    vector<float> scales = floats(path + ".scales", r0 * gpr, r1 * gpr);
    vector<float> biases = floats(path + ".biases", r0 * gpr, r1 * gpr);
    int64_t rows = r1 - r0;
    vector<float> out(rows * logicalCols);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t w = 0; w < packedCols; ++w) {
        uint32_t word = packed[r * packedCols + w];
        for (int j = 0; j < perWord; ++j) {
          int64_t col = w * perWord + j, g = col / spec.groupSize;
          float q = float(word & mask);
          out[r * logicalCols + col] = scales[r * gpr + g] * q + biases[r * gpr + g];
          word >>= spec.bits;
        }
      }
    return out;
  }
  vector<float> moduleWeight(const string& path) const {                 // :137-143
    if (isQuantized(path)) return dequantized(path, 0, -1);
    return floats(path + ".weight");
  }
  vector<float> moduleWeightSlice(const string& path, int64_t r0, int64_t r1) const {  // :148-155
    if (isQuantized(path)) return dequantized(path, r0, r1);
    TensorInfo ti = info(path + ".weight");
    int64_t rowLen = ti.shape.back();
    return floats(path + ".weight", r0 * rowLen, r1 * rowLen);
  }
  vector<float> tensor(const string& n) const { return floats(n); }
};

static void parseQuant(const JVal& cfg, Checkpoint& ck) {                  // Checkpoint.swift:31-49
  const JVal* q = cfg.get("quantization");
  if (!q || q->t != JVal::Obj) return;
  const JVal* g = q->get("group_size"); const JVal* b = q->get("bits");
  if (g && b && g->isInt() && b->isInt()) { ck.hasDefault = true; ck.defQuant = {(int)g->n, (int)b->n}; }
  for (auto& kv : q->o) {
    if (kv.second.t != JVal::Obj) continue;
    const JVal* sg = kv.second.get("group_size"); const JVal* sb = kv.second.get("bits");
    if (sg && sb && sg->isInt() && sb->isInt()) ck.overrides.push_back({kv.first, {(int)sg->n, (int)sb->n}});
  }
}

// Builds the tensor table of a synthetic checkpoint from its config.
static SynthSource* makeSynth(const JVal& top, const Config& c, const Checkpoint& ck) {
  auto* s = new SynthSource();
  const JVal* sy = top.get("synthetic");
  if (const JVal* v = sy->get("seed")) s->sp.seed = (uint64_t)v->n;
  if (const JVal* v = sy->get("weight_std")) s->sp.weightStd = (float)v->n;
  if (const JVal* v = sy->get("scale_dtype")) s->sp.scaleDtype = v->s == "f32" ? "F32" : "BF16";
  if (const JVal* v = sy->get("plain_dtype")) s->sp.plainDtype = v->s == "f32" ? "F32" : "BF16";
  auto qs = [&](const string& path, int64_t in) {
    QuantSpec q = ck.defQuant;
    auto sfx = [](const string& a, const string& b) { return a.size() >= b.size() && a.compare(a.size() - b.size(), b.size(), b) == 0; };
    for (auto& kv : ck.overrides) if (sfx(path, kv.first) || sfx(kv.first, path)) { q = kv.second; break; }
    if (in % q.groupSize) throw Error("synthetic: group size does not divide in-dim of " + path);
    return q;
  };
  auto lin = [&](const string& path, vector<int64_t> lead, int64_t out, int64_t in) {
    QuantSpec q = qs(path, in);
    s->addQuant(path, lead, out, in, q.bits, q.groupSize);
  };
  int64_t D = c.hiddenSize, V = c.vocabSize;
  lin("model.embed_tokens", {}, V, D);
  if (!c.tieWordEmbeddings) lin("lm_head", {}, V, D);
  s->addPlain("model.norm.weight", {D}, SynthSource::NormW);
  for (int i = 0; i < c.numHiddenLayers; ++i) {
    string p = "model.layers." + std::to_string(i) + ".";
    s->addPlain(p + "input_layernorm.weight", {D}, SynthSource::NormW);
    s->addPlain(p + "post_attention_layernorm.weight", {D}, SynthSource::NormW);
    if (c.isLinearLayer(i)) {
      int64_t nv = c.linearNumValueHeads, K = c.linearConvKernelDim;
      s->addPlain(p + "linear_attn.A_log", {nv}, SynthSource::ALog);
      s->addPlain(p + "linear_attn.dt_bias", {nv}, SynthSource::DtBias);
      s->addPlain(p + "linear_attn.conv1d.weight", {c.convDim(), K, 1}, SynthSource::Conv);
      s->addPlain(p + "linear_attn.norm.weight", {c.linearValueHeadDim}, SynthSource::NormW);
      lin(p + "linear_attn.out_proj", {}, D, c.valueDim());
      if (c.splitLayout) {
        lin(p + "linear_attn.in_proj_qkv", {}, c.convDim(), D);
        lin(p + "linear_attn.in_proj_z", {}, c.valueDim(), D);
        lin(p + "linear_attn.in_proj_b", {}, nv, D);
        lin(p + "linear_attn.in_proj_a", {}, nv, D);
      } else {
        lin(p + "linear_attn.in_proj_qkvz", {}, 2 * c.keyDim() + 2 * c.valueDim(), D);
        lin(p + "linear_attn.in_proj_ba", {}, 2 * nv, D);
      }
    } else {
      int64_t H = c.numAttentionHeads, KVH = c.numKeyValueHeads, hd = c.headDim;
      lin(p + "self_attn.q_proj", {}, 2 * H * hd, D);
      lin(p + "self_attn.k_proj", {}, KVH * hd, D);
      lin(p + "self_attn.v_proj", {}, KVH * hd, D);
      lin(p + "self_attn.o_proj", {}, D, H * hd);
      s->addPlain(p + "self_attn.q_norm.weight", {hd}, SynthSource::NormW);
      s->addPlain(p + "self_attn.k_norm.weight", {hd}, SynthSource::NormW);
    }
    int64_t E = c.numExperts, I = c.moeIntermediateSize, SI = c.sharedExpertIntermediateSize;
    lin(p + "mlp.gate", {}, E, D);
    lin(p + "mlp.switch_mlp.gate_proj", {E}, I, D);
    lin(p + "mlp.switch_mlp.up_proj", {E}, I, D);
    lin(p + "mlp.switch_mlp.down_proj", {E}, D, I);
    lin(p + "mlp.shared_expert.gate_proj", {}, SI, D);
    lin(p + "mlp.shared_expert.up_proj", {}, SI, D);
    lin(p + "mlp.shared_expert.down_proj", {}, D, SI);
    lin(p + "mlp.shared_expert_gate", {}, 1, D);
  }
  return s;
}

// ---------------------------------------------------------------------------
// Ops (QwenCPUModel.swift:20-71).
// ---------------------------------------------------------------------------
// y = x @ W^T, W row-major (outDim, inDim) — QwenCPUModel.linear :20-30.
static vector<float> linear(const vector<float>& x, int rows, int inDim, const vector<float>& W, int outDim) {
  vector<float> out((size_t)rows * outDim, 0.f);
#pragma omp parallel for schedule(static) collapse(2)
  for (int r = 0; r < rows; ++r)
    for (int o = 0; o < outDim; ++o) {
      const float* w = &W[(size_t)o * inDim]; const float* xr = &x[(size_t)r * inDim];
      float acc = 0.f;
#pragma omp simd reduction(+ : acc)
      for (int i = 0; i < inDim; ++i) acc += xr[i] * w[i];
      out[(size_t)r * outDim + o] = acc;
    }
  return out;
}
// out[o] = W[o,:] . x — QwenCPUModel.matvec :32-45.
static void matvec(const float* W, int outDim, int inDim, const float* x, float* out) {
  for (int o = 0; o < outDim; ++o) {
    const float* w = W + (size_t)o * inDim; float acc = 0.f;
#pragma omp simd reduction(+ : acc)
    for (int i = 0; i < inDim; ++i) acc += w[i] * x[i];
    out[o] = acc;
  }
}
static void rmsNorm(float* x, int rows, int dim, const float* weight, float eps) {   // :47-59
  for (int r = 0; r < rows; ++r) {
    float* b = x + (size_t)r * dim; float ss = 0.f;
    for (int i = 0; i < dim; ++i) ss += b[i] * b[i];
    float scale = 1.f / std::sqrt(ss / float(dim) + eps);
    if (weight) for (int i = 0; i < dim; ++i) b[i] *= scale * weight[i];
    else for (int i = 0; i < dim; ++i) b[i] *= scale;
  }
}
static inline float sigmoidf_(float v) { return 1.f / (1.f + std::exp(-v)); }           // :61
static inline float siluf_(float v) { return v * sigmoidf_(v); }                        // :62
static inline float softplusf_(float v) { return v > 20.f ? v : std::log1p(std::exp(v)); }  // :63
static void softmaxRow(float* x, int count) {                                           // :65-71
  float m = -INFINITY;
  for (int i = 0; i < count; ++i) m = std::max(m, x[i]);
  float sum = 0.f;
  for (int i = 0; i < count; ++i) { x[i] = std::exp(x[i] - m); sum += x[i]; }
  for (int i = 0; i < count; ++i) x[i] /= sum;
}

// ---------------------------------------------------------------------------
// The model (QwenCPUModel.swift:73-569).
// ---------------------------------------------------------------------------
struct DecodeState {                                                                    // :183-193
  int position = 0;
  std::map<int, std::pair<vector<float>, vector<float>>> kv;
  std::map<int, vector<float>> convTail;
  std::map<int, vector<float>> deltaState;
};

struct Pick { int id; float p; };

struct Model {
  Config cfg;
  Checkpoint ck;
  vector<float> embed, finalNorm, lmHead;
  bool retainAll = false;

  struct AttnW { vector<float> q, k, v, o, qn, kn; };
  struct DeltaW { vector<float> qkvz, ba, qkv, z, b, a, conv, dtBias, aLog, norm, out; };
  struct MoEW { vector<float> gate; string prefix; vector<float> sg, su, sd, seg; };
  struct LayerW { vector<float> inNorm, postNorm; bool isDelta = false; AttnW attn; DeltaW delta; MoEW moe; };
  std::map<int, std::shared_ptr<LayerW>> all;
  std::pair<int, std::shared_ptr<LayerW>> cache{-1, nullptr};
  std::mutex mu;
  vector<vector<Pick>>* pickLog = nullptr;   // when set, moeForward appends each row's picks
  // Smallest relative gap between the k-th and (k+1)-th router probability
  // routed since the last orc_route_gap(reset): a test-side measure of how
  // close an input comes to a top-k tie, where float summation order alone
  // can change the picks of any other implementation.
  double minRouteGap = INFINITY;
  std::mutex gapMu;

  explicit Model(const string& dir) {
    string text;
    if (!readFile(dir + "/config.json", text)) throw Error("cannot read " + dir + "/config.json");
    JVal top = parseJSON(text);
    cfg.parse(top);
    parseQuant(top, ck);
    std::sort(ck.overrides.begin(), ck.overrides.end(), [](auto& a, auto& b) { return a.first < b.first; });
    if (top.get("synthetic")) ck.src.reset(makeSynth(top, cfg, ck));
    else ck.src.reset(new FileSource(dir));
    embed = ck.moduleWeight("model.embed_tokens");                                       // :124-126
    finalNorm = ck.tensor("model.norm.weight");
    lmHead = cfg.tieWordEmbeddings ? embed : ck.moduleWeight("lm_head");
  }

  std::shared_ptr<LayerW> layerWeights(int i) {                                         // :129-177
    std::lock_guard<std::mutex> g(mu);
    auto it = all.find(i);
    if (it != all.end()) return it->second;
    if (cache.first == i) return cache.second;
    string p = "model.layers." + std::to_string(i) + ".";
    auto L = std::make_shared<LayerW>();
    L->moe.gate = ck.moduleWeight(p + "mlp.gate");
    L->moe.prefix = p + "mlp.switch_mlp.";
    L->moe.sg = ck.moduleWeight(p + "mlp.shared_expert.gate_proj");
    L->moe.su = ck.moduleWeight(p + "mlp.shared_expert.up_proj");
    L->moe.sd = ck.moduleWeight(p + "mlp.shared_expert.down_proj");
    L->moe.seg = ck.moduleWeight(p + "mlp.shared_expert_gate");
    L->inNorm = ck.tensor(p + "input_layernorm.weight");
    L->postNorm = ck.tensor(p + "post_attention_layernorm.weight");
    if (cfg.isLinearLayer(i)) {
      L->isDelta = true;
      DeltaW& d = L->delta;
      d.conv = ck.tensor(p + "linear_attn.conv1d.weight");
      d.dtBias = ck.tensor(p + "linear_attn.dt_bias");
      d.aLog = ck.tensor(p + "linear_attn.A_log");
      d.norm = ck.tensor(p + "linear_attn.norm.weight");
      d.out = ck.moduleWeight(p + "linear_attn.out_proj");
      if (!cfg.splitLayout) {
        d.qkvz = ck.moduleWeight(p + "linear_attn.in_proj_qkvz");
        d.ba = ck.moduleWeight(p + "linear_attn.in_proj_ba");
      } else {
        d.qkv = ck.moduleWeight(p + "linear_attn.in_proj_qkv");
        d.z = ck.moduleWeight(p + "linear_attn.in_proj_z");
        d.b = ck.moduleWeight(p + "linear_attn.in_proj_b");
        d.a = ck.moduleWeight(p + "linear_attn.in_proj_a");
      }
    } else {
      AttnW& a = L->attn;
      a.q = ck.moduleWeight(p + "self_attn.q_proj");
      a.k = ck.moduleWeight(p + "self_attn.k_proj");
      a.v = ck.moduleWeight(p + "self_attn.v_proj");
      a.o = ck.moduleWeight(p + "self_attn.o_proj");
      a.qn = ck.tensor(p + "self_attn.q_norm.weight");
      a.kn = ck.tensor(p + "self_attn.k_norm.weight");
    }
    if (retainAll) all[i] = L; else cache = {i, L};
    return L;
  }

  // --- forward / step / layerForward (:205-281) ---
  vector<float> embedRows(const vector<int>& toks) {
    int D = cfg.hiddenSize;
    vector<float> h((size_t)toks.size() * D);
    for (size_t s = 0; s < toks.size(); ++s) {
      if (toks[s] < 0 || toks[s] >= cfg.vocabSize) throw Error("token id out of range");
      memcpy(&h[s * D], &embed[(size_t)toks[s] * D], D * 4);
    }
    return h;
  }

  vector<float> layerForward(const vector<float>& hin, int S, int li, DecodeState* st) {
    int D = cfg.hiddenSize;
    auto L = layerWeights(li);
    DecodeState local; DecodeState& state = st ? *st : local;
    vector<float> h = hin, x = hin;
    rmsNorm(x.data(), S, D, L->inNorm.data(), (float)cfg.rmsNormEps);
    vector<float> r = L->isDelta ? deltaNetForward(x, S, L->delta, li, state) : attentionForward(x, S, L->attn, li, state);
    for (size_t i = 0; i < h.size(); ++i) h[i] += r[i];
    vector<float> x2 = h;
    rmsNorm(x2.data(), S, D, L->postNorm.data(), (float)cfg.rmsNormEps);
    vector<float> m = moeForward(x2, S, L->moe, nullptr, nullptr);
    for (size_t i = 0; i < h.size(); ++i) h[i] += m[i];
    return h;
  }

  vector<float> attentionForward(const vector<float>& x, int S, const AttnW& w, int li, DecodeState& st) {   // :285-346
    int H = cfg.numAttentionHeads, KVH = cfg.numKeyValueHeads, hd = cfg.headDim, D = cfg.hiddenSize;
    float eps = (float)cfg.rmsNormEps;
    int past = st.position;
    vector<float> qOut = linear(x, S, D, w.q, H * hd * 2);
    vector<float> q((size_t)S * H * hd), gate((size_t)S * H * hd);
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < H; ++h) {
        size_t src = (size_t)s * H * hd * 2 + (size_t)h * 2 * hd;
        for (int i = 0; i < hd; ++i) {
          q[((size_t)s * H + h) * hd + i] = qOut[src + i];
          gate[((size_t)s * H + h) * hd + i] = qOut[src + hd + i];
        }
      }
    vector<float> k = linear(x, S, D, w.k, KVH * hd);
    vector<float> v = linear(x, S, D, w.v, KVH * hd);
    rmsNorm(q.data(), S * H, hd, w.qn.data(), eps);
    rmsNorm(k.data(), S * KVH, hd, w.kn.data(), eps);
    applyRope(q, S, H, past);
    applyRope(k, S, KVH, past);
    auto& cache = st.kv[li];
    cache.first.insert(cache.first.end(), k.begin(), k.end());
    cache.second.insert(cache.second.end(), v.begin(), v.end());
    const vector<float>& kAll = cache.first; const vector<float>& vAll = cache.second;
    float scale = 1.f / std::sqrt(float(hd));
    vector<float> attnOut((size_t)S * H * hd, 0.f);
    int group = H / KVH;
#pragma omp parallel for schedule(static)
    for (int head = 0; head < H; ++head) {
      vector<float> scores(past + S);
      int kvHead = head / group;
      for (int si = 0; si < S; ++si) {
        int kvLen = past + si + 1;
        for (int sj = 0; sj < kvLen; ++sj) {
          float dot = 0.f;
          for (int i = 0; i < hd; ++i) dot += q[((size_t)si * H + head) * hd + i] * kAll[((size_t)sj * KVH + kvHead) * hd + i];
          scores[sj] = dot * scale;
        }
        softmaxRow(scores.data(), kvLen);
        size_t dst = ((size_t)si * H + head) * hd;
        for (int sj = 0; sj < kvLen; ++sj) {
          float p = scores[sj];
          size_t vb = ((size_t)sj * KVH + kvHead) * hd;
          for (int i = 0; i < hd; ++i) attnOut[dst + i] += p * vAll[vb + i];
        }
      }
    }
    for (size_t i = 0; i < attnOut.size(); ++i) attnOut[i] *= sigmoidf_(gate[i]);
    return linear(attnOut, S, H * hd, w.o, D);
  }

  void applyRope(vector<float>& x, int S, int heads, int offset) {                      // :349-367
    int hd = cfg.headDim, rot = cfg.rotaryDims(), half = rot / 2;
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < heads; ++h) {
        size_t base = ((size_t)s * heads + h) * hd;
        for (int j = 0; j < half; ++j) {
          float invFreq = std::pow((float)cfg.ropeTheta, -float(2 * j) / float(rot));
          float angle = float(offset + s) * invFreq;
          float c = std::cos(angle), sn = std::sin(angle);
          float a = x[base + j], b = x[base + half + j];
          x[base + j] = a * c - b * sn;
          x[base + half + j] = b * c + a * sn;
        }
      }
  }

  vector<float> deltaNetForward(const vector<float>& x, int S, const DeltaW& w, int li, DecodeState& st) {  // :371-496
    int nk = cfg.linearNumKeyHeads, nv = cfg.linearNumValueHeads, dk = cfg.linearKeyHeadDim, dv = cfg.linearValueHeadDim;
    int rep = nv / nk, keyDim = cfg.keyDim(), valueDim = cfg.valueDim(), convDim = cfg.convDim(), K = cfg.linearConvKernelDim;
    int D = cfg.hiddenSize;
    vector<float> mixed, z, bArr, aArr;
    if (!cfg.splitLayout) {
      vector<float> qkvz = linear(x, S, D, w.qkvz, 2 * keyDim + 2 * valueDim);
      vector<float> ba = linear(x, S, D, w.ba, 2 * nv);
      int chunk = 2 * dk + 2 * rep * dv;
      mixed.assign((size_t)S * convDim, 0.f); z.assign((size_t)S * valueDim, 0.f);
      bArr.assign((size_t)S * nv, 0.f); aArr.assign((size_t)S * nv, 0.f);
      for (int s = 0; s < S; ++s)
        for (int hk = 0; hk < nk; ++hk) {
          size_t src = (size_t)s * (2 * keyDim + 2 * valueDim) + (size_t)hk * chunk;
          for (int i = 0; i < dk; ++i) {
            mixed[(size_t)s * convDim + hk * dk + i] = qkvz[src + i];
            mixed[(size_t)s * convDim + keyDim + hk * dk + i] = qkvz[src + dk + i];
          }
          for (int ri = 0; ri < rep; ++ri) {
            int hv = hk * rep + ri;
            for (int i = 0; i < dv; ++i) {
              mixed[(size_t)s * convDim + 2 * keyDim + hv * dv + i] = qkvz[src + 2 * dk + ri * dv + i];
              z[(size_t)s * valueDim + hv * dv + i] = qkvz[src + 2 * dk + rep * dv + ri * dv + i];
            }
          }
          size_t baSrc = (size_t)s * 2 * nv + hk * 2 * rep;
          for (int ri = 0; ri < rep; ++ri) {
            bArr[(size_t)s * nv + hk * rep + ri] = ba[baSrc + ri];
            aArr[(size_t)s * nv + hk * rep + ri] = ba[baSrc + rep + ri];
          }
        }
    } else {
      mixed = linear(x, S, D, w.qkv, convDim);
      z = linear(x, S, D, w.z, valueDim);
      bArr = linear(x, S, D, w.b, nv);
      aArr = linear(x, S, D, w.a, nv);
    }
    // Causal depthwise conv1d + silu over the session's conv tail (:423-439).
    int tailRows = K - 1;
    vector<float> padded;
    auto ct = st.convTail.find(li);
    if (ct != st.convTail.end()) padded = ct->second; else padded.assign((size_t)tailRows * convDim, 0.f);
    padded.insert(padded.end(), mixed.begin(), mixed.end());
    vector<float> convOut((size_t)S * convDim);
    for (int s = 0; s < S; ++s)
      for (int c = 0; c < convDim; ++c) {
        float acc = 0.f;
        for (int j = 0; j < K; ++j) acc += w.conv[(size_t)c * K + j] * padded[(size_t)(s + j) * convDim + c];
        convOut[(size_t)s * convDim + c] = siluf_(acc);
      }
    st.convTail[li] = vector<float>(padded.end() - (size_t)tailRows * convDim, padded.end());
    // q/k RMSNorm (no weight, eps 1e-6) scaled 1/dk and 1/sqrt(dk) (:441-457).
    vector<float> qh((size_t)S * keyDim), kh((size_t)S * keyDim), vh((size_t)S * valueDim);
    for (int s = 0; s < S; ++s) {
      for (int i = 0; i < keyDim; ++i) {
        qh[(size_t)s * keyDim + i] = convOut[(size_t)s * convDim + i];
        kh[(size_t)s * keyDim + i] = convOut[(size_t)s * convDim + keyDim + i];
      }
      for (int i = 0; i < valueDim; ++i) vh[(size_t)s * valueDim + i] = convOut[(size_t)s * convDim + 2 * keyDim + i];
    }
    rmsNorm(qh.data(), S * nk, dk, nullptr, 1e-6f);
    rmsNorm(kh.data(), S * nk, dk, nullptr, 1e-6f);
    float invScale = 1.f / std::sqrt(float(dk));
    for (auto& v : qh) v *= invScale * invScale;
    for (auto& v : kh) v *= invScale;
    // Gated delta rule recurrence (:459-488).
    auto ds = st.deltaState.find(li);
    vector<float> d0 = ds != st.deltaState.end() ? ds->second : vector<float>((size_t)nv * dv * dk, 0.f);
    vector<float> out((size_t)S * valueDim, 0.f);
    for (int s = 0; s < S; ++s) {
#pragma omp parallel for schedule(static)
      for (int hv = 0; hv < nv; ++hv) {
        int hk = hv / rep;
        float g = std::exp(-std::exp(w.aLog[hv]) * softplusf_(aArr[(size_t)s * nv + hv] + w.dtBias[hv]));
        float beta = sigmoidf_(bArr[(size_t)s * nv + hv]);
        size_t qB = (size_t)s * keyDim + hk * dk, kB = qB, vB = (size_t)s * valueDim + hv * dv;
        for (int dvi = 0; dvi < dv; ++dvi) {
          size_t sb = ((size_t)hv * dv + dvi) * dk;
          float kvMem = 0.f;
          for (int i = 0; i < dk; ++i) { d0[sb + i] *= g; kvMem += d0[sb + i] * kh[kB + i]; }
          float delta = (vh[vB + dvi] - kvMem) * beta;
          float y = 0.f;
          for (int i = 0; i < dk; ++i) { d0[sb + i] += kh[kB + i] * delta; y += d0[sb + i] * qh[qB + i]; }
          out[(size_t)s * valueDim + hv * dv + dvi] = y;
        }
      }
    }
    st.deltaState[li] = std::move(d0);
    // Gated RMSNorm: silu(z) * (rmsnorm(out) * weight) (:490-495).
    vector<float> normed = out;
    rmsNorm(normed.data(), S * nv, dv, w.norm.data(), (float)cfg.rmsNormEps);
    for (size_t i = 0; i < normed.size(); ++i) normed[i] *= siluf_(z[i]);
    return linear(normed, S, valueDim, w.out, D);
  }

  // Router softmax + insertion top-k (:506-521). Returns picks per row.
  vector<vector<Pick>> route(const vector<float>& x, int S, const MoEW& w, vector<float>* probsOut) {
    int D = cfg.hiddenSize, E = cfg.numExperts, topK = cfg.numExpertsPerTok;
    vector<float> router = linear(x, S, D, w.gate, E);
    vector<vector<Pick>> rows;
    for (int s = 0; s < S; ++s) {
      softmaxRow(&router[(size_t)s * E], E);
      vector<Pick> picks;
      auto byProb = [](const Pick& a, const Pick& b) { return a.p > b.p; };
      for (int e = 0; e < E; ++e) {
        float p = router[(size_t)s * E + e];
        if ((int)picks.size() < topK) { picks.push_back({e, p}); std::stable_sort(picks.begin(), picks.end(), byProb); }
        else if (p > picks[topK - 1].p) { picks[topK - 1] = {e, p}; std::stable_sort(picks.begin(), picks.end(), byProb); }
      }
      if (E > topK) {
        float next = -INFINITY;
        for (int e = 0; e < E; ++e) {
          bool picked = false;
          for (const Pick& pk : picks) picked |= pk.id == e;
          if (!picked) next = std::max(next, router[(size_t)s * E + e]);
        }
        const double kth = picks[topK - 1].p;
        const double gap = kth > 0 ? (kth - next) / kth : 0.0;
        std::lock_guard<std::mutex> g(gapMu);
        minRouteGap = std::min(minRouteGap, gap);
      }
      rows.push_back(picks);
    }
    if (probsOut) *probsOut = router;
    return rows;
  }

  vector<float> moeForward(const vector<float>& x, int S, const MoEW& w, vector<vector<Pick>>* picksOut, vector<float>* probsOut) {  // :500-569
    int D = cfg.hiddenSize, inter = cfg.moeIntermediateSize, sInter = cfg.sharedExpertIntermediateSize;
    vector<vector<Pick>> picksPerRow = route(x, S, w, probsOut);
    if (picksOut) *picksOut = picksPerRow;
    if (pickLog) pickLog->insert(pickLog->end(), picksPerRow.begin(), picksPerRow.end());
    std::map<int, std::array<vector<float>, 3>> ew;                                   // batch union (:524-535)
    for (auto& picks : picksPerRow)
      for (auto& pk : picks)
        if (!ew.count(pk.id)) {
          int e = pk.id;
          ew[e] = {ck.moduleWeightSlice(w.prefix + "gate_proj", (int64_t)e * inter, (int64_t)(e + 1) * inter),
                   ck.moduleWeightSlice(w.prefix + "up_proj", (int64_t)e * inter, (int64_t)(e + 1) * inter),
                   ck.moduleWeightSlice(w.prefix + "down_proj", (int64_t)e * D, (int64_t)(e + 1) * D)};
        }
    vector<float> out((size_t)S * D, 0.f);
#pragma omp parallel for schedule(static)
    for (int s = 0; s < S; ++s) {
      vector<float> gBuf(inter), uBuf(inter), dBuf(D), sG(sInter), sU(sInter);
      const vector<Pick>& picks = picksPerRow[s];
      float scoreSum = 0.f;
      for (auto& pk : picks) scoreSum += pk.p;
      const float* xs = &x[(size_t)s * D];
      for (auto& pk : picks) {
        float weight = cfg.normTopkProb ? pk.p / scoreSum : pk.p;
        auto& e = ew.at(pk.id);
        matvec(e[0].data(), inter, D, xs, gBuf.data());
        matvec(e[1].data(), inter, D, xs, uBuf.data());
        for (int i = 0; i < inter; ++i) gBuf[i] = siluf_(gBuf[i]) * uBuf[i];
        matvec(e[2].data(), D, inter, gBuf.data(), dBuf.data());
        for (int i = 0; i < D; ++i) out[(size_t)s * D + i] += weight * dBuf[i];
      }
      matvec(w.sg.data(), sInter, D, xs, sG.data());
      matvec(w.su.data(), sInter, D, xs, sU.data());
      for (int i = 0; i < sInter; ++i) sG[i] = siluf_(sG[i]) * sU[i];
      matvec(w.sd.data(), D, sInter, sG.data(), dBuf.data());
      float sg = 0.f;
      for (int i = 0; i < D; ++i) sg += w.seg[i] * xs[i];
      float sharedScale = sigmoidf_(sg);
      for (int i = 0; i < D; ++i) out[(size_t)s * D + i] += sharedScale * dBuf[i];
    }
    return out;
  }

  vector<float> step(const vector<int>& toks, DecodeState& st) {                          // :238-255
    int S = (int)toks.size(), D = cfg.hiddenSize;
    vector<float> h = embedRows(toks);
    for (int li = 0; li < cfg.numHiddenLayers; ++li) h = layerForward(h, S, li, &st);
    st.position += S;
    vector<float> last(h.end() - D, h.end());
    rmsNorm(last.data(), 1, D, finalNorm.data(), (float)cfg.rmsNormEps);
    return linear(last, 1, D, lmHead, cfg.vocabSize);
  }
};

static thread_local string g_err;

}  // namespace orc

using namespace orc;

#define ORC_TRY(...) try { __VA_ARGS__ } catch (const std::exception& e) { g_err = e.what(); return -1; }

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void* orc_open(const char* dir, int retain_all) {
  try { auto* m = new Model(dir); m->retainAll = retain_all != 0; return m; }
  catch (const std::exception& e) { g_err = e.what(); return nullptr; }
}
void orc_close(void* m) { delete (Model*)m; }

// Integer config fields by their config.json key names.
int orc_config_int(void* mp, const char* key) {
  Config& c = ((Model*)mp)->cfg; string k = key;
  if (k == "hidden_size") return c.hiddenSize;
  if (k == "num_hidden_layers") return c.numHiddenLayers;
  if (k == "num_attention_heads") return c.numAttentionHeads;
  if (k == "num_key_value_heads") return c.numKeyValueHeads;
  if (k == "head_dim") return c.headDim;
  if (k == "vocab_size") return c.vocabSize;
  if (k == "full_attention_interval") return c.fullAttentionInterval;
  if (k == "linear_num_value_heads") return c.linearNumValueHeads;
  if (k == "linear_num_key_heads") return c.linearNumKeyHeads;
  if (k == "linear_key_head_dim") return c.linearKeyHeadDim;
  if (k == "linear_value_head_dim") return c.linearValueHeadDim;
  if (k == "linear_conv_kernel_dim") return c.linearConvKernelDim;
  if (k == "num_experts") return c.numExperts;
  if (k == "num_experts_per_tok") return c.numExpertsPerTok;
  if (k == "moe_intermediate_size") return c.moeIntermediateSize;
  if (k == "shared_expert_intermediate_size") return c.sharedExpertIntermediateSize;
  if (k == "norm_topk_prob") return c.normTopkProb;
  if (k == "tie_word_embeddings") return c.tieWordEmbeddings;
  if (k == "split_layout") return c.splitLayout;
  if (k == "rotary_dims") return c.rotaryDims();
  return -1;
}

// Whole-sequence forward (QwenCPUModel.forward :205-233). Any output may be NULL.
int orc_forward(void* mp, const int32_t* tokens, int n, float* logits, float* layers, float* embed_out,
                float* final_norm, int32_t* greedy, int32_t* picks) {
  ORC_TRY({
    Model& m = *(Model*)mp; int D = m.cfg.hiddenSize, V = m.cfg.vocabSize;
    vector<vector<Pick>> log;
    m.pickLog = picks ? &log : nullptr;
    vector<int> toks(tokens, tokens + n);
    DecodeState st;
    vector<float> h = m.embedRows(toks);
    if (embed_out) memcpy(embed_out, h.data(), h.size() * 4);
    for (int li = 0; li < m.cfg.numHiddenLayers; ++li) {
      h = m.layerForward(h, n, li, &st);
      if (layers) memcpy(layers + (size_t)li * n * D, h.data(), h.size() * 4);
    }
    rmsNorm(h.data(), n, D, m.finalNorm.data(), (float)m.cfg.rmsNormEps);
    if (final_norm) memcpy(final_norm, h.data(), h.size() * 4);
    m.pickLog = nullptr;
    if (picks) {   // [layers][n][K] in layer order
      int K = m.cfg.numExpertsPerTok;
      for (size_t r = 0; r < log.size(); ++r)
        for (int k = 0; k < K; ++k) picks[r * K + k] = log[r][k].id;
    }
    vector<float> lg = linear(h, n, D, m.lmHead, V);
    if (logits) memcpy(logits, lg.data(), lg.size() * 4);
    if (greedy)
      for (int s = 0; s < n; ++s) {
        int best = 0;
        for (int v = 1; v < V; ++v) if (lg[(size_t)s * V + v] > lg[(size_t)s * V + best]) best = v;
        greedy[s] = best;
      }
    return 0;
  })
}

// One decoder layer from a given input (stateless unless `state` is given).
int orc_layer_forward(void* mp, const float* h_in, int S, int layer, void* state, float* h_out) {
  ORC_TRY({
    Model& m = *(Model*)mp;
    vector<float> h(h_in, h_in + (size_t)S * m.cfg.hiddenSize);
    vector<float> o = m.layerForward(h, S, layer, (DecodeState*)state);
    memcpy(h_out, o.data(), o.size() * 4);
    return 0;
  })
}

// The MoE block alone on an already-normalised input x [S, D]: output [S, D],
// picks [S, K] ids and their raw softmax probabilities, full probs [S, E].
int orc_moe_forward(void* mp, int layer, const float* x, int S, float* out, int32_t* pick_ids, float* pick_probs, float* probs) {
  ORC_TRY({
    Model& m = *(Model*)mp;
    auto L = m.layerWeights(layer);
    vector<float> xv(x, x + (size_t)S * m.cfg.hiddenSize), pr;
    vector<vector<Pick>> picks;
    vector<float> o = m.moeForward(xv, S, L->moe, &picks, &pr);
    if (out) memcpy(out, o.data(), o.size() * 4);
    if (probs) memcpy(probs, pr.data(), pr.size() * 4);
    int K = m.cfg.numExpertsPerTok;
    for (int s = 0; s < S; ++s)
      for (int k = 0; k < K; ++k) {
        if (pick_ids) pick_ids[s * K + k] = picks[s][k].id;
        if (pick_probs) pick_probs[s * K + k] = picks[s][k].p;
      }
    return 0;
  })
}

// The token mixer (DeltaNet or attention) alone on a normalised input.
int orc_mixer_forward(void* mp, int layer, const float* x, int S, void* state, float* out) {
  ORC_TRY({
    Model& m = *(Model*)mp;
    auto L = m.layerWeights(layer);
    DecodeState local; DecodeState& st = state ? *(DecodeState*)state : local;
    vector<float> xv(x, x + (size_t)S * m.cfg.hiddenSize);
    vector<float> o = L->isDelta ? m.deltaNetForward(xv, S, L->delta, layer, st) : m.attentionForward(xv, S, L->attn, layer, st);
    memcpy(out, o.data(), o.size() * 4);
    return 0;
  })
}

void* orc_state_new(void) { return new DecodeState(); }
void orc_state_free(void* s) { delete (DecodeState*)s; }
int orc_state_position(void* s) { return ((DecodeState*)s)->position; }
// Advance position without compute (used to pair mixer-only calls).
void orc_state_advance(void* s, int n) { ((DecodeState*)s)->position += n; }

// Delta state of a DeltaNet layer [nv, dv, dk] (zeros when absent).
int orc_state_delta(void* mp, void* s, int layer, float* out) {
  Model& m = *(Model*)mp; DecodeState& st = *(DecodeState*)s;
  size_t n = (size_t)m.cfg.linearNumValueHeads * m.cfg.linearValueHeadDim * m.cfg.linearKeyHeadDim;
  auto it = st.deltaState.find(layer);
  if (it == st.deltaState.end()) memset(out, 0, n * 4); else memcpy(out, it->second.data(), n * 4);
  return 0;
}

// Incremental step (QwenCPUModel.step :238-255): last position's logits.
// Smallest relative top-k router gap since the last reset (+inf if none).
double orc_route_gap(void* mp, int reset) {
  Model& m = *(Model*)mp;
  std::lock_guard<std::mutex> g(m.gapMu);
  const double v = m.minRouteGap;
  if (reset) m.minRouteGap = INFINITY;
  return v;
}

int orc_step(void* mp, void* state, const int32_t* tokens, int n, float* logits) {
  ORC_TRY({
    Model& m = *(Model*)mp;
    vector<int> toks(tokens, tokens + n);
    vector<float> lg = m.step(toks, *(DecodeState*)state);
    memcpy(logits, lg.data(), lg.size() * 4);
    return 0;
  })
}

// Dequantised rows [r0, r1) of a module (Checkpoint.moduleWeightSlice).
int orc_dequant(void* mp, const char* path, int64_t r0, int64_t r1, float* out) {
  ORC_TRY({
    vector<float> w = ((Model*)mp)->ck.moduleWeightSlice(path, r0, r1);
    memcpy(out, w.data(), w.size() * 4);
    return 0;
  })
}

// Raw bytes of elements [e0, e1) of a tensor (resolved name), file or synthetic.
int orc_tensor_bytes(void* mp, const char* name, int64_t e0, int64_t e1, void* out) {
  ORC_TRY({
    Model& m = *(Model*)mp;
    m.ck.src->bytes(m.ck.resolve(name), e0, e1, (uint8_t*)out);
    return 0;
  })
}

// dtype into dt (>= 8 bytes), shape into shape (<= 8 dims); returns ndim.
int orc_tensor_info(void* mp, const char* name, char* dt, int64_t* shape) {
  ORC_TRY({
    TensorInfo ti = ((Model*)mp)->ck.info(name);
    snprintf(dt, 8, "%s", ti.dtype.c_str());
    for (size_t i = 0; i < ti.shape.size() && i < 8; ++i) shape[i] = ti.shape[i];
    return (int)ti.shape.size();
  })
}

// --- model-free kernel oracles --------------------------------------------

// y[o] = sum_i (scale[g] * q + bias[g]) * x[i] over MLX-packed rows
// (MetalKernelTests.swift:136-151 cpuReference). sdtype 0 = f32, 1 = bf16, 2 = f16.
int orc_gemv_affine(const uint32_t* packed, const void* scales, const void* biases, int sdtype, int outDim, int inDim,
                    int gs, int bits, const float* x, float* y) {
  int perWord = 32 / bits, groups = inDim / gs; uint32_t mask = (1u << bits) - 1;
  auto ld = [&](const void* p, int i) -> float {
    if (sdtype == 0) return ((const float*)p)[i];
    uint16_t u = ((const uint16_t*)p)[i];
    return sdtype == 1 ? bf16ToF32(u) : f16ToF32(u);
  };
#pragma omp parallel for schedule(static)
  for (int o = 0; o < outDim; ++o) {
    float acc = 0.f;
    for (int i = 0; i < inDim; ++i) {
      uint32_t word = packed[(size_t)o * (inDim / perWord) + i / perWord];
      float q = float((word >> (bits * (i % perWord))) & mask);
      int g = o * groups + i / gs;
      acc += (ld(scales, g) * q + ld(biases, g)) * x[i];
    }
    y[o] = acc;
  }
  return 0;
}

// One expert's SwiGLU, y = down (silu(gate x) * (up x)), on MLX-affine
// matrices (QwenCPUModel.swift:552-555). gate/up [I, D], down [D, I].
int orc_expert_swiglu(const uint32_t* gw, const void* gs_, const void* gb, const uint32_t* uw, const void* us,
                      const void* ub, const uint32_t* dw, const void* ds, const void* db, int sdtype, int bits,
                      int group, int D, int I, const float* x, float* y) {
  std::vector<float> g(I), u(I);
  orc_gemv_affine(gw, gs_, gb, sdtype, I, D, group, bits, x, g.data());
  orc_gemv_affine(uw, us, ub, sdtype, I, D, group, bits, x, u.data());
  for (int i = 0; i < I; ++i) g[i] = siluf_(g[i]) * u[i];
  return orc_gemv_affine(dw, ds, db, sdtype, D, I, group, bits, g.data(), y);
}

// Gated delta rule over T steps (MetalKernelTests.swift:194-220; gated_delta.py ops path).
// q,k [T,Hk,Dk], v [T,Hv,Dv], g,beta [T,Hv], state [Hv,Dv,Dk] in/out, y [T,Hv,Dv].
int orc_gated_delta(const float* q, const float* k, const float* v, const float* g, const float* beta, float* state,
                    float* y, int T, int Hk, int Hv, int Dk, int Dv) {
  int rep = Hv / Hk;
  for (int t = 0; t < T; ++t)
    for (int hv = 0; hv < Hv; ++hv) {
      int hk = hv / rep;
      const float* qb = q + ((size_t)t * Hk + hk) * Dk; const float* kb = k + ((size_t)t * Hk + hk) * Dk;
      const float* vb = v + ((size_t)t * Hv + hv) * Dv;
      for (int d = 0; d < Dv; ++d) {
        float* sb = state + ((size_t)hv * Dv + d) * Dk;
        float kv = 0.f;
        for (int i = 0; i < Dk; ++i) { sb[i] *= g[t * Hv + hv]; kv += sb[i] * kb[i]; }
        float delta = (vb[d] - kv) * beta[t * Hv + hv];
        float out = 0.f;
        for (int i = 0; i < Dk; ++i) { sb[i] += kb[i] * delta; out += sb[i] * qb[i]; }
        y[((size_t)t * Hv + hv) * Dv + d] = out;
      }
    }
  return 0;
}

}  // extern "C"
