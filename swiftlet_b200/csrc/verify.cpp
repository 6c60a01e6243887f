// Container verification: the library-side counterpart of Swiftlet's
// scripts/verify_container.py. Every file listed in the container's
// hashes.json ({"files": {relative path: sha256 hex}}) is hashed and compared,
// every size listed in manifest.json ("files": {relative path: bytes}) is
// checked, and optionally the corrupt files and manifest.json are deleted so
// the installer reads the container as incomplete and fetches only those
// files again (verify_container.py:103-110). Host code only; no CUDA.
#include <sys/stat.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/swiftlet_cuda.h"
#include "common.h"
#include "host_io.h"

namespace swl {
namespace {

// ------------------------------------------------------------ SHA-256 ----
// FIPS 180-4. The round constants are the first 32 bits of the fractional
// parts of the cube roots of the first 64 primes, the initial hash those of
// the square roots of the first 8 primes; both are derived here from that
// definition (64-bit long double keeps the 32 bits exact for primes < 312).
struct Sha256Tables {
  uint32_t k[64], h0[8];
  Sha256Tables() {
    int primes[64], n = 0;
    for (int c = 2; n < 64; ++c) {
      bool p = true;
      for (int d = 2; d * d <= c; ++d) if (c % d == 0) { p = false; break; }
      if (p) primes[n++] = c;
    }
    auto frac32 = [](long double v) {
      const long double f = v - floorl(v);
      return uint32_t(uint64_t(floorl(f * 4294967296.0L)) & 0xffffffffu);
    };
    for (int i = 0; i < 64; ++i) k[i] = frac32(cbrtl((long double)primes[i]));
    for (int i = 0; i < 8; ++i) h0[i] = frac32(sqrtl((long double)primes[i]));
  }
};
const Sha256Tables& tables() {
  static const Sha256Tables t;
  return t;
}

inline uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }

struct Sha256 {
  uint32_t h[8];
  uint8_t buf[64];
  uint64_t total = 0;
  int fill = 0;
  Sha256() { memcpy(h, tables().h0, sizeof h); }

  void block(const uint8_t* p) {
    const uint32_t* K = tables().k;
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = uint32_t(p[4 * i]) << 24 | uint32_t(p[4 * i + 1]) << 16 | uint32_t(p[4 * i + 2]) << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const uint8_t* p, size_t n) {
    total += n;
    if (fill) {
      const size_t take = std::min(n, size_t(64 - fill));
      memcpy(buf + fill, p, take);
      fill += int(take); p += take; n -= take;
      if (fill == 64) { block(buf); fill = 0; }
    }
    for (; n >= 64; p += 64, n -= 64) block(p);
    if (n) { memcpy(buf, p, n); fill = int(n); }
  }
  std::string hex() {
    const uint64_t bits = total * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (fill != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = uint8_t(bits >> (56 - 8 * i));
    update(len, 8);
    static const char* dig = "0123456789abcdef";
    std::string s;
    for (uint32_t v : h)
      for (int i = 7; i >= 0; --i) s += dig[(v >> (4 * i)) & 15];
    return s;
  }
};

bool sha256_file(const std::string& path, std::string& hex) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  Sha256 s;
  std::vector<uint8_t> chunk(size_t(4) << 20);
  size_t n;
  while ((n = fread(chunk.data(), 1, chunk.size(), f)) > 0) s.update(chunk.data(), n);
  const bool ok = !ferror(f);
  fclose(f);
  if (ok) hex = s.hex();
  return ok;
}

int64_t file_size(const std::string& path) {
  struct stat st;
  return stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode) ? int64_t(st.st_size) : -1;
}

std::string lower(std::string s) {
  for (auto& c : s) c = char(tolower(c));
  return s;
}

}  // namespace
}  // namespace swl

using namespace swl;

extern "C" int swl_sha256_file(const char* path, char* hex_out) {
  try {
    if (!path || !hex_out) throw Error(ERR_INVALID, "null argument");
    std::string hex;
    if (!sha256_file(path, hex)) throw Error(ERR_IO, std::string("cannot read ") + path);
    memcpy(hex_out, hex.c_str(), 65);
    return SWL_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  }
}

extern "C" int swl_qpack_verify(const char* dir, const char* hashes_json, int32_t delete_corrupt,
                                swl_verify_report* out) {
  try {
    if (!dir) throw Error(ERR_INVALID, "null container directory");
    const std::string root(dir);
    const std::string hpath = hashes_json ? std::string(hashes_json) : root + "/hashes.json";
    if (!path_exists(hpath)) throw Error(ERR_IO, "no hash list at " + hpath);
    const Json hj = Json::parse(read_text_file(hpath));
    const Json* files = hj.find("files");
    if (!files || files->kind != Json::OBJ || files->obj.empty()) throw Error(ERR_FORMAT, hpath + ": no \"files\" map");
    struct Item { std::string rel, want; int state = 0; };  // 0 ok, 1 corrupt, 2 missing
    std::vector<Item> items;
    for (const auto& kv : files->obj) {
      if (kv.second.kind != Json::STR) throw Error(ERR_FORMAT, hpath + ": hash of " + kv.first + " is not a string");
      items.push_back({kv.first, lower(kv.second.str)});
    }
    // manifest.json sizes, where the container has one (Qpack.swift:38-46)
    std::map<std::string, int64_t> sizes;
    if (path_exists(root + "/manifest.json")) {
      const Json man = Json::parse(read_text_file(root + "/manifest.json"));
      if (const Json* mf = man.find("files"); mf && mf->kind == Json::OBJ)
        for (const auto& kv : mf->obj) if (kv.second.is_int()) sizes[kv.first] = int64_t(kv.second.num);
    }
    std::atomic<size_t> next{0};
    auto work = [&] {
      for (size_t i; (i = next.fetch_add(1)) < items.size();) {
        Item& it = items[i];
        const std::string path = root + "/" + it.rel;
        const int64_t sz = file_size(path);
        if (sz < 0) { it.state = 2; continue; }
        auto ms = sizes.find(it.rel);
        if (ms != sizes.end() && ms->second != sz) { it.state = 1; continue; }
        std::string got;
        it.state = sha256_file(path, got) && got == it.want ? 0 : 1;
      }
    };
    const unsigned nt = std::max(1u, std::min(unsigned(items.size()), std::thread::hardware_concurrency()));
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < nt; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    swl_verify_report r{};
    std::string first_bad;
    for (const Item& it : items) {
      ++r.checked;
      if (it.state == 0) ++r.ok;
      else if (it.state == 1) ++r.corrupt;
      else ++r.missing;
      if (it.state && first_bad.empty()) first_bad = it.rel;
    }
    snprintf(r.first_bad, sizeof r.first_bad, "%s", first_bad.c_str());
    if (delete_corrupt && r.corrupt) {
      for (const Item& it : items) if (it.state == 1) remove((root + "/" + it.rel).c_str());
      remove((root + "/manifest.json").c_str());
    }
    if (out) *out = r;
    if (r.corrupt || r.missing)
      throw Error(ERR_FORMAT, std::to_string(r.corrupt) + " corrupt, " + std::to_string(r.missing) + " missing of " +
                                  std::to_string(r.checked) + " files (first: " + first_bad + ")");
    return SWL_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return SWL_ERR_FORMAT;
  }
}
