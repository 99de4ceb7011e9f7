// Packed expert store, format v2: the reference's per-layer expert files,
// read into the pinned-host tier (host code only).
//
// Format (Sources/QwenFieldfareCore/Storage/QwenQ4ExpertStore.swift:50-159,
// written by QwenQ4ExpertStoreBuilder.swift:284-352):
//   <dir>/manifest.json       {"schemaVersion": 2, "sourceIndexSHA256": hex,
//                              "layers": [{"layerIndex", "filename",
//                              "fileSize", "payloadSHA256"} x 40]}
//   <dir>/layer_NN.q4exp      4,096-byte header, then 256 expert records of
//                              1,769,472 bytes in expert order (the slot
//                              layout of the HBM arena, byte for byte)
// Header, little-endian: magic "Q4EXP02\0" [0,8), u32 schema 2 @8, u32
// header length 4096 @12, u32 layer @16, u32 experts per layer @20, u32
// record bytes @24, u64 payload bytes @32, payload SHA-256 as 64 lowercase
// hex characters [40,104), source-index SHA-256 [104,168), zeros after.
// The payload digest is the SHA-256 of the 256 records.

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qf_moe.h"

namespace qf {
// qf_sha256_ni.cpp (compiled with the SHA extensions enabled)
bool sha256_ni_available();
void sha256_ni_blocks(uint32_t* state, const uint8_t* p, size_t n);
}  // namespace qf

namespace {

constexpr int kLayers = 40;
constexpr int kExpertsPerLayer = 256;
constexpr uint64_t kRecordBytes = 1769472;
constexpr uint64_t kHeaderBytes = QF_STORE_HEADER_BYTES;
constexpr uint64_t kPayloadBytes = kExpertsPerLayer * kRecordBytes;
constexpr uint64_t kLayerFileBytes = kHeaderBytes + kPayloadBytes;
constexpr uint32_t kSchema = 2;
const uint8_t kMagic[8] = {'Q', '4', 'E', 'X', 'P', '0', '2', 0};

thread_local std::string g_err;

qf_status fail(qf_status s, const std::string& msg) {
  g_err = msg;
  return s;
}

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4, section 6.2: 64-byte blocks, big-endian words, 64 rounds.
class Sha256 {
 public:
  Sha256() { reset(); }
  void reset() {
    static const uint32_t h0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    std::memcpy(h_, h0, sizeof(h_));
    len_ = 0;
    fill_ = 0;
  }
  void update(const void* data, size_t n) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    len_ += n;
    if (fill_) {
      const size_t take = std::min(n, sizeof(buf_) - fill_);
      std::memcpy(buf_ + fill_, p, take);
      fill_ += take;
      p += take;
      n -= take;
      if (fill_ < sizeof(buf_)) return;
      blocks(buf_, 1);
      fill_ = 0;
    }
    blocks(p, n / 64);
    p += n & ~size_t(63);
    n &= 63;
    std::memcpy(buf_, p, n);
    fill_ = n;
  }
  std::string hex() {
    const uint64_t bits = len_ * 8;
    const uint8_t pad0 = 0x80, zero = 0;
    update(&pad0, 1);
    while (fill_ != 56) update(&zero, 1);
    uint8_t lenbe[8];
    for (int i = 0; i < 8; i++) lenbe[i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
    update(lenbe, 8);
    static const char* digits = "0123456789abcdef";
    std::string out(64, '0');
    for (int i = 0; i < 8; i++)
      for (int b = 0; b < 4; b++) {
        const uint8_t v = static_cast<uint8_t>(h_[i] >> (24 - 8 * b));
        out[i * 8 + b * 2] = digits[v >> 4];
        out[i * 8 + b * 2 + 1] = digits[v & 15];
      }
    return out;
  }

 private:
  // the SHA extensions when the CPU has them, else the FIPS 180-4 rounds below
  void blocks(const uint8_t* p, size_t n) {
    // QF_SHA256_PORTABLE=1 selects the portable rounds (tests compare both)
    static const bool ni = qf::sha256_ni_available() && !std::getenv("QF_SHA256_PORTABLE");
    if (ni) {
      qf::sha256_ni_blocks(h_, p, n);
      return;
    }
    for (; n; n--, p += 64) block(p);
  }
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; i++)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; i++) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; i++) {
      const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h_[0] += a;
    h_[1] += b;
    h_[2] += c;
    h_[3] += d;
    h_[4] += e;
    h_[5] += f;
    h_[6] += g;
    h_[7] += h;
  }
  uint32_t h_[8];
  uint64_t len_;
  uint8_t buf_[64];
  size_t fill_;
};

bool is_sha256(const char* s, size_t n) {
  if (n != 64) return false;
  for (size_t i = 0; i < n; i++)
    if (!((s[i] >= '0' && s[i] <= '9') || (s[i] >= 'a' && s[i] <= 'f'))) return false;
  return true;
}
bool is_sha256(const std::string& s) { return is_sha256(s.data(), s.size()); }

// ---------------------------------------------------------------- JSON
// Just enough JSON for the manifest: objects, arrays, strings, numbers,
// literals; numbers keep their integral value when they have one.
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  bool integral = false;
  int64_t i = 0;
  std::string s;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(Json& out) {
    if (!value(out, 0)) return false;
    ws();
    return p_ == end_;
  }

 private:
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(end_ - p_) < n || std::strncmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) {
      o += (char)c;
    } else if (c < 0x800) {
      o += (char)(0xC0 | (c >> 6));
      o += (char)(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      o += (char)(0xE0 | (c >> 12));
      o += (char)(0x80 | ((c >> 6) & 0x3F));
      o += (char)(0x80 | (c & 0x3F));
    } else {
      o += (char)(0xF0 | (c >> 18));
      o += (char)(0x80 | ((c >> 12) & 0x3F));
      o += (char)(0x80 | ((c >> 6) & 0x3F));
      o += (char)(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t& v) {
    if (end_ - p_ < 4) return false;
    v = 0;
    for (int k = 0; k < 4; k++) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool str(std::string& o) {
    if (p_ >= end_ || *p_ != '"') return false;
    p_++;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if ((unsigned char)c < 0x20) return false;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p_ >= end_) return false;
      c = *p_++;
      switch (c) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t v;
          if (!hex4(v)) return false;
          if (v >= 0xD800 && v < 0xDC00) {
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return false;
            p_ += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
            v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(o, v);
          break;
        }
        default: return false;
      }
    }
    if (p_ >= end_) return false;
    p_++;
    return true;
  }
  bool number(Json& o) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') p_++;
    if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
    if (*p_ == '0') p_++;
    else while (p_ < end_ && *p_ >= '0' && *p_ <= '9') p_++;
    bool plain = true;
    if (p_ < end_ && *p_ == '.') {
      plain = false;
      p_++;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') p_++;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      plain = false;
      p_++;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) p_++;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') p_++;
    }
    const std::string text(s, p_);
    o.kind = Json::Num;
    o.num = std::strtod(text.c_str(), nullptr);
    if (plain && text.size() <= 18) {
      o.integral = true;
      o.i = std::strtoll(text.c_str(), nullptr, 10);
    } else if (o.num == (double)(int64_t)o.num && std::abs(o.num) < 9.0e15) {
      o.integral = true;
      o.i = (int64_t)o.num;
    }
    return true;
  }
  bool value(Json& o, int depth) {
    if (depth > 16) return false;
    ws();
    if (p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      p_++;
      o.kind = Json::Obj;
      ws();
      if (p_ < end_ && *p_ == '}') {
        p_++;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!str(key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        p_++;
        Json v;
        if (!value(v, depth + 1)) return false;
        o.obj[key] = std::move(v);
        ws();
        if (p_ < end_ && *p_ == ',') {
          p_++;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          p_++;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      p_++;
      o.kind = Json::Arr;
      ws();
      if (p_ < end_ && *p_ == ']') {
        p_++;
        return true;
      }
      for (;;) {
        Json v;
        if (!value(v, depth + 1)) return false;
        o.arr.push_back(std::move(v));
        ws();
        if (p_ < end_ && *p_ == ',') {
          p_++;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          p_++;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      o.kind = Json::Str;
      return str(o.s);
    }
    if (lit("true")) {
      o.kind = Json::Bool;
      o.b = true;
      return true;
    }
    if (lit("false")) {
      o.kind = Json::Bool;
      return true;
    }
    if (lit("null")) return true;
    return number(o);
  }
  const char* p_;
  const char* end_;
};

// ---------------------------------------------------------------- manifest
struct LayerEntry {
  int64_t layer_index = -1;
  std::string filename;
  int64_t file_size = 0;
  std::string payload_sha256;
};
struct Manifest {
  int64_t schema_version = 0;
  std::string source_index_sha256;
  std::vector<LayerEntry> layers;  // sorted by layer index once validated
};

std::string layer_filename(int layer) {
  char b[32];
  std::snprintf(b, sizeof b, "layer_%02d.q4exp", layer);
  return b;
}

bool get_int(const Json& o, const char* key, int64_t& v) {
  auto it = o.obj.find(key);
  if (it == o.obj.end() || it->second.kind != Json::Num || !it->second.integral) return false;
  v = it->second.i;
  return true;
}
bool get_str(const Json& o, const char* key, std::string& v) {
  auto it = o.obj.find(key);
  if (it == o.obj.end() || it->second.kind != Json::Str) return false;
  v = it->second.s;
  return true;
}

// JSONDecoder of QwenQ4ExpertStoreManifest (QwenQ4ExpertStore.swift:24-48),
// then QwenQ4ExpertStore.validateManifest (:322-342)
qf_status parse_manifest(const char* text, size_t n, Manifest& m) {
  Json root;
  if (!JsonParser(text, n).parse(root) || root.kind != Json::Obj)
    return fail(QF_ERR_ARG, "invalid manifest: not a JSON object");
  auto lay = root.obj.find("layers");
  if (!get_int(root, "schemaVersion", m.schema_version) ||
      !get_str(root, "sourceIndexSHA256", m.source_index_sha256) || lay == root.obj.end() ||
      lay->second.kind != Json::Arr)
    return fail(QF_ERR_ARG, "invalid manifest: missing or mistyped schemaVersion / sourceIndexSHA256 / layers");
  for (const Json& e : lay->second.arr) {
    LayerEntry le;
    if (e.kind != Json::Obj || !get_int(e, "layerIndex", le.layer_index) || !get_str(e, "filename", le.filename) ||
        !get_int(e, "fileSize", le.file_size) || !get_str(e, "payloadSHA256", le.payload_sha256))
      return fail(QF_ERR_ARG, "invalid manifest: malformed layer entry");
    m.layers.push_back(le);
  }
  if (m.schema_version != (int64_t)kSchema)
    return fail(QF_ERR_ARG, "invalid manifest: unsupported schema version " + std::to_string(m.schema_version));
  if (!is_sha256(m.source_index_sha256)) return fail(QF_ERR_ARG, "invalid manifest: invalid source index SHA-256");
  if ((int)m.layers.size() != kLayers)
    return fail(QF_ERR_ARG, "invalid manifest: expected 40 layers, got " + std::to_string(m.layers.size()));
  std::stable_sort(m.layers.begin(), m.layers.end(),
                   [](const LayerEntry& a, const LayerEntry& b) { return a.layer_index < b.layer_index; });
  for (int i = 0; i < kLayers; i++) {
    const LayerEntry& le = m.layers[i];
    if (le.layer_index != i || le.filename != layer_filename(i) || le.file_size != (int64_t)kLayerFileBytes ||
        !is_sha256(le.payload_sha256))
      return fail(QF_ERR_ARG, "invalid manifest: invalid layer entry " + std::to_string(i));
  }
  return QF_OK;
}

// ---------------------------------------------------------------- files
void put32(uint8_t* b, uint32_t v) {
  for (int i = 0; i < 4; i++) b[i] = (uint8_t)(v >> (8 * i));
}
void put64(uint8_t* b, uint64_t v) {
  for (int i = 0; i < 8; i++) b[i] = (uint8_t)(v >> (8 * i));
}
uint32_t get32(const uint8_t* b) {
  uint32_t v = 0;
  for (int i = 0; i < 4; i++) v |= (uint32_t)b[i] << (8 * i);
  return v;
}
uint64_t get64(const uint8_t* b) {
  uint64_t v = 0;
  for (int i = 0; i < 8; i++) v |= (uint64_t)b[i] << (8 * i);
  return v;
}

// QwenQ4ExpertStore.preadFully (:344-364): retries on EINTR, stops at EOF
size_t pread_fully(int fd, void* dst, size_t count, uint64_t offset) {
  size_t done = 0;
  while (done < count) {
    const ssize_t r = ::pread(fd, static_cast<uint8_t*>(dst) + done, count - done, (off_t)(offset + done));
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return done;
    done += (size_t)r;
  }
  return done;
}

bool read_file(const std::string& path, std::string& out) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return false;
  char buf[1 << 16];
  for (;;) {
    const ssize_t r = ::read(fd, buf, sizeof buf);
    if (r < 0 && errno == EINTR) continue;
    if (r < 0) {
      ::close(fd);
      return false;
    }
    if (r == 0) break;
    out.append(buf, (size_t)r);
  }
  ::close(fd);
  return true;
}

bool hash_file(const std::string& path, std::string& hex) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return false;
  Sha256 h;
  std::vector<uint8_t> buf(1 << 20);
  uint64_t off = 0;
  for (;;) {
    const size_t got = pread_fully(fd, buf.data(), buf.size(), off);
    h.update(buf.data(), got);
    off += got;
    if (got < buf.size()) break;
  }
  ::close(fd);
  hex = h.hex();
  return true;
}

// ---------------------------------------------------------------- checkpoint
// MLX safetensors shards: u64 little-endian header length, JSON header
// {name: {"dtype", "shape", "data_offsets": [begin, end]}}, then the data.
struct Slice {
  int fd = -1;
  uint64_t offset = 0;  // absolute file offset
  uint64_t bytes = 0;
  std::string dtype;
};

struct Shard {
  std::string path;
  int fd = -1;
  bool parsed = false;
  std::map<std::string, Slice> tensors;
};

// the 9 record components in record order (QwenQ4ExpertStoreBuilder.swift:41-55)
const char* const kComponentSuffix[9] = {"gate_proj.weight", "gate_proj.scales", "gate_proj.biases",
                                         "up_proj.weight",   "up_proj.scales",   "up_proj.biases",
                                         "down_proj.weight", "down_proj.scales", "down_proj.biases"};
const uint64_t kComponentBytes[9] = {524288, 32768, 32768, 524288, 32768, 32768, 524288, 32768, 32768};
const uint64_t kComponentOffset[9] = {0, 524288, 557056, 589824, 1114112, 1146880, 1179648, 1703936, 1736704};

}  // namespace

struct qf_checkpoint {
  std::string dir;
  std::map<std::string, std::string> weight_map;  // tensor name -> shard file
  std::map<std::string, Shard> shards;             // shard file -> parsed header + fd
  ~qf_checkpoint() {
    for (auto& kv : shards)
      if (kv.second.fd >= 0) ::close(kv.second.fd);
  }
  // The safetensors header of one shard: u64 length, then JSON whose tensors
  // carry data_offsets relative to the end of the header.
  qf_status parse_shard_header(int fd, const std::string& file, const std::string& path,
                               std::map<std::string, Slice>& tensors) {
    uint8_t lb[8];
    if (pread_fully(fd, lb, 8, 0) != 8) return fail(QF_ERR_IO, "short read from " + path);
    const uint64_t hlen = get64(lb);
    if (hlen == 0 || hlen > (256ull << 20))
      return fail(QF_ERR_ARG, "invalid manifest: invalid safetensors header length in " + file);
    std::string text(hlen, '\0');
    if (pread_fully(fd, &text[0], hlen, 8) != hlen) return fail(QF_ERR_IO, "short read from " + path);
    Json root;
    if (!JsonParser(text.data(), text.size()).parse(root) || root.kind != Json::Obj)
      return fail(QF_ERR_ARG, "invalid manifest: invalid safetensors header in " + file);
    for (auto& kv : root.obj) {
      if (kv.first == "__metadata__" || kv.second.kind != Json::Obj) continue;
      auto off = kv.second.obj.find("data_offsets");
      if (off == kv.second.obj.end() || off->second.kind != Json::Arr || off->second.arr.size() != 2 ||
          !off->second.arr[0].integral || !off->second.arr[1].integral)
        continue;
      const int64_t b = off->second.arr[0].i, e = off->second.arr[1].i;
      if (b < 0 || e < b) continue;
      Slice sl;
      sl.fd = fd;
      sl.offset = 8 + hlen + (uint64_t)b;
      sl.bytes = (uint64_t)(e - b);
      get_str(kv.second, "dtype", sl.dtype);
      tensors[kv.first] = sl;
    }
    return QF_OK;
  }
  // the tensor's slice; QwenQ4ExpertStoreBuilder.discoverSlices (:202-282)
  qf_status find(const std::string& name, Slice& out) {
    auto w = weight_map.find(name);
    if (w == weight_map.end()) return fail(QF_ERR_ARG, "invalid manifest: source index is missing " + name);
    Shard& sh = shards[w->second];
    if (!sh.parsed) {
      sh.path = dir + "/" + w->second;
      // the shard's descriptor is kept only once its header parsed; every
      // failure closes it, so a later find on the same shard opens afresh
      const int fd = ::open(sh.path.c_str(), O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
      if (fd < 0) return fail(QF_ERR_IO, "open failed for " + sh.path + ": errno " + std::to_string(errno));
      std::map<std::string, Slice> tensors;
      const qf_status ps = parse_shard_header(fd, w->second, sh.path, tensors);
      if (ps != QF_OK) {
        ::close(fd);
        return ps;
      }
      sh.fd = fd;
      sh.tensors.swap(tensors);
      sh.parsed = true;
    }
    auto t = sh.tensors.find(name);
    if (t == sh.tensors.end()) return fail(QF_ERR_ARG, "invalid manifest: missing tensor metadata for " + name);
    out = t->second;
    return QF_OK;
  }
};

namespace {

bool pwrite_fully(int fd, const void* src, size_t count, uint64_t offset) {
  size_t done = 0;
  while (done < count) {
    const ssize_t r = ::pwrite(fd, static_cast<const uint8_t*>(src) + done, count - done, (off_t)(offset + done));
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    done += (size_t)r;
  }
  return true;
}

qf_status fsync_dir(const std::string& dir) {
  const int fd = ::open(dir.c_str(), O_RDONLY | O_DIRECTORY | O_CLOEXEC | O_NOFOLLOW);
  if (fd < 0) return fail(QF_ERR_IO, "open directory failed for " + dir + ": errno " + std::to_string(errno));
  const int r = ::fsync(fd);
  ::close(fd);
  return r == 0 ? QF_OK : fail(QF_ERR_IO, "fsync directory failed for " + dir);
}

// QwenQ4ExpertStoreBuilder.atomicWrite (:437-473): <path>.tmp, fsync, rename, fsync dir
qf_status atomic_write(const std::string& text, const std::string& path, const std::string& dir) {
  const std::string tmp = path + ".tmp";
  if (::unlink(tmp.c_str()) != 0 && errno != ENOENT) return fail(QF_ERR_IO, "unlink failed for " + tmp);
  const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC | O_NOFOLLOW, 0644);
  if (fd < 0) return fail(QF_ERR_IO, "open failed for " + tmp + ": errno " + std::to_string(errno));
  const bool ok = pwrite_fully(fd, text.data(), text.size(), 0) && ::fsync(fd) == 0;
  ::close(fd);
  if (!ok || ::rename(tmp.c_str(), path.c_str()) != 0) {
    ::unlink(tmp.c_str());
    return fail(QF_ERR_IO, "write failed for " + path);
  }
  return fsync_dir(dir);
}

qf_status mkdirs(const std::string& path) {
  std::string cur;
  size_t i = 0;
  while (i <= path.size()) {
    const size_t j = path.find('/', i);
    cur = path.substr(0, j == std::string::npos ? path.size() : j);
    if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
      return fail(QF_ERR_IO, "mkdir failed for " + cur + ": errno " + std::to_string(errno));
    if (j == std::string::npos) break;
    i = j + 1;
  }
  return QF_OK;
}

// JSON as the builder's encoder writes it (pretty-printed, keys sorted)
std::string json_layer(const LayerEntry& e, const char* indent) {
  const std::string in(indent);
  return in + "{\n" + in + "  \"fileSize\" : " + std::to_string(e.file_size) + ",\n" + in + "  \"filename\" : \"" +
         e.filename + "\",\n" + in + "  \"layerIndex\" : " + std::to_string(e.layer_index) + ",\n" + in +
         "  \"payloadSHA256\" : \"" + e.payload_sha256 + "\"\n" + in + "}";
}
std::string json_layers(const std::vector<LayerEntry>& ls) {
  if (ls.empty()) return "[\n\n  ]";
  std::string o = "[\n";
  for (size_t i = 0; i < ls.size(); i++) o += json_layer(ls[i], "    ") + (i + 1 < ls.size() ? ",\n" : "\n");
  return o + "  ]";
}
std::string manifest_json(const std::string& src, const std::vector<LayerEntry>& ls) {
  return "{\n  \"layers\" : " + json_layers(ls) + ",\n  \"schemaVersion\" : 2,\n  \"sourceIndexSHA256\" : \"" + src +
         "\"\n}";
}
std::string resume_json(const std::string& src, const std::vector<LayerEntry>& ls) {
  return "{\n  \"completedLayers\" : " + json_layers(ls) + ",\n  \"schemaVersion\" : 2,\n  \"sourceIndexSHA256\" : \"" +
         src + "\"\n}";
}

bool file_exists(const std::string& p) {
  struct stat st;
  return ::lstat(p.c_str(), &st) == 0;
}

// QwenQ4ExpertStoreBuilder.verifyLayerFile (:373-401)
qf_status verify_layer_file(const std::string& path, const LayerEntry& expected, const std::string& src) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
  if (fd < 0) return fail(QF_ERR_IO, "open failed for " + path + ": errno " + std::to_string(errno));
  struct stat info;
  if (::fstat(fd, &info) != 0 || (int64_t)info.st_size != expected.file_size) {
    ::close(fd);
    return fail(QF_ERR_ARG, "invalid header: file size mismatch for " + path);
  }
  uint8_t hb[kHeaderBytes];
  qf_store_header h;
  if (pread_fully(fd, hb, kHeaderBytes, 0) != kHeaderBytes) {
    ::close(fd);
    return fail(QF_ERR_IO, "short read from " + path);
  }
  qf_status st = qf_store_header_decode(hb, kHeaderBytes, &h);
  if (st == QF_OK && (h.layer_index != expected.layer_index || h.experts_per_layer != kExpertsPerLayer ||
                      (uint64_t)h.expert_byte_length != kRecordBytes || h.payload_byte_length != kPayloadBytes ||
                      std::string(h.payload_sha256, 64) != expected.payload_sha256 ||
                      std::string(h.source_index_sha256, 64) != src))
    st = fail(QF_ERR_ARG, "invalid header: metadata mismatch for " + path);
  if (st == QF_OK) {
    Sha256 hs;
    std::vector<uint8_t> buf(1u << 20);
    uint64_t off = kHeaderBytes, left = kPayloadBytes;
    while (left && st == QF_OK) {
      const size_t want = (size_t)std::min<uint64_t>(left, buf.size());
      if (pread_fully(fd, buf.data(), want, off) != want) st = fail(QF_ERR_IO, "short read from " + path);
      hs.update(buf.data(), want);
      off += want;
      left -= want;
    }
    if (st == QF_OK && hs.hex() != expected.payload_sha256)
      st = fail(QF_ERR_ARG, "invalid header: payload SHA-256 mismatch for " + path);
  }
  ::close(fd);
  return st;
}

qf_status read_slice(const Slice& sl, uint64_t at, void* dst, uint64_t n, const std::string& name) {
  if (pread_fully(sl.fd, dst, n, sl.offset + at) != n) return fail(QF_ERR_IO, "short read of " + name);
  return QF_OK;
}

}  // namespace

struct qf_store {
  std::string dir;
  Manifest manifest;
  int fds[kLayers];
  std::atomic<int64_t> packed_reads{0};
  std::atomic<int64_t> pread_ops{0};
  std::atomic<int64_t> failures{0};
  qf_store() {
    for (int& f : fds) f = -1;
  }
  ~qf_store() {
    for (int f : fds)
      if (f >= 0) ::close(f);
  }
  bool read_expert(int layer, int expert, void* dst) {
    if (layer < 0 || layer >= kLayers || expert < 0 || expert >= kExpertsPerLayer || !dst) {
      failures++;
      return false;
    }
    const size_t got = pread_fully(fds[layer], dst, kRecordBytes, kHeaderBytes + (uint64_t)expert * kRecordBytes);
    pread_ops++;
    if (got != kRecordBytes) {
      failures++;
      return false;
    }
    packed_reads++;
    return true;
  }
};

extern "C" {

qf_status qf_sha256_hex(const void* data, size_t n, char* out) {
  if ((!data && n) || !out) return fail(QF_ERR_ARG, "qf_sha256_hex: null pointer");
  Sha256 h;
  h.update(data, n);
  const std::string hex = h.hex();
  std::memcpy(out, hex.c_str(), 65);
  return QF_OK;
}

qf_status qf_store_header_encode(const qf_store_header* h, uint8_t* out) {
  if (!h || !out) return fail(QF_ERR_ARG, "invalid header: null pointer");
  const size_t lp = strnlen(h->payload_sha256, sizeof h->payload_sha256);
  const size_t ls = strnlen(h->source_index_sha256, sizeof h->source_index_sha256);
  if (!is_sha256(h->payload_sha256, lp) || !is_sha256(h->source_index_sha256, ls))
    return fail(QF_ERR_ARG, "invalid header: SHA-256 fields must be 64 lowercase hexadecimal characters");
  if (h->layer_index < 0 || h->experts_per_layer <= 0 || h->expert_byte_length <= 0)
    return fail(QF_ERR_ARG, "invalid header: numeric field is out of range");
  std::memset(out, 0, kHeaderBytes);
  std::memcpy(out, kMagic, 8);
  put32(out + 8, kSchema);
  put32(out + 12, (uint32_t)kHeaderBytes);
  put32(out + 16, (uint32_t)h->layer_index);
  put32(out + 20, (uint32_t)h->experts_per_layer);
  put32(out + 24, (uint32_t)h->expert_byte_length);
  put64(out + 32, h->payload_byte_length);
  std::memcpy(out + 40, h->payload_sha256, 64);
  std::memcpy(out + 104, h->source_index_sha256, 64);
  return QF_OK;
}

qf_status qf_store_header_decode(const uint8_t* b, size_t n, qf_store_header* out) {
  if (!b || !out) return fail(QF_ERR_ARG, "invalid header: null pointer");
  if (n != kHeaderBytes)
    return fail(QF_ERR_ARG, "invalid header: expected 4096 bytes, got " + std::to_string(n));
  if (std::memcmp(b, kMagic, 8) != 0) return fail(QF_ERR_ARG, "invalid header: magic mismatch");
  if (get32(b + 8) != kSchema) return fail(QF_ERR_ARG, "invalid header: unsupported schema version");
  if (get32(b + 12) != (uint32_t)kHeaderBytes) return fail(QF_ERR_ARG, "invalid header: header byte length mismatch");
  if (!is_sha256(reinterpret_cast<const char*>(b + 40), 64) ||
      !is_sha256(reinterpret_cast<const char*>(b + 104), 64))
    return fail(QF_ERR_ARG, "invalid header: invalid SHA-256 field");
  const uint32_t layer = get32(b + 16), experts = get32(b + 20), bytes = get32(b + 24);
  if (layer > 0x7fffffffu || experts > 0x7fffffffu || bytes > 0x7fffffffu)
    return fail(QF_ERR_ARG, "invalid header: numeric field is out of range");
  qf_store_header h;
  std::memset(&h, 0, sizeof h);
  h.layer_index = (int32_t)layer;
  h.experts_per_layer = (int32_t)experts;
  h.expert_byte_length = (int32_t)bytes;
  h.payload_byte_length = get64(b + 32);
  std::memcpy(h.payload_sha256, b + 40, 64);
  std::memcpy(h.source_index_sha256, b + 104, 64);
  *out = h;
  return QF_OK;
}

qf_status qf_store_validate_manifest(const char* json, size_t n) {
  if (!json) return fail(QF_ERR_ARG, "invalid manifest: null pointer");
  Manifest m;
  return parse_manifest(json, n, m);
}

qf_status qf_store_open(const char* directory, const char* source_index_path, qf_store** out) {
  if (!directory || !out) return fail(QF_ERR_ARG, "qf_store_open: null pointer");
  *out = nullptr;
  std::unique_ptr<qf_store> s(new qf_store);
  s->dir = directory;
  const std::string mpath = s->dir + "/manifest.json";
  std::string text;
  if (!read_file(mpath, text)) return fail(QF_ERR_IO, "open failed for " + mpath + ": errno " + std::to_string(errno));
  qf_status st = parse_manifest(text.data(), text.size(), s->manifest);
  if (st != QF_OK) return st;
  if (source_index_path) {
    std::string actual;
    if (!hash_file(source_index_path, actual))
      return fail(QF_ERR_IO, std::string("open failed for ") + source_index_path);
    if (actual != s->manifest.source_index_sha256)
      return fail(QF_ERR_ARG, "source mismatch: the store belongs to a different source index (expected " +
                                  s->manifest.source_index_sha256 + ", got " + actual + ")");
  }
  for (int l = 0; l < kLayers; l++) {
    const LayerEntry& le = s->manifest.layers[l];
    const std::string path = s->dir + "/" + le.filename;
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
    if (fd < 0) return fail(QF_ERR_IO, "open failed for " + path + ": errno " + std::to_string(errno));
    s->fds[l] = fd;
    struct stat info;
    if (::fstat(fd, &info) != 0 || !S_ISREG(info.st_mode))
      return fail(QF_ERR_IO, "fstat failed for " + path + ": not a regular file");
    if ((uint64_t)info.st_size != (uint64_t)le.file_size || (uint64_t)le.file_size != kLayerFileBytes)
      return fail(QF_ERR_ARG, "invalid manifest: unexpected size for " + le.filename);
    uint8_t hb[kHeaderBytes];
    const size_t got = pread_fully(fd, hb, kHeaderBytes, 0);
    if (got != kHeaderBytes)
      return fail(QF_ERR_IO, "short read from " + path + ": expected 4096 bytes, got " + std::to_string(got));
    qf_store_header h;
    st = qf_store_header_decode(hb, kHeaderBytes, &h);
    if (st != QF_OK) return st;
    if (h.layer_index != le.layer_index || h.experts_per_layer != kExpertsPerLayer ||
        (uint64_t)h.expert_byte_length != kRecordBytes || h.payload_byte_length != kPayloadBytes ||
        le.payload_sha256 != std::string(h.payload_sha256, 64) ||
        s->manifest.source_index_sha256 != std::string(h.source_index_sha256, 64))
      return fail(QF_ERR_ARG, "invalid header: metadata mismatch in " + le.filename);
  }
  *out = s.release();
  return QF_OK;
}

void qf_store_close(qf_store* s) { delete s; }

qf_status qf_store_read_expert(qf_store* s, int32_t layer, int32_t expert, void* dst) {
  if (!s) return fail(QF_ERR_ARG, "qf_store_read_expert: null store");
  if (!s->read_expert(layer, expert, dst))
    return fail(layer < 0 || layer >= kLayers || expert < 0 || expert >= kExpertsPerLayer || !dst ? QF_ERR_ARG
                                                                                                 : QF_ERR_IO,
                "read of layer " + std::to_string(layer) + " expert " + std::to_string(expert) + " failed");
  return QF_OK;
}

qf_status qf_store_load_tier(qf_store* s, int32_t first_layer, int32_t n_layers, void* host_records,
                             uint64_t host_record_stride, int32_t threads) {
  if (!s || !host_records) return fail(QF_ERR_ARG, "qf_store_load_tier: null pointer");
  if (first_layer < 0 || n_layers < 1 || first_layer + n_layers > kLayers || host_record_stride < kRecordBytes)
    return fail(QF_ERR_ARG, "qf_store_load_tier: layers out of range or stride below one record");
  const int64_t total = (int64_t)n_layers * kExpertsPerLayer;
  const int nt = std::max(1, std::min<int>(threads > 0 ? threads : 8, (int)std::min<int64_t>(total, 64)));
  std::atomic<int64_t> next{0};
  std::atomic<int64_t> bad{-1};
  auto work = [&]() {
    for (;;) {
      const int64_t i = next.fetch_add(1);
      if (i >= total) return;
      uint8_t* dst = static_cast<uint8_t*>(host_records) + (uint64_t)i * host_record_stride;
      if (!s->read_expert(first_layer + (int)(i / kExpertsPerLayer), (int)(i % kExpertsPerLayer), dst)) {
        int64_t expect = -1;
        bad.compare_exchange_strong(expect, i);
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; t++) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  if (bad.load() >= 0) {
    const int64_t i = bad.load();
    return fail(QF_ERR_IO, "short read of layer " + std::to_string(first_layer + i / kExpertsPerLayer) +
                               " expert " + std::to_string(i % kExpertsPerLayer));
  }
  return QF_OK;
}

qf_status qf_store_get_metrics(const qf_store* s, qf_store_metrics* out) {
  if (!s || !out) return fail(QF_ERR_ARG, "qf_store_get_metrics: null pointer");
  out->packed_reads = s->packed_reads.load();
  out->pread_operations = s->pread_ops.load();
  out->read_failures = s->failures.load();
  return QF_OK;
}

qf_status qf_store_verify_layer(qf_store* s, int32_t layer, int32_t* matches) {
  if (!s || !matches) return fail(QF_ERR_ARG, "qf_store_verify_layer: null pointer");
  if (layer < 0 || layer >= kLayers) return fail(QF_ERR_ARG, "qf_store_verify_layer: layer out of range");
  Sha256 h;
  std::vector<uint8_t> buf(8u << 20);
  uint64_t off = kHeaderBytes, left = kPayloadBytes;
  while (left) {
    const size_t want = (size_t)std::min<uint64_t>(left, buf.size());
    const size_t got = pread_fully(s->fds[layer], buf.data(), want, off);
    if (got != want) return fail(QF_ERR_IO, "short read while hashing layer " + std::to_string(layer));
    h.update(buf.data(), got);
    off += got;
    left -= got;
  }
  *matches = h.hex() == s->manifest.layers[layer].payload_sha256 ? 1 : 0;
  return QF_OK;
}

qf_status qf_checkpoint_open(const char* model_path, qf_checkpoint** out) {
  if (!model_path || !out) return fail(QF_ERR_ARG, "qf_checkpoint_open: null pointer");
  *out = nullptr;
  std::unique_ptr<qf_checkpoint> c(new qf_checkpoint);
  c->dir = model_path;
  const std::string ipath = c->dir + "/model.safetensors.index.json";
  std::string text;
  if (!read_file(ipath, text)) return fail(QF_ERR_IO, "open failed for " + ipath + ": errno " + std::to_string(errno));
  Json root;
  if (!JsonParser(text.data(), text.size()).parse(root) || root.kind != Json::Obj)
    return fail(QF_ERR_ARG, "invalid manifest: source index is not a JSON object");
  auto wm = root.obj.find("weight_map");
  if (wm == root.obj.end() || wm->second.kind != Json::Obj)
    return fail(QF_ERR_ARG, "invalid manifest: source index has no weight_map");
  for (auto& kv : wm->second.obj) {
    if (kv.second.kind != Json::Str || kv.second.s.empty() || kv.second.s.find('/') != std::string::npos)
      return fail(QF_ERR_ARG, "invalid manifest: bad shard name for " + kv.first);
    c->weight_map[kv.first] = kv.second.s;
  }
  *out = c.release();
  return QF_OK;
}

void qf_checkpoint_close(qf_checkpoint* c) { delete c; }

qf_status qf_checkpoint_load_layer(qf_checkpoint* c, int32_t layer, const qf_layer_host* dst, int32_t threads,
                                   int32_t* scale_dtype) {
  if (!c || !dst) return fail(QF_ERR_ARG, "qf_checkpoint_load_layer: null pointer");
  if (layer < 0 || layer >= kLayers) return fail(QF_ERR_ARG, "qf_checkpoint_load_layer: layer out of range");
  if (dst->expert_bank && dst->record_stride < kRecordBytes)
    return fail(QF_ERR_ARG, "qf_checkpoint_load_layer: record_stride below one record");
  const std::string pre = "language_model.model.layers." + std::to_string(layer) + ".mlp.";
  struct Want {
    std::string name;
    uint64_t bytes;
    void* dst;
    bool scales;  // a 16-bit scale or bias tensor
  };
  // QwenQ4ActiveExpertStreamingRunner.swift:596-614 (router, shared gate, shared expert)
  std::vector<Want> direct = {
      {pre + "gate.weight", 256 * 2048, dst->router_w, false},
      {pre + "gate.scales", 256 * 32 * 2, dst->router_s, true},
      {pre + "gate.biases", 256 * 32 * 2, dst->router_b, true},
      {pre + "shared_expert_gate.weight", 2048, dst->coef_w, false},
      {pre + "shared_expert_gate.scales", 32 * 2, dst->coef_s, true},
      {pre + "shared_expert_gate.biases", 32 * 2, dst->coef_b, true},
  };
  std::string dtype16;
  auto check16 = [&](const Want& w, const Slice& sl) -> qf_status {
    if (!w.scales) return QF_OK;
    if (sl.dtype != "BF16" && sl.dtype != "F16")
      return fail(QF_ERR_ARG, "invalid manifest: " + w.name + " is " + sl.dtype + ", not BF16 or F16");
    if (dtype16.empty()) dtype16 = sl.dtype;
    if (sl.dtype != dtype16) return fail(QF_ERR_ARG, "invalid manifest: mixed scale types in layer " + std::to_string(layer));
    return QF_OK;
  };
  auto sized = [&](const Want& w, const Slice& sl, uint64_t expected) -> qf_status {
    if (sl.bytes != expected)
      return fail(QF_ERR_ARG, "invalid manifest: unexpected byte length for " + w.name + ": expected " +
                                  std::to_string(expected) + ", got " + std::to_string(sl.bytes));
    return check16(w, sl);
  };
  std::vector<std::pair<Want, Slice>> plain;
  for (const Want& w : direct) {
    Slice sl;
    qf_status st = c->find(w.name, sl);
    if (st == QF_OK) st = sized(w, sl, w.bytes);
    if (st != QF_OK) return st;
    plain.push_back({w, sl});
  }
  // shared expert: one record (QwenQ4ActiveExpertStreamingRunner.swift:605-613)
  for (int k = 0; k < 9; k++) {
    Want w{pre + "shared_expert." + kComponentSuffix[k], kComponentBytes[k],
           dst->shared_record ? static_cast<uint8_t*>(dst->shared_record) + kComponentOffset[k] : nullptr, k % 3 != 0};
    Slice sl;
    qf_status st = c->find(w.name, sl);
    if (st == QF_OK) st = sized(w, sl, w.bytes);
    if (st != QF_OK) return st;
    plain.push_back({w, sl});
  }
  // routed experts: [256][component] slices packed into records (builder packLayer, :284-327)
  Slice sw[9];
  std::string swname[9];
  for (int k = 0; k < 9; k++) {
    swname[k] = pre + "switch_mlp." + kComponentSuffix[k];
    Want w{swname[k], 0, nullptr, k % 3 != 0};
    qf_status st = c->find(w.name, sw[k]);
    if (st == QF_OK) st = sized(w, sw[k], kComponentBytes[k] * kExpertsPerLayer);
    if (st != QF_OK) return st;
  }
  for (auto& pw : plain)
    if (pw.first.dst) {
      const qf_status st = read_slice(pw.second, 0, pw.first.dst, pw.first.bytes, pw.first.name);
      if (st != QF_OK) return st;
    }
  if (dst->expert_bank) {
    const int nt = std::max(1, std::min(threads > 0 ? threads : 8, 64));
    std::atomic<int> next{0};
    std::atomic<int> bad{-1};
    auto work = [&]() {
      for (;;) {
        const int e = next.fetch_add(1);
        if (e >= kExpertsPerLayer) return;
        uint8_t* rec = static_cast<uint8_t*>(dst->expert_bank) + (uint64_t)e * dst->record_stride;
        for (int k = 0; k < 9; k++)
          if (pread_fully(sw[k].fd, rec + kComponentOffset[k], kComponentBytes[k],
                          sw[k].offset + (uint64_t)e * kComponentBytes[k]) != kComponentBytes[k]) {
            int expect = -1;
            bad.compare_exchange_strong(expect, e * 9 + k);
          }
      }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < nt; t++) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    if (bad.load() >= 0)
      return fail(QF_ERR_IO, "short read of " + swname[bad.load() % 9] + " expert " + std::to_string(bad.load() / 9));
  }
  if (scale_dtype) *scale_dtype = dtype16 == "BF16" ? QF_SCALE_BF16 : QF_SCALE_F16;
  return QF_OK;
}

}  // extern "C"

namespace {

// QwenQ4ExpertStoreBuilder.packLayer (:284-352): the layer's 256 records
// from the checkpoint slices into <final>.partial, digest, header, fsync,
// rename.  Records that read as all zeros are left as holes of the
// pre-sized file (same bytes, no write).
qf_status pack_layer(int layer, const Slice* sl, const std::string& src, const std::string& dir,
                     const std::string& partial, const std::string& final_path, LayerEntry& entry) {
  const int fd = ::open(partial.c_str(), O_RDWR | O_CREAT | O_EXCL | O_CLOEXEC | O_NOFOLLOW, 0644);
  if (fd < 0) return fail(QF_ERR_IO, "open failed for " + partial + ": errno " + std::to_string(errno));
  qf_status st = QF_OK;
  if (::ftruncate(fd, (off_t)kLayerFileBytes) != 0) st = fail(QF_ERR_IO, "ftruncate failed for " + partial);
  std::vector<uint64_t> rec64(kRecordBytes / 8);
  uint8_t* rec = reinterpret_cast<uint8_t*>(rec64.data());
  Sha256 h;
  for (int e = 0; e < kExpertsPerLayer && st == QF_OK; e++) {
    for (int k = 0; k < 9 && st == QF_OK; k++)
      if (pread_fully(sl[k].fd, rec + kComponentOffset[k], kComponentBytes[k],
                      sl[k].offset + (uint64_t)e * kComponentBytes[k]) != kComponentBytes[k])
        st = fail(QF_ERR_IO, "short read of layer " + std::to_string(layer) + " expert " + std::to_string(e));
    if (st != QF_OK) break;
    h.update(rec, kRecordBytes);
    bool zero = true;
    for (uint64_t w : rec64)
      if (w) {
        zero = false;
        break;
      }
    if (!zero && !pwrite_fully(fd, rec, kRecordBytes, kHeaderBytes + (uint64_t)e * kRecordBytes))
      st = fail(QF_ERR_IO, "pwrite failed for " + partial);
  }
  if (st == QF_OK) {
    qf_store_header hd;
    std::memset(&hd, 0, sizeof hd);
    hd.layer_index = layer;
    hd.experts_per_layer = kExpertsPerLayer;
    hd.expert_byte_length = (int32_t)kRecordBytes;
    hd.payload_byte_length = kPayloadBytes;
    const std::string digest = h.hex();
    std::memcpy(hd.payload_sha256, digest.c_str(), 65);
    std::memcpy(hd.source_index_sha256, src.c_str(), 65);
    uint8_t hb[kHeaderBytes];
    st = qf_store_header_encode(&hd, hb);
    if (st == QF_OK && !pwrite_fully(fd, hb, kHeaderBytes, 0)) st = fail(QF_ERR_IO, "pwrite failed for " + partial);
    if (st == QF_OK && ::fsync(fd) != 0) st = fail(QF_ERR_IO, "fsync failed for " + partial);
    entry.layer_index = layer;
    entry.filename = layer_filename(layer);
    entry.file_size = (int64_t)kLayerFileBytes;
    entry.payload_sha256 = digest;
  }
  ::close(fd);
  if (st == QF_OK && ::rename(partial.c_str(), final_path.c_str()) != 0)
    st = fail(QF_ERR_IO, "rename failed for " + partial);
  if (st == QF_OK) st = fsync_dir(dir);
  return st;
}

qf_status write_resume(const std::string& path, const std::string& dir, const std::string& src,
                       const std::map<int64_t, LayerEntry>& done) {
  std::vector<LayerEntry> ls;
  for (auto& kv : done) ls.push_back(kv.second);
  return atomic_write(resume_json(src, ls), path, dir);
}

}  // namespace

extern "C" {

qf_status qf_store_pack(const char* model_path, const char* out_dir, int32_t resume, qf_store_pack_result* res) {
  if (!model_path) return fail(QF_ERR_ARG, "qf_store_pack: null model path");
  const std::string model = model_path;
  const std::string out = out_dir ? std::string(out_dir) : model + "/qwen_q4_experts";
  const std::string index = model + "/model.safetensors.index.json";
  std::string src;
  if (!hash_file(index, src)) return fail(QF_ERR_IO, "open failed for " + index);
  auto report = [&](int written) {
    if (res) {
      res->layers_written = written;
      res->total_bytes = (uint64_t)kLayers * kLayerFileBytes;
      std::memcpy(res->source_index_sha256, src.c_str(), 65);
    }
    return QF_OK;
  };
  // an existing store is opened (and so validated), not rebuilt
  if (file_exists(out + "/manifest.json")) {
    qf_store* st = nullptr;
    const qf_status s = qf_store_open(out.c_str(), index.c_str(), &st);
    if (s != QF_OK) return s;
    qf_store_close(st);
    return report(0);
  }
  qf_status st = mkdirs(out);
  if (st != QF_OK) return st;
  const std::string ck = out + "/pack.resume.json";
  std::map<int64_t, LayerEntry> done;
  if (file_exists(ck)) {
    if (!resume) return fail(QF_ERR_ARG, "partial store: use resume to continue " + ck);
    std::string text;
    Json root;
    if (!read_file(ck, text) || !JsonParser(text.data(), text.size()).parse(root) || root.kind != Json::Obj)
      return fail(QF_ERR_ARG, "partial store: unreadable " + ck);
    int64_t schema = 0;
    std::string csrc;
    auto cl = root.obj.find("completedLayers");
    if (!get_int(root, "schemaVersion", schema) || !get_str(root, "sourceIndexSHA256", csrc) ||
        cl == root.obj.end() || cl->second.kind != Json::Arr || schema != (int64_t)kSchema || csrc != src)
      return fail(QF_ERR_ARG, "partial store: checkpoint does not match this source model");
    for (const Json& e : cl->second.arr) {
      LayerEntry le;
      if (e.kind != Json::Obj || !get_int(e, "layerIndex", le.layer_index) || !get_str(e, "filename", le.filename) ||
          !get_int(e, "fileSize", le.file_size) || !get_str(e, "payloadSHA256", le.payload_sha256) ||
          le.layer_index < 0 || le.layer_index >= kLayers)
        return fail(QF_ERR_ARG, "partial store: malformed completed layer in " + ck);
      done[le.layer_index] = le;
    }
  } else {
    st = write_resume(ck, out, src, done);
    if (st != QF_OK) return st;
  }
  qf_checkpoint* cp = nullptr;
  st = qf_checkpoint_open(model_path, &cp);
  if (st != QF_OK) return st;
  std::unique_ptr<qf_checkpoint> guard(cp);
  std::vector<Slice> sl((size_t)kLayers * 9);
  for (int l = 0; l < kLayers; l++)
    for (int k = 0; k < 9; k++) {
      const std::string name = "language_model.model.layers." + std::to_string(l) + ".mlp.switch_mlp." +
                               kComponentSuffix[k];
      st = cp->find(name, sl[(size_t)l * 9 + k]);
      if (st != QF_OK) return st;
      if (sl[(size_t)l * 9 + k].bytes != kComponentBytes[k] * kExpertsPerLayer)
        return fail(QF_ERR_ARG, "invalid manifest: unexpected byte length for " + name);
    }
  int written = 0;
  for (int l = 0; l < kLayers; l++) {
    const std::string fname = layer_filename(l), final_path = out + "/" + fname, partial = final_path + ".partial";
    auto it = done.find(l);
    if (it != done.end()) {
      st = verify_layer_file(final_path, it->second, src);
      if (st != QF_OK) return st;
      continue;
    }
    if (file_exists(final_path)) {
      if (!resume) return fail(QF_ERR_ARG, "partial store: unexpected completed file " + final_path + "; use resume");
      const int fd = ::open(final_path.c_str(), O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
      uint8_t hb[kHeaderBytes];
      const bool got = fd >= 0 && pread_fully(fd, hb, kHeaderBytes, 0) == kHeaderBytes;
      if (fd >= 0) ::close(fd);
      if (!got) return fail(QF_ERR_IO, "short read from " + final_path);
      qf_store_header h;
      st = qf_store_header_decode(hb, kHeaderBytes, &h);
      if (st != QF_OK) return st;
      LayerEntry le;
      le.layer_index = l;
      le.filename = fname;
      le.file_size = (int64_t)kLayerFileBytes;
      le.payload_sha256 = std::string(h.payload_sha256, 64);
      st = verify_layer_file(final_path, le, src);
      if (st == QF_OK) {
        done[l] = le;
        st = write_resume(ck, out, src, done);
      }
      if (st != QF_OK) return st;
      continue;
    }
    if (file_exists(partial)) {
      if (!resume) return fail(QF_ERR_ARG, "partial store: unfinished layer file " + partial + "; use resume");
      if (::unlink(partial.c_str()) != 0) return fail(QF_ERR_IO, "unlink failed for " + partial);
      st = fsync_dir(out);
      if (st != QF_OK) return st;
    }
    LayerEntry le;
    st = pack_layer(l, &sl[(size_t)l * 9], src, out, partial, final_path, le);
    if (st == QF_OK) {
      done[l] = le;
      st = write_resume(ck, out, src, done);
    }
    if (st != QF_OK) return st;
    written++;
  }
  std::vector<LayerEntry> ls;
  for (auto& kv : done) ls.push_back(kv.second);
  const std::string text = manifest_json(src, ls);
  Manifest m;
  st = parse_manifest(text.data(), text.size(), m);
  if (st == QF_OK) st = atomic_write(text, out + "/manifest.json", out);
  if (st != QF_OK) return st;
  if (::unlink(ck.c_str()) != 0 && errno != ENOENT) return fail(QF_ERR_IO, "unlink failed for " + ck);
  st = fsync_dir(out);
  return st == QF_OK ? report(written) : st;
}

qf_status qf_store_verify(const char* model_path, const char* out_dir, int32_t* layers_verified) {
  if (!model_path) return fail(QF_ERR_ARG, "qf_store_verify: null model path");
  const std::string model = model_path;
  const std::string out = out_dir ? std::string(out_dir) : model + "/qwen_q4_experts";
  const std::string index = model + "/model.safetensors.index.json";
  qf_store* s = nullptr;
  qf_status st = qf_store_open(out.c_str(), index.c_str(), &s);
  if (st != QF_OK) return st;
  std::unique_ptr<qf_store> guard(s);
  int n = 0;
  for (int l = 0; l < kLayers; l++) {
    const LayerEntry& le = s->manifest.layers[l];
    st = verify_layer_file(out + "/" + le.filename, le, s->manifest.source_index_sha256);
    if (st != QF_OK) return st;
    n++;
  }
  if (layers_verified) *layers_verified = n;
  return QF_OK;
}

const char* qf_store_last_error(void) { return g_err.c_str(); }

}  // extern "C"
