// Host side of the model boundary. See model_host.hpp for the reference map.
#include "model_host.hpp"

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <set>
#include <sstream>

namespace so3lr_b200 {
namespace {

[[noreturn]] void fail(const std::string &msg) { throw Error("SO3LR model: " + msg); }

std::uint32_t le32(const std::uint8_t *p) {
  return std::uint32_t(p[0]) | std::uint32_t(p[1]) << 8 | std::uint32_t(p[2]) << 16 |
         std::uint32_t(p[3]) << 24;
}
std::uint64_t le64(const std::uint8_t *p) {
  return std::uint64_t(le32(p)) | std::uint64_t(le32(p + 4)) << 32;
}

}  // namespace

// ---- SHA-256 (FIPS 180-4) ---------------------------------------------------
namespace {
constexpr std::uint32_t kSha[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
    0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
    0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
    0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
    0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
    0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
    0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
    0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};
inline std::uint32_t rotr(std::uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha_block(std::uint32_t h[8], const std::uint8_t *blk) {
  std::uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = std::uint32_t(blk[4 * i]) << 24 | std::uint32_t(blk[4 * i + 1]) << 16 |
           std::uint32_t(blk[4 * i + 2]) << 8 | std::uint32_t(blk[4 * i + 3]);
  for (int i = 16; i < 64; ++i) {
    const std::uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const std::uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  std::uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
  for (int i = 0; i < 64; ++i) {
    const std::uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const std::uint32_t ch = (e & f) ^ (~e & g);
    const std::uint32_t t1 = k + S1 + ch + kSha[i] + w[i];
    const std::uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const std::uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    const std::uint32_t t2 = S0 + mj;
    k = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}
}  // namespace

std::array<std::uint8_t, 32> sha256(const std::uint8_t *data, std::size_t size) {
  std::uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                        0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  std::size_t full = size / 64;
  for (std::size_t i = 0; i < full; ++i) sha_block(h, data + 64 * i);
  std::uint8_t tail[128] = {0};
  const std::size_t rem = size - 64 * full;
  if (rem) std::memcpy(tail, data + 64 * full, rem);
  tail[rem] = 0x80;
  const std::size_t tail_len = rem + 1 + 8 <= 64 ? 64 : 128;
  const std::uint64_t bits = std::uint64_t(size) * 8;
  for (int i = 0; i < 8; ++i) tail[tail_len - 1 - i] = std::uint8_t(bits >> (8 * i));
  sha_block(h, tail);
  if (tail_len == 128) sha_block(h, tail + 64);
  std::array<std::uint8_t, 32> out{};
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 4; ++j) out[4 * i + j] = std::uint8_t(h[i] >> (24 - 8 * j));
  return out;
}

std::string sha256_hex(const std::uint8_t *data, std::size_t size) {
  const auto d = sha256(data, size);
  std::ostringstream o;
  o << std::hex << std::setfill('0');
  for (auto b : d) o << std::setw(2) << unsigned(b);
  return o.str();
}

// ---- JSON -------------------------------------------------------------------
class JsonParser {
 public:
  explicit JsonParser(const std::string &s) : s_(s) {}
  Json run() {
    Json v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters in manifest JSON");
    return v;
  }

 private:
  const std::string &s_;
  std::size_t i_ = 0;
  int depth_ = 0;  // nesting of objects and arrays, bounded so a hostile file cannot exhaust the stack
  static constexpr int kMaxDepth = 64;
  bool digit(std::size_t k) const { return k < s_.size() && s_[k] >= '0' && s_[k] <= '9'; }
  // end of the JSON number starting at j: -?(0|[1-9][0-9]*)(.[0-9]+)?([eE][+-]?[0-9]+)?
  std::size_t number_end(std::size_t j) const {
    if (j < s_.size() && s_[j] == '-') ++j;
    if (!digit(j)) fail("malformed manifest JSON value");
    if (s_[j] == '0') {
      ++j;
    } else {
      while (digit(j)) ++j;
    }
    if (j < s_.size() && s_[j] == '.') {
      if (!digit(++j)) fail("malformed manifest JSON number");
      while (digit(j)) ++j;
    }
    if (j < s_.size() && (s_[j] == 'e' || s_[j] == 'E')) {
      ++j;
      if (j < s_.size() && (s_[j] == '+' || s_[j] == '-')) ++j;
      if (!digit(j)) fail("malformed manifest JSON number");
      while (digit(j)) ++j;
    }
    return j;
  }
  void ws() {
    while (i_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[i_]))) ++i_;
  }
  char peek() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end of manifest JSON");
    return s_[i_];
  }
  void expect(char c) {
    if (peek() != c) fail(std::string("malformed manifest JSON: expected '") + c + "'");
    ++i_;
  }
  std::string string() {
    expect('"');
    std::string out;
    while (true) {
      if (i_ >= s_.size()) fail("unterminated JSON string");
      char c = s_[i_++];
      if (c == '"') break;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (i_ >= s_.size()) fail("bad JSON escape");
      char e = s_[i_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (i_ + 4 > s_.size()) fail("bad JSON unicode escape");
          unsigned code = 0;
          for (int k = 0; k < 4; ++k) {
            const char h = s_[i_++];
            const int v = h >= '0' && h <= '9' ? h - '0'
                          : h >= 'a' && h <= 'f' ? h - 'a' + 10
                          : h >= 'A' && h <= 'F' ? h - 'A' + 10 : -1;
            if (v < 0) fail("bad JSON unicode escape");
            code = code * 16 + unsigned(v);
          }
          if (code < 0x80) {
            out.push_back(char(code));
          } else if (code < 0x800) {
            out.push_back(char(0xC0 | (code >> 6)));
            out.push_back(char(0x80 | (code & 0x3F)));
          } else {
            out.push_back(char(0xE0 | (code >> 12)));
            out.push_back(char(0x80 | ((code >> 6) & 0x3F)));
            out.push_back(char(0x80 | (code & 0x3F)));
          }
          break;
        }
        default: fail("bad JSON escape");
      }
    }
    return out;
  }
  Json value() {
    Json v;
    const char c = peek();
    if ((c == '{' || c == '[') && ++depth_ > kMaxDepth) fail("manifest JSON is nested too deeply");
    if (c == '{') {
      ++i_;
      Json::Object obj;
      if (peek() == '}') {
        ++i_;
      } else {
        while (true) {
          std::string key = string();
          expect(':');
          if (!obj.emplace(key, value()).second) fail("duplicate JSON key " + key);
          if (peek() == ',') { ++i_; continue; }
          expect('}');
          break;
        }
      }
      v.v_ = std::move(obj);
      --depth_;
    } else if (c == '[') {
      ++i_;
      Json::Array arr;
      if (peek() == ']') {
        ++i_;
      } else {
        while (true) {
          arr.push_back(value());
          if (peek() == ',') { ++i_; continue; }
          expect(']');
          break;
        }
      }
      v.v_ = std::move(arr);
      --depth_;
    } else if (c == '"') {
      v.v_ = string();
    } else if (s_.compare(i_, 4, "true") == 0) {
      i_ += 4; v.v_ = true;
    } else if (s_.compare(i_, 5, "false") == 0) {
      i_ += 5; v.v_ = false;
    } else if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4; v.v_ = nullptr;
    } else {
      const std::size_t end = number_end(i_);
      const double d = std::strtod(s_.substr(i_, end - i_).c_str(), nullptr);
      if (!std::isfinite(d)) fail("manifest JSON number out of range");
      i_ = end;
      v.v_ = d;
    }
    return v;
  }
};

Json Json::parse(const std::string &text) { return JsonParser(text).run(); }
bool Json::has(const std::string &key) const {
  const auto *o = std::get_if<Object>(&v_);
  return o && o->count(key);
}
const Json &Json::at(const std::string &key) const {
  const auto *o = std::get_if<Object>(&v_);
  if (!o) fail("JSON value is not an object (looking up '" + key + "')");
  auto it = o->find(key);
  if (it == o->end()) fail("manifest is missing key '" + key + "'");
  return it->second;
}
const Json::Array &Json::array() const {
  const auto *a = std::get_if<Array>(&v_);
  if (!a) fail("JSON value is not an array");
  return *a;
}
const Json::Object &Json::object() const {
  const auto *o = std::get_if<Object>(&v_);
  if (!o) fail("JSON value is not an object");
  return *o;
}
const std::string &Json::str() const {
  const auto *s = std::get_if<std::string>(&v_);
  if (!s) fail("JSON value is not a string");
  return *s;
}
double Json::num() const {
  const auto *d = std::get_if<double>(&v_);
  if (!d) fail("JSON value is not a number");
  return *d;
}
bool Json::boolean() const {
  if (const auto *b = std::get_if<bool>(&v_)) return *b;
  if (const auto *d = std::get_if<double>(&v_)) return *d != 0.0;
  fail("JSON value is not a boolean");
}
std::uint64_t Json::uint() const {
  const double d = num();
  if (d < 0 || std::floor(d) != d || d > 9007199254740991.0) fail("JSON value is not an exact unsigned integer");
  return std::uint64_t(d);
}

// ---- model file -------------------------------------------------------------
Model Model::load(const std::string &path) {
  // a regular file of bounded size (a device such as /dev/zero never ends)
  std::error_code ec;
  const auto st = std::filesystem::status(path, ec);
  if (ec || !std::filesystem::exists(st)) fail("cannot open " + path);
  if (!std::filesystem::is_regular_file(st)) fail("cannot open " + path + ": not a regular file");
  const std::uintmax_t size = std::filesystem::file_size(path, ec);
  if (ec) fail("cannot open " + path);
  if (size > (std::uintmax_t(1) << 32)) fail(path + " is larger than 4 GiB");
  std::ifstream in(path, std::ios::binary);
  if (!in) fail("cannot open " + path);
  std::vector<std::uint8_t> bytes(static_cast<std::size_t>(size));
  in.read(reinterpret_cast<char *>(bytes.data()), static_cast<std::streamsize>(size));
  if (static_cast<std::uintmax_t>(in.gcount()) != size) fail("cannot read " + path);
  return load_bytes(std::move(bytes), path);
}

static std::size_t dtype_width(const std::string &d) {
  if (d == "float64" || d == "int64") return 8;
  if (d == "float32" || d == "int32") return 4;
  if (d == "uint8" || d == "bool") return 1;
  fail("unsupported tensor dtype " + d);
}

Model Model::load_bytes(std::vector<std::uint8_t> bytes, const std::string &origin) {
  constexpr std::size_t header = 128;
  static const std::uint8_t magic[8] = {'S', 'O', '3', 'L', 'R', 'N', '1', 0};
  if (bytes.size() < header) fail(origin + ": file is shorter than the 128-byte header");
  if (std::memcmp(bytes.data(), magic, 8) != 0) fail(origin + ": wrong magic");
  if (le32(bytes.data() + 8) != 1 || le32(bytes.data() + 12) != 0) fail("unsupported version or flags");
  const std::size_t msize = std::size_t(le64(bytes.data() + 16));
  const std::size_t psize = std::size_t(le64(bytes.data() + 24));
  if (msize > bytes.size() - header || psize != bytes.size() - header - msize) fail("header length mismatch");
  for (std::size_t i = 96; i < 128; ++i)
    if (bytes[i]) fail("nonzero reserved header bytes");
  const std::uint8_t *mdata = bytes.data() + header;
  const std::uint8_t *pdata = mdata + msize;
  const auto mdig = sha256(mdata, msize);
  const auto pdig = sha256(pdata, psize);
  if (std::memcmp(mdig.data(), bytes.data() + 32, 32) != 0) fail("manifest SHA-256 mismatch");
  if (std::memcmp(pdig.data(), bytes.data() + 64, 32) != 0) fail("payload SHA-256 mismatch");

  Model m;
  m.manifest_ = Json::parse(std::string(reinterpret_cast<const char *>(mdata), msize));
  const Json &man = m.manifest_;
  if (man.at("format").str() != "so3lr-native" || man.at("format_version").uint() != 1)
    fail("manifest format mismatch");
  if (man.at("endianness").str() != "little" || man.at("tensor_alignment").uint() != 64)
    fail("manifest endianness/alignment mismatch");
  if (man.at("model_family").str() != "SO3LR") fail("wrong model family");

  std::set<std::string> names, keys;
  std::size_t prev_end = 0, total = 0;
  for (const Json &item : man.at("tensors").array()) {
    TensorRecord t;
    t.name = item.at("name").str();
    t.state_key = item.at("state_key").str();
    t.dtype = item.at("dtype").str();
    t.role = item.at("role").str();
    t.sha = item.at("sha256").str();
    t.offset = std::size_t(item.at("offset").uint());
    t.nbytes = std::size_t(item.at("nbytes").uint());
    for (const Json &e : item.at("shape").array()) t.shape.push_back(std::size_t(e.uint()));
    if (!names.insert(t.name).second || !keys.insert(t.state_key).second) fail("duplicate tensor name/state key");
    std::size_t elems = 1, bytes_needed = 0;  // shape product without wrap-around
    for (auto e : t.shape)
      if (__builtin_mul_overflow(elems, e, &elems)) fail("tensor shape overflows: " + t.state_key);
    if (__builtin_mul_overflow(elems, dtype_width(t.dtype), &bytes_needed)) fail("tensor shape overflows: " + t.state_key);
    if (t.offset % 64 != 0 || t.nbytes != bytes_needed) fail("tensor alignment/size mismatch: " + t.state_key);
    if (t.offset < prev_end || t.offset > psize || t.nbytes > psize - t.offset) fail("tensor overlap/range error: " + t.state_key);
    for (std::size_t p = prev_end; p < t.offset; ++p)
      if (pdata[p]) fail("nonzero payload padding");
    if (sha256_hex(pdata + t.offset, t.nbytes) != t.sha) fail("per-tensor SHA-256 mismatch: " + t.state_key);
    prev_end = t.offset + t.nbytes;
    total += t.nbytes;
    m.by_key_.emplace(t.state_key, m.tensors_.size());
    m.tensors_.push_back(std::move(t));
  }
  if (prev_end != psize) fail("unreferenced trailing payload bytes");
  if (man.at("tensor_count").uint() != m.tensors_.size() || man.at("tensor_bytes").uint() != total)
    fail("tensor totals mismatch");
  m.bytes_ = std::move(bytes);
  m.payload_ = header + msize;
  m.describe_and_negotiate();
  return m;
}

const TensorRecord &Model::tensor(const std::string &key) const {
  auto it = by_key_.find(key);
  if (it == by_key_.end()) fail("missing tensor " + key);
  return tensors_[it->second];
}

std::vector<double> Model::f64(const std::string &key, const std::vector<std::size_t> &shape) const {
  const TensorRecord &t = tensor(key);
  if (t.dtype != "float64" || t.shape != shape) fail("tensor contract mismatch: " + key);
  std::vector<double> out(t.count());
  std::memcpy(out.data(), bytes_.data() + payload_ + t.offset, t.nbytes);
  return out;
}

std::vector<std::int64_t> Model::i64(const std::string &key) const {
  const TensorRecord &t = tensor(key);
  if (t.dtype != "int64") fail("tensor is not int64: " + key);
  std::vector<std::int64_t> out(t.count());
  std::memcpy(out.data(), bytes_.data() + payload_ + t.offset, t.nbytes);
  return out;
}

double Model::arch_number(const std::string &key) const {
  return manifest_.at("architecture").at(key).num();
}

std::size_t Model::parameter_count() const {
  std::size_t n = 0;
  for (const auto &t : tensors_)
    if (t.role == "parameter") n += t.count();
  return n;
}

LongRangeParams Model::long_range() const {
  LongRangeParams p{};
  p.ke = arch_number("lr_electrostatic_ke");
  p.sigma = arch_number("lr_electrostatic_sigma");
  p.cutoff = arch_number("long_range_cutoff_angstrom");
  p.elec_cuton = arch_number("lr_electrostatic_cuton_angstrom");
  p.fine_structure = arch_number("lr_fine_structure");
  p.bohr = arch_number("lr_bohr_angstrom");
  p.hartree = arch_number("lr_hartree_ev");
  p.disp_scale = arch_number("lr_dispersion_scale");
  p.disp_cuton = arch_number("lr_dispersion_cuton_angstrom");
  p.pair_scale = arch_number("lr_pair_scale");
  for (double v : {p.ke, p.sigma, p.cutoff, p.fine_structure, p.bohr, p.hartree, p.disp_scale, p.pair_scale})
    if (!std::isfinite(v) || v <= 0.0) fail("invalid long-range parameter");
  if (!(p.cutoff > p.elec_cuton) || !(p.elec_cuton > 0) || !(p.cutoff > p.disp_cuton) ||
      !(p.disp_cuton > 0) || std::abs(p.pair_scale - 0.5) > 1e-12)
    fail("long-range cutoff/half-pair contract changed");
  return p;
}

ZblParams Model::zbl() const {
  ZblParams z{};
  if (manifest_.at("architecture").at("zbl_cutoff_function").str() != "phys")
    fail("repulsion cutoff contract changed");
  z.ke = arch_number("zbl_ke");
  z.cutoff = arch_number("short_range_cutoff_angstrom");
  z.switch_off = arch_number("zbl_switch_off_angstrom");
  for (double v : {z.ke, z.cutoff, z.switch_off})
    if (!std::isfinite(v) || !(v > 0)) fail("invalid ZBL parameter");
  if (arch_.repulsion == "nlh") {
    // parameter-free NLH: the screening comes from the pair tables
    // (so3lr_repulsion_setup.cpp:17-21, 37-55)
    z.kind = 1;
    const TensorRecord &ta = tensor("physical.nlh_a");
    const TensorRecord &tb = tensor("physical.nlh_b");
    if (ta.shape.size() != 3 || ta.shape[0] == 0 || ta.shape[1] != ta.shape[0] || ta.shape[2] != 3 ||
        tb.shape != ta.shape || ta.dtype != "float64" || tb.dtype != "float64")
      fail("NLH tables physical.nlh_a / nlh_b must be float64 [cap, cap, 3]");
    if (ta.shape[0] > 118) fail("NLH table capacity exceeds 118 elements");
    z.nlh_cap = int(ta.shape[0]);
    return z;
  }
  z.p = arch_number("zbl_p");
  z.d = arch_number("zbl_d");
  double csum = 0;
  for (int k = 0; k < 4; ++k) {
    z.a[k] = arch_number("zbl_a" + std::to_string(k + 1));
    z.c[k] = arch_number("zbl_c" + std::to_string(k + 1));
    if (!(z.a[k] > 0) || !(z.c[k] > 0)) fail("invalid ZBL coefficient");
    csum += z.c[k];
  }
  if (std::abs(csum - 1.0) > 2e-12) fail("normalized ZBL coefficients changed");
  for (double v : {z.ke, z.cutoff, z.switch_off, z.p, z.d})
    if (!std::isfinite(v) || !(v > 0)) fail("invalid ZBL parameter");
  return z;
}

std::string Architecture::summary() const {
  std::ostringstream o;
  o << "layers=" << layers << " features=" << features << " heads=" << heads << "x" << head_width
    << " degrees=[";
  for (std::size_t i = 0; i < degree_repeats.size(); ++i) o << (i ? "," : "") << (degree_repeats[i] - 1) / 2;
  o << "] ev_width=" << ev_width << " rbf=" << rbf << " r_cut=" << sr_cutoff << " r_cut_lr=" << lr_cutoff
    << " repulsion=" << repulsion << " heads={";
  for (std::size_t i = 0; i < output_heads.size(); ++i) o << (i ? "," : "") << output_heads[i];
  o << "}";
  return o.str();
}

// Architecture record + capability negotiation. The kernels of this library are
// compiled for the two released SO3LR widths (F=128: 4 heads of 32, degrees
// 1..4, 32 Bernstein functions; F=256: 8 heads of 32, degrees 1..4 twice, 64
// Bernstein functions), with the optional block operators below, learned ZBL or
// NLH repulsion and energy/charge/Hirshfeld (and C6) heads; everything else is
// refused here, before any device memory exists (so3lr_capabilities.cpp:181-289
// does the same against the reference's own table).
void Model::describe_and_negotiate() {
  const Json &a = manifest_.at("architecture");
  std::vector<std::string> problems;
  auto need = [&](bool ok, const std::string &msg) {
    if (!ok) problems.push_back(msg);
  };
  if (manifest_.at("schema").str() != "so3lr-native-model-v2")
    problems.push_back("schema '" + manifest_.at("schema").str() + "' is not so3lr-native-model-v2");
  static const std::set<std::string> known = {
      "atomic_number_capacity", "attention_head_width", "attention_heads", "avg_num_neighbors",
      "embedding_scale", "energy_theory_level_selected", "euclidean_degree_channels",
      "interaction_blocks", "invariant_features", "layer_norm_epsilon", "long_range_cutoff_angstrom",
      "lr_bohr_angstrom", "lr_dispersion_cuton_angstrom", "lr_dispersion_scale",
      "lr_electrostatic_cuton_angstrom", "lr_electrostatic_ke", "lr_electrostatic_sigma",
      "lr_fine_structure", "lr_hartree_ev", "lr_pair_scale", "layer_normalization_1",
      "layer_normalization_2", "message_normalization", "module_type_registry",
      "native_long_range_observables", "native_long_range_terms", "native_short_range_physical_terms",
      "num_embeddings", "output_heads", "parameter_elements", "physical_reference_table_state_keys",
      "qk_nonlinearity", "qk_norm", "radial_basis_features", "repulsion_type", "residual_mlp_1",
      "residual_mlp_2", "runtime_element_mapping", "short_range_cutoff_angstrom", "state_tensor_count",
      "use_residual_scalars", "use_rms_norm", "zbl_a1", "zbl_a2", "zbl_a3", "zbl_a4", "zbl_c1",
      "zbl_c2", "zbl_c3", "zbl_c4", "zbl_cutoff_function", "zbl_d", "zbl_enabled", "zbl_ke", "zbl_p",
      "zbl_switch_off_angstrom"};
  for (const auto &kv : a.object())
    if (!known.count(kv.first)) problems.push_back("unknown architecture key '" + kv.first + "'");

  Architecture &r = arch_;
  r.layers = int(a.at("interaction_blocks").uint());
  r.features = int(a.at("invariant_features").uint());
  r.heads = int(a.at("attention_heads").uint());
  r.head_width = int(a.at("attention_head_width").uint());
  r.ev_degrees = int(a.at("euclidean_degree_channels").uint());
  r.rbf = int(a.at("radial_basis_features").uint());
  need(r.layers >= 1 && r.layers <= 8, "interaction_blocks must be 1..8");
  // the two compiled widths (so3lr_capabilities.cpp:58-59 lists the same two):
  // F = 128 with 32 radial functions and degrees [1,2,3,4], F = 256 with 64
  // radial functions and the duplicated degrees [1,1,2,2,3,3,4,4]
  need(r.features == 128 || r.features == 256,
       "invariant_features must be 128 or 256 (the widths the kernels are compiled for)");
  const bool wide = r.features == 256;
  const int want_heads = r.features / 32;
  need(r.heads == want_heads && r.head_width == 32,
       "attention must be " + std::to_string(want_heads) + " heads of width 32 for invariant_features = " +
           std::to_string(r.features));
  need(r.ev_degrees == r.heads, "euclidean_degree_channels must equal attention_heads");
  need(r.rbf == r.features / 4, "radial_basis_features must be " + std::to_string(r.features / 4) +
                                    " for invariant_features = " + std::to_string(r.features));
  const std::string block0 = "model.euclidean_transformers.0.euclidean_attention_block.degree_repeats";
  if (has_tensor(block0)) {
    for (auto v : i64(block0)) r.degree_repeats.push_back(int(v));
  }
  const std::vector<int> want_reps = wide ? std::vector<int>({3, 3, 5, 5, 7, 7, 9, 9}) : std::vector<int>({3, 5, 7, 9});
  need(r.degree_repeats == want_reps, wide ? "degree_repeats must be [3,3,5,5,7,7,9,9] for invariant_features = 256"
                                           : "degree_repeats must be [3,5,7,9] for invariant_features = 128");
  // every block declares the same degree layout
  for (int b = 1; b < r.layers; ++b)
    for (const char *part : {".euclidean_attention_block.degree_repeats", ".interaction_block.degree_repeats"}) {
      const std::string key = "model.euclidean_transformers." + std::to_string(b) + part;
      if (has_tensor(key)) {
        std::vector<int> reps;
        for (auto v : i64(key)) reps.push_back(int(v));
        need(reps == r.degree_repeats, key + " differs from block 0's degree layout");
      }
    }
  int off = 0;
  for (int rep : r.degree_repeats) {
    r.degree_offsets.push_back(off);
    off += rep;
  }
  r.ev_width = off;
  r.max_degree = r.degree_repeats.empty() ? 0 : (r.degree_repeats.back() - 1) / 2;
  r.sh_width = r.max_degree * (r.max_degree + 2);  // distinct harmonics l = 1..Lmax
  r.interaction_width = r.features + r.ev_degrees;
  r.sr_cutoff = a.has("short_range_cutoff_angstrom") ? a.at("short_range_cutoff_angstrom").num() : 0.0;
  r.lr_cutoff = a.has("long_range_cutoff_angstrom") ? a.at("long_range_cutoff_angstrom").num() : 0.0;
  need(r.sr_cutoff > 0 && r.lr_cutoff >= r.sr_cutoff, "cutoffs must satisfy 0 < r_sr <= r_lr");
  r.embedding_scale = a.has("embedding_scale") ? a.at("embedding_scale").num() : 1.0;
  need(std::isfinite(r.embedding_scale) && r.embedding_scale > 0, "embedding_scale must be positive");
  r.attention_norm_kind = a.has("message_normalization") ? a.at("message_normalization").str() : "identity";
  if (r.attention_norm_kind == "avg_num_neighbors") {
    need(a.has("avg_num_neighbors"), "avg_num_neighbors missing");
    r.attention_norm = a.has("avg_num_neighbors") ? a.at("avg_num_neighbors").num() : 1.0;
  } else if (r.attention_norm_kind == "sqrt_num_features") {
    r.attention_norm = std::sqrt(double(r.head_width));
  } else if (r.attention_norm_kind == "identity") {
    r.attention_norm = 1.0;
  } else {
    problems.push_back("unsupported message_normalization '" + r.attention_norm_kind + "'");
  }
  r.layer_norm_eps = a.has("layer_norm_epsilon") ? a.at("layer_norm_epsilon").num() : 1e-6;
  auto flag = [&](const char *k, bool dflt) { return a.has(k) ? a.at(k).boolean() : dflt; };
  // optional operators (so3lr_architecture.cpp:369-389): one norm module for
  // both positions (affine LayerNorm or RMSNorm without scale), the second
  // position switchable; the first norm and exactly the first residual MLP are
  // required, as in the reference (post_attention_block0.cpp:386-390)
  const int norm_kind = flag("use_rms_norm", false) ? 1 : 0;
  need(flag("layer_normalization_1", true), "the first block norm must be enabled");
  r.norm1 = norm_kind;
  r.norm2 = flag("layer_normalization_2", true) ? norm_kind : 2;
  r.qk_norm = flag("qk_norm", false);
  r.residual_scalars = flag("use_residual_scalars", false);
  need(flag("residual_mlp_1", true) && !flag("residual_mlp_2", false),
       "exactly residual_mlp_1 must be enabled");
  if (a.has("qk_nonlinearity")) need(a.at("qk_nonlinearity").str() == "identity", "qk_nonlinearity must be identity");
  r.repulsion = a.has("repulsion_type") ? a.at("repulsion_type").str()
                                        : (flag("zbl_enabled", false) ? "zbl_learned" : "none");
  need(r.repulsion == "zbl_learned" || r.repulsion == "nlh",
       "repulsion_type '" + r.repulsion + "' is not implemented (zbl_learned or nlh)");
  if (r.residual_scalars)
    for (const char *k : {"model.resid_lambdas", "model.x0_lambdas"})
      need(has_tensor(k) && tensor(k).dtype == "float64" && tensor(k).shape == std::vector<std::size_t>{std::size_t(r.layers)},
           std::string(k) + " must be a float64 vector of length interaction_blocks");
  for (const Json &h : a.at("output_heads").array()) r.output_heads.push_back(h.str());
  // energy, charge and Hirshfeld (a0) heads in this order, optionally a fourth,
  // the C6 ratio head (output_heads.cpp:273-283)
  const std::vector<std::string> three = {"atomic_energy_output_block", "partial_charges_output_block",
                                          "hirshfeld_output_block"};
  std::vector<std::string> four = three;
  four.push_back("c6_ratios_output_block");
  need(r.output_heads == three || r.output_heads == four,
       "output heads must be [atomic_energy, partial_charges, hirshfeld] or the same plus c6_ratios");
  r.has_c6 = r.output_heads == four;
  r.head_hidden = has_tensor("model.atomic_energy_output_block.layers.0.weight")
                      ? int(tensor("model.atomic_energy_output_block.layers.0.weight").shape.at(0))
                      : 0;
  need(r.head_hidden == 128, "energy head hidden width must be 128");
  // ratio heads: 64 hidden units, 1..64 keys (output_heads.cpp:105-133)
  auto ratio_head = [&](const std::string &prefix, int &hidden, int &keys) {
    const std::string w1 = prefix + ".transform_features.0.weight", w2 = prefix + ".transform_features.2.weight";
    if (!has_tensor(w1) || !has_tensor(w2) || tensor(w1).shape.size() != 2 || tensor(w2).shape.size() != 2) {
      problems.push_back(prefix + ": ratio-head weights missing");
      return;
    }
    hidden = int(tensor(w1).shape[0]);
    keys = int(tensor(w2).shape[0]);
    need(hidden == 64 && int(tensor(w1).shape[1]) == r.features && int(tensor(w2).shape[1]) == hidden &&
             keys >= 1 && keys <= 64,
         prefix + ": ratio heads must have 64 hidden units and 1..64 keys");
  };
  ratio_head("model.hirshfeld_output_block", r.hirshfeld_hidden, r.hirshfeld_keys);
  if (r.has_c6) {
    int c6_hidden = 0;
    ratio_head("model.c6_ratios_output_block", c6_hidden, r.c6_keys);
  }
  need(std::abs(r.layer_norm_eps - 1e-6) < 1e-15, "layer_norm_epsilon must be 1e-6");
  if (problems.empty()) {
    try {  // repulsion parameters and tables
      zbl();
    } catch (const std::exception &e) {
      problems.push_back(e.what());
    }
  }
  if (!problems.empty()) {
    std::string msg = "this build cannot execute the model:";
    for (const auto &p : problems) msg += "\n  - " + p;
    fail(msg);
  }
}

// ---- charge / spin ----------------------------------------------------------
namespace {
double softplus(double x) { return std::max(x, 0.0) + std::log1p(std::exp(-std::abs(x))); }
double silu(double x) { return x / (1.0 + std::exp(-x)); }
}  // namespace

std::vector<double> charge_spin_table(const Model &model, const std::array<std::int64_t, 119> &counts,
                                      double total_charge, double unpaired) {
  const std::size_t w = std::size_t(model.arch().features);
  std::vector<double> table(118 * w, 0.0);
  auto add = [&](const std::string &name, double psi) {
    const std::string base = "model." + name + ".";
    if (!model.has_tensor(base + "Wq.weight")) {
      if (psi != 0.0) throw Error("SO3LR: this model has no " + name + "; it cannot evaluate this charge/spin state");
      return;
    }
    if (psi == 0.0) return;
    const auto wq = model.f64(base + "Wq.weight", {w, 118});
    const auto wk = model.f64(base + "Wk", {2, w});
    const auto wv = model.f64(base + "Wv", {2, w});
    const auto w1 = model.f64(base + "mlp.1.weight", {w, w});
    const auto w3 = model.f64(base + "mlp.3.weight", {w, w});
    const std::size_t row = psi < 0.0 ? 1 : 0;
    const double *k = wk.data() + row * w;
    const double *v = wv.data() + row * w;
    const double inv_sqrt = 1.0 / std::sqrt(double(w));
    std::array<double, 119> y{};
    double den = 0.0;
    for (int z = 1; z <= 118; ++z) {
      if (counts[z] <= 0) continue;
      double qk = 0.0;
      for (std::size_t c = 0; c < w; ++c) qk += wq[c * 118 + std::size_t(z - 1)] * k[c];
      y[z] = softplus(qk * inv_sqrt);
      den += double(counts[z]) * y[z];
    }
    std::vector<double> x(w), h(w), g(w), sx(w), sh(w);
    for (int z = 1; z <= 118; ++z) {
      if (counts[z] <= 0) continue;
      const double a = psi * y[z] / den;
      for (std::size_t c = 0; c < w; ++c) { x[c] = a * v[c]; sx[c] = silu(x[c]); }
      for (std::size_t o = 0; o < w; ++o) {
        double s = 0.0;
        for (std::size_t i = 0; i < w; ++i) s += w1[o * w + i] * sx[i];
        h[o] = s;
      }
      for (std::size_t c = 0; c < w; ++c) sh[c] = silu(h[c]);
      for (std::size_t o = 0; o < w; ++o) {
        double s = 0.0;
        for (std::size_t i = 0; i < w; ++i) s += w3[o * w + i] * sh[i];
        g[o] = s;
      }
      double *out = table.data() + std::size_t(z - 1) * w;
      for (std::size_t c = 0; c < w; ++c) out[c] += x[c] + g[c];
    }
  };
  add("charge_embedding", total_charge);
  add("spin_embedding", unpaired);
  return table;
}

std::string charge_multiplicity_problem(const std::array<std::int64_t, 119> &counts, double total_charge,
                                        double multiplicity) {
  if (!std::isfinite(total_charge) || std::round(total_charge) != total_charge)
    return "the total charge must be an integer";
  if (!std::isfinite(multiplicity) || std::round(multiplicity) != multiplicity || multiplicity < 1.0)
    return "the spin multiplicity must be an integer >= 1";
  // bounds that keep the integer arithmetic below exact (no overflow)
  if (std::fabs(total_charge) > 1e15) return "the total charge is out of range";
  if (multiplicity > 1e15) return "the spin multiplicity is out of range";
  std::int64_t protons = 0;
  for (int z = 1; z <= 118; ++z) {
    if (counts[z] < 0 || counts[z] > (std::int64_t(1) << 40)) return "element counts must be in 0..2^40";
    protons += counts[z] * z;
  }
  const std::int64_t electrons = protons - std::int64_t(total_charge);
  const std::int64_t unpaired = std::int64_t(multiplicity) - 1;
  if (electrons < 0) return "the total charge leaves a negative number of electrons";
  if (unpaired > electrons)
    return "multiplicity " + std::to_string((long long)multiplicity) + " needs more unpaired electrons than the system's " +
           std::to_string((long long)electrons) + " electrons";
  if ((electrons - unpaired) % 2 != 0)
    return std::to_string((long long)electrons) + " electrons cannot have multiplicity " +
           std::to_string((long long)multiplicity) +
           " (an even electron count needs an odd multiplicity and vice versa)";
  return std::string();
}

int element_token_to_z(const std::string &token) {
  if (token.empty()) return 0;
  bool numeric = true;
  for (char c : token) numeric = numeric && std::isdigit(static_cast<unsigned char>(c));
  if (numeric) {
    if (token.size() > 3) return 0;
    const int v = std::stoi(token);
    return v >= 1 && v <= 99 ? v : 0;
  }
  static const char *symbols[100] = {
      "",   "H",  "He", "Li", "Be", "B",  "C",  "N",  "O",  "F",  "Ne", "Na", "Mg", "Al", "Si", "P",  "S",
      "Cl", "Ar", "K",  "Ca", "Sc", "Ti", "V",  "Cr", "Mn", "Fe", "Co", "Ni", "Cu", "Zn", "Ga", "Ge", "As",
      "Se", "Br", "Kr", "Rb", "Sr", "Y",  "Zr", "Nb", "Mo", "Tc", "Ru", "Rh", "Pd", "Ag", "Cd", "In", "Sn",
      "Sb", "Te", "I",  "Xe", "Cs", "Ba", "La", "Ce", "Pr", "Nd", "Pm", "Sm", "Eu", "Gd", "Tb", "Dy", "Ho",
      "Er", "Tm", "Yb", "Lu", "Hf", "Ta", "W",  "Re", "Os", "Ir", "Pt", "Au", "Hg", "Tl", "Pb", "Bi", "Po",
      "At", "Rn", "Fr", "Ra", "Ac", "Th", "Pa", "U",  "Np", "Pu", "Am", "Cm", "Bk", "Cf", "Es"};
  std::string s = token;
  s[0] = char(std::toupper(static_cast<unsigned char>(s[0])));
  for (std::size_t i = 1; i < s.size(); ++i) s[i] = char(std::tolower(static_cast<unsigned char>(s[i])));
  for (int z = 1; z <= 99; ++z)
    if (s == symbols[z]) return z;
  return 0;
}

}  // namespace so3lr_b200
