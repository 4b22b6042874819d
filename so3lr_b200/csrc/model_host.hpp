// Host side of the SO3LR model boundary: `.so3lr` loader, architecture record,
// capability negotiation, charge/spin embedding table and element map.
//
// Mirrors, with an independent implementation:
//   source/so3lr-lammps-native/src/native_model.cpp:338-441  (file format, integrity)
//   source/so3lr-lammps-native/src/so3lr_architecture.cpp:296-450 (architecture record)
//   source/so3lr-lammps-native/src/so3lr_capabilities.cpp:46-289 (refuse what is not implemented)
//   source/so3lr-lammps-native/src/so3lr_charge_spin.cpp:46-141 (charge/spin table, parity)
//   source/so3lr-lammps-native/plugins/lammps/so3lr_element_map.h:19-52 (pair_coeff tokens)
#pragma once

#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <variant>
#include <vector>

namespace so3lr_b200 {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---- minimal JSON value -----------------------------------------------------
class Json {
 public:
  using Object = std::map<std::string, Json>;
  using Array = std::vector<Json>;
  Json() : v_(nullptr) {}
  static Json parse(const std::string &text);
  bool is_object() const { return std::holds_alternative<Object>(v_); }
  bool has(const std::string &key) const;
  const Json &at(const std::string &key) const;
  const Array &array() const;
  const Object &object() const;
  const std::string &str() const;
  double num() const;
  bool boolean() const;  // accepts JSON booleans and 0/1 numbers
  std::uint64_t uint() const;

 private:
  std::variant<std::nullptr_t, bool, double, std::string, Array, Object> v_;
  friend class JsonParser;
};

std::array<std::uint8_t, 32> sha256(const std::uint8_t *data, std::size_t size);
std::string sha256_hex(const std::uint8_t *data, std::size_t size);

struct TensorRecord {
  std::string name, state_key, dtype, role, sha;
  std::vector<std::size_t> shape;
  std::size_t offset = 0, nbytes = 0;
  std::size_t count() const {
    std::size_t c = 1;
    for (auto s : shape) c *= s;
    return c;
  }
};

// Architecture record (the subset the kernels depend on, plus descriptive fields).
struct Architecture {
  int layers = 0, features = 0, heads = 0, head_width = 0, ev_degrees = 0;
  int rbf = 0, ev_width = 0, sh_width = 0, max_degree = 0, interaction_width = 0;
  int head_hidden = 0, hirshfeld_hidden = 0, hirshfeld_keys = 0;
  // optional fourth head: C6 ratios (dispersion C6_i = C6_ref c6_i, alpha from
  // the Hirshfeld / a0 ratio); 0 keys when absent
  bool has_c6 = false;
  int c6_keys = 0;
  std::vector<int> degree_repeats, degree_offsets;
  double sr_cutoff = 0, lr_cutoff = 0, embedding_scale = 1, attention_norm = 1;
  double layer_norm_eps = 1e-6;
  // block norms: 0 = affine LayerNorm, 1 = RMSNorm without scale, 2 = none
  // (second position only)
  int norm1 = 0, norm2 = 0;
  bool qk_norm = false;           // RMS normalisation of q, k per (atom, head)
  bool residual_scalars = false;  // x = resid[b] x + x0[b] x0 before block b
  std::string attention_norm_kind, repulsion;
  std::vector<std::string> output_heads;
  std::string summary() const;
};

// Physics parameters of the long-range and repulsion terms.
struct LongRangeParams {
  double ke, sigma, cutoff, elec_cuton, fine_structure, bohr, hartree, disp_scale,
      disp_cuton, pair_scale;
};
// Short-range repulsion: kind 0 = learned ZBL (p, d, a, c), kind 1 = NLH pair
// tables physical.nlh_a / nlh_b of shape [cap, cap, 3].
struct ZblParams {
  double ke, cutoff, switch_off, p, d, a[4], c[4];
  int kind = 0, nlh_cap = 0;
};

class Model {
 public:
  static Model load(const std::string &path);
  static Model load_bytes(std::vector<std::uint8_t> bytes, const std::string &origin);

  const Json &manifest() const { return manifest_; }
  const Architecture &arch() const { return arch_; }
  const TensorRecord &tensor(const std::string &key) const;
  bool has_tensor(const std::string &key) const { return by_key_.count(key) != 0; }
  // float64 contents of a tensor, shape-checked.
  std::vector<double> f64(const std::string &key, const std::vector<std::size_t> &shape) const;
  std::vector<std::int64_t> i64(const std::string &key) const;
  double arch_number(const std::string &key) const;
  LongRangeParams long_range() const;
  ZblParams zbl() const;
  std::size_t parameter_count() const;

 private:
  std::vector<std::uint8_t> bytes_;
  std::size_t payload_ = 0;
  Json manifest_;
  std::vector<TensorRecord> tensors_;
  std::map<std::string, std::size_t> by_key_;
  Architecture arch_;
  void describe_and_negotiate();
};

// 118 x F composition-only offset table for total charge Q and psi = M - 1
// (so3lr_charge_spin.cpp:46-114). counts[z] for z in 1..118.
std::vector<double> charge_spin_table(const Model &model, const std::array<std::int64_t, 119> &counts,
                                      double total_charge, double unpaired);
// Empty string when (Q, M) is valid for this composition (so3lr_charge_spin.cpp:116-141).
std::string charge_multiplicity_problem(const std::array<std::int64_t, 119> &counts,
                                        double total_charge, double multiplicity);

// pair_coeff token -> Z: element symbol H..Es (case-insensitive) or a number 1..99
// (so3lr_element_map.h:19-52). Returns 0 for an unknown token.
int element_token_to_z(const std::string &token);

}  // namespace so3lr_b200
