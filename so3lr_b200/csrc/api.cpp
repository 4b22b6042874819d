// Width-independent pieces of the evaluator interface: the brick partition of
// a periodic box over GPUs and the choice of the evaluator that matches a
// model's invariant width.
#include "api.hpp"

#include <cmath>

namespace so3lr_b200 {

static int brick_of(const double *x, const SystemSpec &s, const int dims[3]) {
  int idx[3];
  for (int d = 0; d < 3; ++d) {
    double p = x[d] - s.lo[d];
    p -= std::floor(p / s.len[d]) * s.len[d];
    int c = int(p * dims[d] / s.len[d]);
    idx[d] = c < 0 ? 0 : (c >= dims[d] ? dims[d] - 1 : c);
  }
  return (idx[2] * dims[1] + idx[1]) * dims[0] + idx[0];
}

void brick_dims(int nranks, int dims[3]) {
  dims[0] = dims[1] = dims[2] = 1;
  int rest = nranks;
  for (int f = 2; rest > 1;) {
    if (rest % f == 0) {
      // give the factor to the dimension with the fewest bricks, z first
      int k = 2;
      if (dims[1] < dims[k]) k = 1;
      if (dims[0] < dims[k]) k = 0;
      dims[k] *= f;
      rest /= f;
    } else {
      ++f;
    }
  }
}

std::vector<int> partition_atoms(const SystemSpec &s, const double *x, int nranks) {
  std::vector<int> owner(std::size_t(s.n), 0);
  if (nranks == 1) return owner;
  int dims[3];
  brick_dims(nranks, dims);
  for (int i = 0; i < s.n; ++i) owner[std::size_t(i)] = brick_of(x + 3 * std::size_t(i), s, dims);
  return owner;
}

std::unique_ptr<EvaluatorApi> make_evaluator(const std::string &model_path, int device) {
  Model model = Model::load(model_path);
  const int f = model.arch().features;
  if (f == 128) return create_evaluator_f128(std::move(model), device);
  if (f == 256) return create_evaluator_f256(std::move(model), device);
  throw Error("SO3LR: no evaluator for invariant_features = " + std::to_string(f));
}

}  // namespace so3lr_b200
