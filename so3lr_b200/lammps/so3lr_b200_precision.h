// $SO3LR_B200_PRECISION for the handles of the so3lr/b200 pair styles:
// "float64" (or unset) keeps the reference's float64 arithmetic, "mixed" runs the
// pair-filter GEMMs as three-pass TF32 tensor-core MMAs (so3lr_set_precision).
#pragma once

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "so3lr_b200.h"

inline int so3lr_b200_precision_from_env(so3lr_handle *h, char *err, size_t errlen) {
  const char *p = std::getenv("SO3LR_B200_PRECISION");
  if (p == nullptr || p[0] == '\0' || std::strcmp(p, "float64") == 0) return 0;
  if (std::strcmp(p, "mixed") == 0) return so3lr_set_precision(h, SO3LR_PRECISION_MIXED, err, errlen);
  std::snprintf(err, errlen, "SO3LR_B200_PRECISION must be 'float64' or 'mixed', not '%s'", p);
  return 1;
}
