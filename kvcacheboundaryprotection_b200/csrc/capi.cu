// C ABI glue: version, error reporting, policy names, protection sizes.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "../../include/kvbp.h"
#include "kvbp_internal.h"

namespace kvbp {

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

}  // namespace kvbp

extern "C" {

const char* kvbp_version(void) { return "kvbp-b200 0.1 (sm_100a)"; }

const char* kvbp_last_error(void) { return kvbp::g_last_error; }

int kvbp_policy_id(const char* name) {
  if (!name) return -1;
  static const struct {
    const char* n;
    int id;
  } table[] = {
      {"lru", KVBP_POLICY_LRU},
      {"h2o_faithful", KVBP_POLICY_H2O_FAITHFUL},
      {"attention-mass", KVBP_POLICY_H2O_FAITHFUL},
      {"attention_mass", KVBP_POLICY_H2O_FAITHFUL},
      {"h2o", KVBP_POLICY_H2O},
      {"snapkv", KVBP_POLICY_SNAPKV},
      {"snapkv_faithful", KVBP_POLICY_SNAPKV_FAITHFUL},
      {"adakv", KVBP_POLICY_ADAKV},
      {"quest", KVBP_POLICY_QUEST},
      {"streamingllm", KVBP_POLICY_STREAMINGLLM},
      {"random", KVBP_POLICY_RANDOM},
  };
  for (const auto& e : table)
    if (strcmp(e.n, name) == 0) return e.id;
  return -1;
}

void kvbp_protection_sizes(int32_t capacity, double prefix_frac, double suffix_frac, int32_t* n_prefix,
                           int32_t* n_suffix) {
  // max(4, int(cap * frac)) if frac > 0 else 0; Python int() truncates toward zero.
  auto sz = [&](double f) -> int32_t {
    if (!(f > 0.0)) return 0;
    const double v = static_cast<double>(capacity) * f;
    const int32_t t = static_cast<int32_t>(trunc(v));
    return t > 4 ? t : 4;
  };
  if (n_prefix) *n_prefix = sz(prefix_frac);
  if (n_suffix) *n_suffix = sz(suffix_frac);
}

}  // extern "C"
