// extern "C" entry points over the reference's own host code, so the oracle
// tests can compare against it (test infrastructure only; built into
// oracle/_ref/ by `make -C oracle ref`, never committed as a binary).
#include <cstring>
#include <string>
#include <vector>

#include "config.h"

extern "C" {

// Parses a config.json document with lcr::ModelConfig::from_json_string
// (src/config.cpp:46-133) and writes lcr::compute_rope_inv_freq
// (src/config.cpp:223-259) into out. Returns the number of entries, or -1 and
// the error message in err.
int ref_rope_inv_freq(const char* config_json, float* out, int capacity,
                      char* err, int err_len) {
  try {
    const lcr::ModelConfig c = lcr::ModelConfig::from_json_string(config_json);
    const std::vector<float> f = lcr::compute_rope_inv_freq(c);
    const int n = static_cast<int>(f.size());
    for (int i = 0; i < n && i < capacity; ++i) out[i] = f[static_cast<size_t>(i)];
    return n;
  } catch (const std::exception& e) {
    if (err && err_len > 0) {
      std::strncpy(err, e.what(), static_cast<size_t>(err_len - 1));
      err[err_len - 1] = 0;
    }
    return -1;
  }
}

}  // extern "C"
