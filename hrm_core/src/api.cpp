// C ABI over hrm::Engine (see include/hrm/api.h).  Errors are reported through a thread-local message.
#include "hrm/api.h"
#include "hrm/hrm.h"

#include <cstdlib>
#include <cstring>
#include <string>

struct hrm_handle_t {
  hrm::Engine engine;
};

namespace {
thread_local std::string g_err;

char* dup_c(const std::string& s) {
  char* p = static_cast<char*>(std::malloc(s.size() + 1));
  if (p) {
    std::memcpy(p, s.data(), s.size());
    p[s.size()] = '\0';
  }
  return p;
}
}  // namespace

extern "C" {

hrm_handle_t* hrm_open(const char* model_dir) {
  if (!model_dir) {
    g_err = "hrm_open: model_dir is null";
    return nullptr;
  }
  auto* h = new (std::nothrow) hrm_handle_t();
  if (!h) {
    g_err = "hrm_open: out of memory";
    return nullptr;
  }
  try {
    h->engine.open(model_dir);
    return h;
  } catch (const std::exception& e) {
    g_err = std::string("hrm_open failed: ") + e.what();
    delete h;
    return nullptr;
  }
}

void hrm_close(hrm_handle_t* h) { delete h; }

char* hrm_query_json(hrm_handle_t* h, const char* prompt_utf8, int top_k, int top_m, int k, int lam_num,
                     int lam_den) {
  if (!h || !h->engine.is_open()) {
    g_err = "hrm_query_json: handle not open";
    return nullptr;
  }
  if (!prompt_utf8) {
    g_err = "hrm_query_json: prompt is null";
    return nullptr;
  }
  try {
    hrm::QueryParams qp{top_k, top_m, k, lam_num, lam_den};
    const std::string prompt(prompt_utf8);
    char* out = dup_c(hrm::result_json(prompt, h->engine.query(prompt, qp)));
    if (!out) g_err = "hrm_query_json: out of memory";
    return out;
  } catch (const std::exception& e) {
    g_err = std::string("hrm_query_json failed: ") + e.what();
    return nullptr;
  }
}

void hrm_free(void* p) { std::free(p); }

const char* hrm_last_error(void) { return g_err.c_str(); }

}  // extern "C"
