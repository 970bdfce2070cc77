// Error reporting and version string of libpkv_b200 (C ABI in include/pkv_b200.h).
#include "pkv_b200.h"
#include "pkv_error.h"

#include <string>

namespace {
thread_local std::string g_last_error;
}

void pkv_set_error(const std::string& msg) { g_last_error = msg; }
void pkv_clear_error() { g_last_error.clear(); }

extern "C" const char* pkv_last_error(void) { return g_last_error.c_str(); }
extern "C" const char* pkv_version(void) { return "pkv_b200 1.0 sm_100a"; }
