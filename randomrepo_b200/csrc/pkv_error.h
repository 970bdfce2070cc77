// Thread-local error message shared by every C entry point of libpkv_b200.
#pragma once
#include <string>

void pkv_set_error(const std::string& msg);
void pkv_clear_error();
