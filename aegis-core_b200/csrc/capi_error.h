#pragma once
// Thread-local detail behind aegis_last_error_string(), shared by the C ABI
// translation units.
#include <string>

namespace aegis::capi {
void set_error(const std::string& detail);
}  // namespace aegis::capi
