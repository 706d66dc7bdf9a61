// Helpers shared by the C ABI translation units.
#pragma once
#include <string>

struct MojoTreesError;

namespace mtb {
// Writes a failed call's reason into the caller's error object (NULL is fine).
void capi_set_error(MojoTreesError* e, const std::string& msg);
void capi_clear_error(MojoTreesError* e);
}  // namespace mtb
