// Host-side helpers shared by the C-ABI translation units: thread-local last error.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>

namespace pa {

// Formats the calling thread's last-error message and returns `code`.
int32_t fail(int32_t code, const char* fmt, ...);

}  // namespace pa
