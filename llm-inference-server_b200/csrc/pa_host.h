// Host-side helpers shared by the C-ABI translation units: thread-local last error.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "paged_attention_b200.h"

namespace pa {

// Formats the calling thread's last-error message and returns `code`.
int32_t fail(int32_t code, const char* fmt, ...);

// Clears the calling thread's record of the kernels its last attention call launched.
void reset_last_launches();

// The checks pa_paged_attention_fwd makes before it looks at any pointer or workspace:
// dtype, head shape, and that `plan` was built for this token count and block size.
int32_t check_attention_args(int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t block_size,
                             int32_t num_kv_heads, int32_t dtype, const pa_step_plan* plan);

}  // namespace pa
