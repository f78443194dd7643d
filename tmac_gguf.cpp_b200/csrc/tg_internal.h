// tg_internal.h -- helpers shared between the library's source files (not
// part of the C ABI).
#pragma once

namespace tg {
// Sets the calling thread's tg_last_error() message; returns code.
int set_last_error(int code, const char* msg);
}  // namespace tg
