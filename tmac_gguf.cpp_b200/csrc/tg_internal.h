// tg_internal.h -- helpers shared between the library's source files (not
// part of the C ABI).
#pragma once

#include "tg_cuda_backend.h"

namespace tg {
// Sets the calling thread's tg_last_error() message; returns code.
int set_last_error(int code, const char* msg);
// CUDA device of a context (TG_ERR_INVALID_ARG for a null context).
int context_device(tg_context* ctx, int* device);
}  // namespace tg
