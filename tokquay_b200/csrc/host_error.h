// Thread-local error message behind tq_last_error().
#pragma once

#include <cstdarg>
#include <cstdio>

namespace tq {

// Defined in capi.cu.
char* error_buffer();
constexpr int kErrorBufferLen = 512;

// Formats the message for tq_last_error() and returns `status`.
inline int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(error_buffer(), kErrorBufferLen, fmt, ap);
  va_end(ap);
  return status;
}

}  // namespace tq
