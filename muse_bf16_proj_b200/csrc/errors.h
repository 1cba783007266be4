// Per-thread error state shared by the library's translation units.
#pragma once

#include <cstdarg>
#include <cstdio>

namespace muse {

struct ErrorState {
  int code = 0;
  char msg[512] = {0};
};

inline ErrorState& error_state() {
  static thread_local ErrorState s;
  return s;
}

inline void clear_error() {
  error_state().code = 0;
  error_state().msg[0] = '\0';
}

inline int last_code() { return error_state().code; }

// Records (code, message) for muse_last_error() and returns code.
inline int fail(int code, const char* fmt, ...) {
  ErrorState& s = error_state();
  s.code = code;
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(s.msg, sizeof(s.msg), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace muse
