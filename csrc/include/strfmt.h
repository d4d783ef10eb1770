// strfmt.h - printf-style std::string formatting.  The extension builds no
// iostreams: their locale facets are resolved against whatever libstdc++ the
// host process loaded, which need not match the compiler's headers.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace rab {

inline std::string strfmt(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
inline std::string strfmt(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  const int n = vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (n < 0) return std::string("<format error>");
  if (static_cast<size_t>(n) < sizeof(buf)) return std::string(buf, static_cast<size_t>(n));
  std::string out(static_cast<size_t>(n) + 1, '\0');
  va_start(ap, fmt);
  vsnprintf(&out[0], out.size(), fmt, ap);
  va_end(ap);
  out.resize(static_cast<size_t>(n));
  return out;
}

}  // namespace rab

// Argument check for the Python bindings: throws std::runtime_error (a Python
// RuntimeError through pybind11) with a printf-style message.  Used instead of
// TORCH_CHECK, whose message builder goes through std::ostringstream.
#define RAB_CHECK(cond, ...)                                      \
  do {                                                            \
    if (!(cond)) throw std::runtime_error(::rab::strfmt(__VA_ARGS__)); \
  } while (0)
