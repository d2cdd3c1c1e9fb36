// Argument checks of the host entry points.
//
// SB_CHECK(cond, parts...) is TORCH_CHECK with the message assembled without iostreams: numbers go
// through std::to_string and the finished text reaches TORCH_CHECK as one C string.  In a Python
// process whose C++ runtime pieces disagree (a framework library that carries its own copy of the
// C++ standard library next to the system one), formatting a number through an ostream inside an
// extension module can crash the process instead of producing the error text; this path avoids
// that, so a bad argument always ends as a Python RuntimeError.
#pragma once

#include <c10/util/Exception.h>

#include <string>
#include <type_traits>

namespace sb {
namespace detail {

inline void check_append(std::string& s, const char* v) { s += v; }
inline void check_append(std::string& s, const std::string& v) { s += v; }
template <class T>
inline std::enable_if_t<std::is_arithmetic_v<T>> check_append(std::string& s, T v) {
  s += std::to_string(v);
}
template <class... A>
inline std::string check_msg(const A&... a) {
  std::string s;
  (check_append(s, a), ...);
  return s;
}

}  // namespace detail
}  // namespace sb

#define SB_CHECK(cond, ...) TORCH_CHECK((cond), ::sb::detail::check_msg(__VA_ARGS__).c_str())
