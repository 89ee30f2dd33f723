// Oracle-only stand-in for absl::StrCat / StrAppend (ostream formatting;
// bools print as 0/1 like abseil's integral formatting).
#pragma once
#include <sstream>
#include <string>
namespace absl {
template <class... Args> std::string StrCat(const Args&... args) {
  std::ostringstream os;
  (os << ... << args);
  return os.str();
}
template <class... Args> void StrAppend(std::string* out, const Args&... args) {
  out->append(StrCat(args...));
}
}  // namespace absl
