// Oracle-only stand-in for absl::StrJoin with and without a formatter.
#pragma once
#include <sstream>
#include <string>
namespace absl {
template <class Range, class Fmt>
std::string StrJoin(const Range& range, const std::string& sep, Fmt&& fmt) {
  std::string out;
  bool first = true;
  for (const auto& v : range) {
    if (!first) out += sep;
    first = false;
    fmt(&out, v);
  }
  return out;
}
template <class Range>
std::string StrJoin(const Range& range, const std::string& sep) {
  return StrJoin(range, sep, [](std::string* out, const auto& v) {
    std::ostringstream os;
    os << v;
    out->append(os.str());
  });
}
}  // namespace absl
