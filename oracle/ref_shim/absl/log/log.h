// Oracle-only stand-in for abseil logging: LOG(severity) << ... goes to stderr.
#pragma once
#include <iostream>
#include "absl/log/check.h"
namespace absl_shim {
struct LogLine {
  ~LogLine() { std::cerr << std::endl; }
  template <class T> LogLine& operator<<(const T& v) { std::cerr << v; return *this; }
};
}  // namespace absl_shim
#define LOG(severity) ::absl_shim::LogLine()
