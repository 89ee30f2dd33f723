// Oracle-only stand-in: absl::Span as std::span.
#pragma once
#include <span>
#include <vector>
namespace absl {
template <class T> using Span = std::span<T>;
template <class T> std::span<const T> MakeConstSpan(const std::vector<T>& v) { return std::span<const T>(v.data(), v.size()); }
template <class T> std::span<const T> MakeConstSpan(std::span<T> v) { return std::span<const T>(v.data(), v.size()); }
template <class T> std::span<const T> MakeConstSpan(std::span<const T> v) { return v; }
}  // namespace absl
