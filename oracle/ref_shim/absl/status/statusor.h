// Oracle-only stand-in for absl::StatusOr<T>, including reference types.
#pragma once
#include <optional>
#include <type_traits>
#include <utility>
#include "absl/status/status.h"
namespace absl {
template <class T> class StatusOr {
 public:
  StatusOr(const Status& s) : status_(s) {}
  StatusOr(Status&& s) : status_(std::move(s)) {}
  template <class U, class = std::enable_if_t<std::is_constructible_v<T, U&&> && !std::is_same_v<std::decay_t<U>, Status>>>
  StatusOr(U&& v) : value_(std::forward<U>(v)) {}
  bool ok() const { return status_.ok(); }
  const Status& status() const& { return status_; }
  T& value() & { return *value_; }
  const T& value() const& { return *value_; }
  T&& value() && { return std::move(*value_); }
  T& operator*() & { return *value_; }
  T* operator->() { return &*value_; }
 private:
  Status status_;
  std::optional<T> value_;
};
template <class T> class StatusOr<T&> {
 public:
  StatusOr(const Status& s) : status_(s) {}
  StatusOr(T& v) : ptr_(&v) {}
  bool ok() const { return status_.ok(); }
  const Status& status() const { return status_; }
  T& value() const { return *ptr_; }
  T& operator*() const { return *ptr_; }
 private:
  Status status_;
  T* ptr_ = nullptr;
};
}  // namespace absl
