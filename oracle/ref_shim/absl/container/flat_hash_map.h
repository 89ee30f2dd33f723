// Oracle-only stand-in: absl::flat_hash_map as a std::unordered_map that also
// accepts keys convertible to the key type (abseil's heterogeneous lookup,
// e.g. std::string_view for std::string keys).
#pragma once
#include <string>
#include <type_traits>
#include <unordered_map>
#include <utility>
namespace absl {
template <class K, class V, class H = std::hash<K>, class E = std::equal_to<K>>
class flat_hash_map : public std::unordered_map<K, V, H, E> {
  using Base = std::unordered_map<K, V, H, E>;
 public:
  using Base::Base;
  using Base::try_emplace;
  template <class KK, class... Args,
            class = std::enable_if_t<!std::is_same_v<std::decay_t<KK>, K> &&
                                     std::is_constructible_v<K, const KK&>>>
  std::pair<typename Base::iterator, bool> try_emplace(const KK& k, Args&&... args) {
    return Base::try_emplace(K(k), std::forward<Args>(args)...);
  }
};
}  // namespace absl
