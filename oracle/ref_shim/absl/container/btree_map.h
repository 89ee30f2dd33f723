// Oracle-only stand-in: absl::btree_map as std::map (same ordering).
#pragma once
#include <map>
namespace absl {
template <class K, class V, class C = std::less<K>>
using btree_map = std::map<K, V, C>;
}  // namespace absl
