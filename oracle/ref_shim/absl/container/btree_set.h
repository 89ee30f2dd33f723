// Oracle-only stand-in: absl::btree_set as std::set (same ordering).
#pragma once
#include <set>
namespace absl {
template <class K, class C = std::less<K>>
using btree_set = std::set<K, C>;
}  // namespace absl
