// Oracle-only stand-in for abseil's CHECK family (aborts on failure).
#pragma once
#include <cstdio>
#include <cstdlib>
#define CHECK(c) do { if (!(c)) { std::fprintf(stderr, "CHECK failed: %s\n", #c); std::abort(); } } while (0)
#define CHECK_EQ(a, b) CHECK((a) == (b))
#define CHECK_LT(a, b) CHECK((a) < (b))
#define CHECK_LE(a, b) CHECK((a) <= (b))
#ifdef NDEBUG
#define DCHECK(c) do { } while (0)
#else
#define DCHECK(c) CHECK(c)
#endif
#define DCHECK_EQ(a, b) DCHECK((a) == (b))
#define DCHECK_LT(a, b) DCHECK((a) < (b))
#define DCHECK_LE(a, b) DCHECK((a) <= (b))
