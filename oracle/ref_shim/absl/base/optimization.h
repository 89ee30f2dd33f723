// Minimal stand-in for the abseil header of the same name, written for the
// oracle build only: it lets the reference sampler sources compile with g++
// and no abseil install.
#pragma once
#define ABSL_PREDICT_FALSE(x) (__builtin_expect(false || (x), false))
#define ABSL_PREDICT_TRUE(x) (__builtin_expect(false || (x), true))
