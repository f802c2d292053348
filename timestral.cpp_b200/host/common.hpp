// Error type and logging of the host library (same role as reference src/common.hpp:6-14).
#pragma once
#include <cstdio>
#include <stdexcept>
#include <string>

// The C++ API (ts::Model, ts::Forecaster, ts::Error, assemble_rows) is exported from the
// shared library; everything else in it is hidden.
#define TS_API __attribute__((visibility("default")))

#define TS_LOG(...) do { std::fprintf(stderr, "[timestral-b200] " __VA_ARGS__); std::fprintf(stderr, "\n"); } while (0)

namespace ts {

// Thrown for bad input and bad model files; converted to error strings at the C ABI.
struct TS_API Error : std::runtime_error {
    explicit Error(const std::string& what) : std::runtime_error(what) {}
};

}  // namespace ts
