// Error type and logging of the host library (same role as reference src/common.hpp:6-14).
#pragma once
#include <cstdio>
#include <stdexcept>
#include <string>

#define TS_LOG(...) do { std::fprintf(stderr, "[timestral-b200] " __VA_ARGS__); std::fprintf(stderr, "\n"); } while (0)

namespace ts {

// Thrown for bad input and bad model files; converted to error strings at the C ABI.
struct Error : std::runtime_error {
    explicit Error(const std::string& what) : std::runtime_error(what) {}
};

}  // namespace ts
