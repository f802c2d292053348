// Minimal GGUF (v2/v3) reader over a read-only file mapping: key/values and tensor infos.
// Replaces the gguf part of ggml that the reference loader uses (reference
// src/model_loader.cpp:16-47 KV access, :255-306 tensor placement).
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ts {

enum class GgufType : uint32_t {
    U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STRING = 8, ARRAY = 9, U64 = 10,
    I64 = 11, F64 = 12
};
const char* gguf_type_name(GgufType t);

struct GgufValue {
    GgufType type = GgufType::U8;
    GgufType array_type = GgufType::U8;   // for ARRAY
    uint64_t u = 0;                        // unsigned / bool
    int64_t i = 0;                         // signed
    double f = 0;                          // float kinds
    std::string s;
    std::vector<std::string> strings;      // array of strings
    std::vector<double> numbers;           // array of numbers (as double)
};

struct GgufTensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;                     // ggml type id
    uint64_t offset = 0;                   // relative to the data section
};

class MappedFile {
public:
    MappedFile() = default;
    explicit MappedFile(const std::string& path);
    MappedFile(MappedFile&& o) noexcept;
    MappedFile& operator=(MappedFile&& o) noexcept;
    MappedFile(const MappedFile&) = delete;
    MappedFile& operator=(const MappedFile&) = delete;
    ~MappedFile();
    const unsigned char* data() const { return static_cast<const unsigned char*>(base_); }
    size_t size() const { return size_; }

private:
    void release();
    void* base_ = nullptr;
    size_t size_ = 0;
};

class GgufFile {
public:
    // Throws ts::Error on a malformed file.
    explicit GgufFile(const std::string& path);
    const std::map<std::string, GgufValue>& kv() const { return kv_; }
    const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
    size_t data_offset() const { return data_offset_; }
    size_t alignment() const { return alignment_; }
    const MappedFile& file() const { return file_; }
    MappedFile& file() { return file_; }

private:
    MappedFile file_;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensorInfo> tensors_;
    size_t data_offset_ = 0, alignment_ = 32;
};

// Bytes of one row of ne0 elements of ggml type `type` (F32, F16, Q8_0, Q4_K, Q5_K, Q6_K;
// 0 for any other type or a row that is not a whole number of blocks).
size_t ggml_row_bytes(uint32_t type, int64_t ne0);
// Values of one row of a block-quantised ggml type (Q8_0, Q4_K, Q5_K, Q6_K) as float,
// with ggml's published dequantisation (per-block f16 scales and mins; single-precision
// products in the same order). Returns false for other types.
bool dequantize_row(uint32_t type, const uint8_t* src, int64_t ne0, float* dst);
// The same row as integer values q[i] and, per group g of 16 consecutive values, a scale
// a[g] and an offset b[g] such that dequantize_row gives exactly (a[g] * q[i]) - b[g] in
// single precision (b = 0 where the format has no minimum): the form the GEMM's dequantising
// prologue consumes. Q4_K/Q5_K: a = d * scale, b = dmin * min of the 32-value sub-block;
// Q6_K: a = d * scale of the 16 values, q - 32; Q8_0: a = d. Returns false for other types.
bool scaled_int8_row(uint32_t type, const uint8_t* src, int64_t ne0, int8_t* q, float* a, float* b);
const char* ggml_type_name(uint32_t type);

}  // namespace ts
