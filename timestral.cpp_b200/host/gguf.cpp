#include "gguf.hpp"

#include "common.hpp"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace ts {

const char* gguf_type_name(GgufType t) {
    switch (t) {
        case GgufType::U8: return "u8"; case GgufType::I8: return "i8"; case GgufType::U16: return "u16";
        case GgufType::I16: return "i16"; case GgufType::U32: return "u32"; case GgufType::I32: return "i32";
        case GgufType::F32: return "f32"; case GgufType::BOOL: return "bool"; case GgufType::STRING: return "str";
        case GgufType::ARRAY: return "arr"; case GgufType::U64: return "u64"; case GgufType::I64: return "i64";
        case GgufType::F64: return "f64";
    }
    return "?";
}

const char* ggml_type_name(uint32_t t) {
    switch (t) {
        case 0: return "f32"; case 1: return "f16"; case 2: return "q4_0"; case 3: return "q4_1";
        case 6: return "q5_0"; case 7: return "q5_1"; case 8: return "q8_0"; case 12: return "q4_K";
        case 13: return "q5_K"; case 14: return "q6_K"; case 30: return "bf16";
    }
    return "unknown";
}

size_t ggml_row_bytes(uint32_t type, int64_t ne0) {
    if (ne0 < 0) return 0;
    switch (type) {
        case 0: return size_t(ne0) * 4;
        case 1: return size_t(ne0) * 2;
        case 8: return ne0 % 32 ? 0 : size_t(ne0 / 32) * 34;
    }
    return 0;
}

MappedFile::MappedFile(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error("cannot open file: " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); throw Error("cannot stat file: " + path); }
    size_ = size_t(st.st_size);
    if (size_ == 0) { ::close(fd); throw Error("empty file: " + path); }
    base_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (base_ == MAP_FAILED) { base_ = nullptr; throw Error("cannot map file: " + path); }
}
MappedFile::MappedFile(MappedFile&& o) noexcept { *this = std::move(o); }
MappedFile& MappedFile::operator=(MappedFile&& o) noexcept {
    if (this != &o) {
        release();
        base_ = o.base_; size_ = o.size_;
        o.base_ = nullptr; o.size_ = 0;
    }
    return *this;
}
void MappedFile::release() {
    if (base_) munmap(base_, size_);
    base_ = nullptr;
    size_ = 0;
}
MappedFile::~MappedFile() { release(); }

namespace {
struct Cursor {
    const unsigned char* p;
    size_t n, at = 0;
    void need(size_t k) {
        if (k > n || at > n - k) throw Error("truncated GGUF file");
    }
    template <class T> T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (len > (uint64_t(1) << 32)) throw Error("GGUF string too long");
        need(size_t(len));
        std::string s(reinterpret_cast<const char*>(p + at), size_t(len));
        at += size_t(len);
        return s;
    }
};

double scalar(Cursor& c, GgufType t, GgufValue* v) {
    switch (t) {
        case GgufType::U8: { auto x = c.get<uint8_t>(); if (v) v->u = x; return x; }
        case GgufType::I8: { auto x = c.get<int8_t>(); if (v) v->i = x; return x; }
        case GgufType::U16: { auto x = c.get<uint16_t>(); if (v) v->u = x; return x; }
        case GgufType::I16: { auto x = c.get<int16_t>(); if (v) v->i = x; return x; }
        case GgufType::U32: { auto x = c.get<uint32_t>(); if (v) v->u = x; return x; }
        case GgufType::I32: { auto x = c.get<int32_t>(); if (v) v->i = x; return x; }
        case GgufType::F32: { auto x = c.get<float>(); if (v) v->f = x; return x; }
        case GgufType::BOOL: { auto x = c.get<uint8_t>(); if (v) v->u = x != 0; return x != 0; }
        case GgufType::U64: { auto x = c.get<uint64_t>(); if (v) v->u = x; return double(x); }
        case GgufType::I64: { auto x = c.get<int64_t>(); if (v) v->i = x; return double(x); }
        case GgufType::F64: { auto x = c.get<double>(); if (v) v->f = x; return x; }
        default: throw Error("bad GGUF scalar type");
    }
}
}  // namespace

GgufFile::GgufFile(const std::string& path) : file_(path) {
    Cursor c{file_.data(), file_.size()};
    if (c.get<uint32_t>() != 0x46554747u) throw Error("not a GGUF file: " + path);
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) throw Error("unsupported GGUF version " + std::to_string(version));
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (n_tensors > (1u << 20) || n_kv > (1u << 20)) throw Error("implausible GGUF header counts");
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key = c.str();
        GgufValue v;
        v.type = GgufType(c.get<uint32_t>());
        if (v.type == GgufType::STRING) v.s = c.str();
        else if (v.type == GgufType::ARRAY) {
            v.array_type = GgufType(c.get<uint32_t>());
            const uint64_t n = c.get<uint64_t>();
            if (n > (uint64_t(1) << 28)) throw Error("GGUF array too long");
            for (uint64_t i = 0; i < n; ++i) {
                if (v.array_type == GgufType::STRING) v.strings.push_back(c.str());
                else if (v.array_type == GgufType::ARRAY) throw Error("nested GGUF arrays are not supported");
                else v.numbers.push_back(scalar(c, v.array_type, nullptr));
            }
        } else scalar(c, v.type, &v);
        if (!kv_.emplace(key, std::move(v)).second) throw Error("duplicate KV in file: " + key);
    }
    auto al = kv_.find("general.alignment");
    if (al != kv_.end()) {
        if (al->second.type != GgufType::U32 || al->second.u == 0 || (al->second.u & (al->second.u - 1)))
            throw Error("invalid general.alignment");
        alignment_ = size_t(al->second.u);
    }
    for (uint64_t t = 0; t < n_tensors; ++t) {
        GgufTensorInfo ti;
        ti.name = c.str();
        ti.n_dims = c.get<uint32_t>();
        if (ti.n_dims < 1 || ti.n_dims > 4) throw Error("tensor " + ti.name + " has an invalid rank");
        for (uint32_t d = 0; d < ti.n_dims; ++d) {
            const uint64_t ne = c.get<uint64_t>();
            if (ne > (uint64_t(1) << 40)) throw Error("tensor " + ti.name + " has an invalid dimension");
            ti.ne[d] = int64_t(ne);
        }
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        tensors_.push_back(std::move(ti));
    }
    data_offset_ = (c.at + alignment_ - 1) / alignment_ * alignment_;
    if (data_offset_ > file_.size()) throw Error("GGUF data section out of file bounds");
}

}  // namespace ts
