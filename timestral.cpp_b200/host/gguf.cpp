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
        case 12: return ne0 % 256 ? 0 : size_t(ne0 / 256) * 144;   // Q4_K
        case 13: return ne0 % 256 ? 0 : size_t(ne0 / 256) * 176;   // Q5_K
        case 14: return ne0 % 256 ? 0 : size_t(ne0 / 256) * 210;   // Q6_K
    }
    return 0;
}

namespace {
float half_to_float(const uint8_t* p) {
    uint16_t h;
    std::memcpy(&h, p, 2);
    const uint32_t sign = uint32_t(h >> 15) << 31, exp = (h >> 10) & 31, man = h & 1023;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {   // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do { m <<= 1; ++e; } while (!(m & 1024));
            bits = sign | uint32_t(127 - 15 - e) << 23 | (m & 1023) << 13;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | man << 13;
    } else {
        bits = sign | (exp + 112) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
// Six-bit scale and min of sub-block j (0..7) of a Q4_K/Q5_K super-block: bytes 0-3 hold the
// low six bits of scales 0-3, bytes 4-7 those of mins 0-3, bytes 8-11 the low four bits of
// scales/mins 4-7 whose top two bits sit in the top bits of bytes 0-7.
void scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
}  // namespace

bool scaled_int8_row(uint32_t type, const uint8_t* src, int64_t ne0, int8_t* q, float* a, float* b) {
    if (ggml_row_bytes(type, ne0) == 0 && ne0 != 0) return false;
    switch (type) {
        case 12:   // Q4_K
        case 13:   // Q5_K
            for (int64_t blk = 0; blk < ne0 / 256; ++blk) {
                const uint8_t* base = src + blk * (type == 12 ? 144 : 176);
                const float d = half_to_float(base), dmin = half_to_float(base + 2);
                const uint8_t* scales = base + 4;
                const uint8_t* qh = base + 16;
                const uint8_t* qs = base + (type == 12 ? 16 : 48);
                for (int g = 0; g < 4; ++g)
                    for (int half = 0; half < 2; ++half) {
                        int sc, m;
                        scale_min_k4(2 * g + half, scales, &sc, &m);
                        const int64_t p0 = blk * 256 + 64 * g + 32 * half;
                        for (int l = 0; l < 32; ++l) {
                            int v = half ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 0xF);
                            if (type == 13) v |= ((qh[l] >> (2 * g + half)) & 1) << 4;
                            q[p0 + l] = int8_t(v);
                        }
                        for (int k = 0; k < 2; ++k) {
                            a[p0 / 16 + k] = d * float(sc);
                            b[p0 / 16 + k] = dmin * float(m);
                        }
                    }
            }
            return true;
        case 14:   // Q6_K
            for (int64_t blk = 0; blk < ne0 / 256; ++blk) {
                const uint8_t* ql = src + blk * 210;
                const uint8_t* qh = ql + 128;
                const int8_t* sc = reinterpret_cast<const int8_t*>(ql + 192);
                const float d = half_to_float(ql + 208);
                for (int h = 0; h < 2; ++h) {
                    const uint8_t* l0 = ql + 64 * h;
                    const uint8_t* h0 = qh + 32 * h;
                    const int64_t p0 = blk * 256 + 128 * h;
                    for (int l = 0; l < 32; ++l) {
                        q[p0 + l] = int8_t(int((l0[l] & 0xF) | (((h0[l] >> 0) & 3) << 4)) - 32);
                        q[p0 + l + 32] = int8_t(int((l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4)) - 32);
                        q[p0 + l + 64] = int8_t(int((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32);
                        q[p0 + l + 96] = int8_t(int((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32);
                    }
                    // 16-value group j of this half: quadrant j / 2, scale index is + 2 * quadrant.
                    for (int j = 0; j < 8; ++j) {
                        a[p0 / 16 + j] = d * float(sc[8 * h + (j & 1) + 2 * (j >> 1)]);
                        b[p0 / 16 + j] = 0.f;
                    }
                }
            }
            return true;
        case 8:    // Q8_0
            for (int64_t blk = 0; blk < ne0 / 32; ++blk) {
                const uint8_t* base = src + blk * 34;
                const float d = half_to_float(base);
                for (int j = 0; j < 32; ++j) q[blk * 32 + j] = int8_t(base[2 + j]);
                a[blk * 2] = a[blk * 2 + 1] = d;
                b[blk * 2] = b[blk * 2 + 1] = 0.f;
            }
            return true;
        default:
            return false;
    }
}

bool dequantize_row(uint32_t type, const uint8_t* src, int64_t ne0, float* dst) {
    if (ggml_row_bytes(type, ne0) == 0 && ne0 != 0) return false;
    switch (type) {
        case 12:   // Q4_K: d, dmin (f16), scales[12], qs[128]; value = (d*sc) * q - dmin*m
            for (int64_t b = 0; b < ne0 / 256; ++b, src += 144) {
                const float d = half_to_float(src), dmin = half_to_float(src + 2);
                const uint8_t* scales = src + 4;
                const uint8_t* qs = src + 16;
                for (int g = 0; g < 4; ++g) {
                    int sc0, m0, sc1, m1;
                    scale_min_k4(2 * g, scales, &sc0, &m0);
                    scale_min_k4(2 * g + 1, scales, &sc1, &m1);
                    const float d0 = d * float(sc0), mm0 = dmin * float(m0);
                    const float d1 = d * float(sc1), mm1 = dmin * float(m1);
                    for (int l = 0; l < 32; ++l) {
                        const float p0 = d0 * float(qs[32 * g + l] & 0xF);
                        dst[b * 256 + 64 * g + l] = p0 - mm0;
                    }
                    for (int l = 0; l < 32; ++l) {
                        const float p1 = d1 * float(qs[32 * g + l] >> 4);
                        dst[b * 256 + 64 * g + 32 + l] = p1 - mm1;
                    }
                }
            }
            return true;
        case 13:   // Q5_K: d, dmin, scales[12], qh[32], qs[128]; bit j of qh[l] is the fifth bit
                   // of value l of sub-block j
            for (int64_t b = 0; b < ne0 / 256; ++b, src += 176) {
                const float d = half_to_float(src), dmin = half_to_float(src + 2);
                const uint8_t* scales = src + 4;
                const uint8_t* qh = src + 16;
                const uint8_t* qs = src + 48;
                for (int g = 0; g < 4; ++g) {
                    int sc0, m0, sc1, m1;
                    scale_min_k4(2 * g, scales, &sc0, &m0);
                    scale_min_k4(2 * g + 1, scales, &sc1, &m1);
                    const float d0 = d * float(sc0), mm0 = dmin * float(m0);
                    const float d1 = d * float(sc1), mm1 = dmin * float(m1);
                    for (int l = 0; l < 32; ++l) {
                        const int q = (qs[32 * g + l] & 0xF) | (((qh[l] >> (2 * g)) & 1) << 4);
                        const float p0 = d0 * float(q);
                        dst[b * 256 + 64 * g + l] = p0 - mm0;
                    }
                    for (int l = 0; l < 32; ++l) {
                        const int q = (qs[32 * g + l] >> 4) | (((qh[l] >> (2 * g + 1)) & 1) << 4);
                        const float p1 = d1 * float(q);
                        dst[b * 256 + 64 * g + 32 + l] = p1 - mm1;
                    }
                }
            }
            return true;
        case 14:   // Q6_K: ql[128], qh[64], scales[16] (int8), d (f16); value = (d*scale) * (q - 32)
            for (int64_t b = 0; b < ne0 / 256; ++b, src += 210) {
                const uint8_t* ql = src;
                const uint8_t* qh = src + 128;
                const int8_t* sc = reinterpret_cast<const int8_t*>(src + 192);
                const float d = half_to_float(src + 208);
                for (int h = 0; h < 2; ++h) {
                    const uint8_t* l0 = ql + 64 * h;
                    const uint8_t* h0 = qh + 32 * h;
                    const int8_t* s0 = sc + 8 * h;
                    float* y = dst + b * 256 + 128 * h;
                    for (int l = 0; l < 32; ++l) {
                        const int is = l / 16;
                        const int q1 = int((l0[l] & 0xF) | (((h0[l] >> 0) & 3) << 4)) - 32;
                        const int q2 = int((l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4)) - 32;
                        const int q3 = int((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32;
                        const int q4 = int((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32;
                        y[l] = (d * float(s0[is])) * float(q1);
                        y[l + 32] = (d * float(s0[is + 2])) * float(q2);
                        y[l + 64] = (d * float(s0[is + 4])) * float(q3);
                        y[l + 96] = (d * float(s0[is + 6])) * float(q4);
                    }
                }
            }
            return true;
        case 8:    // Q8_0: d (f16), q[32] (int8); value = d * q
            for (int64_t b = 0; b < ne0 / 32; ++b, src += 34) {
                const float d = half_to_float(src);
                for (int j = 0; j < 32; ++j) dst[b * 32 + j] = d * float(int8_t(src[2 + j]));
            }
            return true;
    }
    return false;
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
