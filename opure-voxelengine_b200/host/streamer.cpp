// streamer.cpp -- safetensors mapping: u64 little-endian header length, a JSON header
// {"name": {"dtype", "shape", "data_offsets": [begin, end], "scale"?}}, then the payload;
// data_offsets are relative to the payload start (Opure_Streamer.h:12-24).
#include "streamer.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "json.h"
#include "platform.h"

namespace opure::safetensors {

const char *DtypeName(Dtype d) {
    switch (d) {
        case Dtype::F32: return "F32";
        case Dtype::F16: return "F16";
        case Dtype::BF16: return "BF16";
        case Dtype::U8: return "U8";
        case Dtype::I8: return "I8";
        case Dtype::U4: return "U4";
        case Dtype::I4: return "I4";
        default: return "?";
    }
}

Dtype ParseDtype(std::string_view s) {
    if (s == "F32") return Dtype::F32;
    if (s == "F16") return Dtype::F16;
    if (s == "BF16") return Dtype::BF16;
    if (s == "U8") return Dtype::U8;
    if (s == "I8") return Dtype::I8;
    if (s == "U4") return Dtype::U4;
    if (s == "I4") return Dtype::I4;
    ThrowError("unsupported safetensors dtype '" + std::string(s) + "'");
}

uint64_t StorageBytes(Dtype d, uint64_t n) {
    switch (d) {
        case Dtype::F32: return n * 4;
        case Dtype::F16:
        case Dtype::BF16: return n * 2;
        case Dtype::U8:
        case Dtype::I8: return n;
        case Dtype::U4:
        case Dtype::I4: return (n + 1) / 2;
        default: return 0;
    }
}

uint64_t Tensor::ElementCount() const {
    uint64_t n = 1;
    for (int64_t d : shape) {
        OPURE_CHECK(d >= 0, "safetensors tensor '" + name + "' has a negative dimension");
        n *= uint64_t(d);
    }
    return n;
}

uint64_t Tensor::Rows() const {
    uint64_t r = 1;
    for (size_t i = 0; i + 1 < shape.size(); ++i) r *= uint64_t(shape[i]);
    return r;
}

uint64_t Tensor::Cols() const { return shape.empty() ? 1 : uint64_t(shape.back()); }

void WeightStreamer::Open(const std::string &path) {
    Close();
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) ThrowError("cannot open safetensors file '" + path + "'");
    struct stat sb {};
    if (::fstat(fd, &sb) != 0 || sb.st_size <= 8) {
        ::close(fd);
        ThrowError("safetensors file is too small to contain a length prefix");
    }
    const uint64_t bytes = uint64_t(sb.st_size);
    void *m = ::mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);  // the mapping stays valid
    if (m == MAP_FAILED) ThrowError("mmap failed on '" + path + "'");
    base_ = static_cast<uint8_t *>(m);
    mappingBytes_ = bytes;
    totalBytes_ = bytes;
    try {
        uint64_t hlen = 0;
        std::memcpy(&hlen, base_, 8);  // little endian on every supported host
        OPURE_CHECK(hlen > 0 && hlen <= bytes - 8, "safetensors header length is out of range");
        payloadBegin_ = 8 + hlen;
        payloadBytes_ = bytes - payloadBegin_;
        ParseHeader(base_ + 8, hlen);
    } catch (...) {
        Close();
        throw;
    }
}

void WeightStreamer::Close() {
    if (base_) ::munmap(base_, mappingBytes_);
    base_ = nullptr;
    mappingBytes_ = 0;
    payloadBegin_ = payloadBytes_ = totalBytes_ = 0;
    tensors_.clear();
}

void WeightStreamer::ParseHeader(const uint8_t *header, uint64_t len) {
    const json::Value root = json::ParseObject(
        std::string_view(reinterpret_cast<const char *>(header), len), "safetensors header");
    for (const auto &[name, v] : root.obj) {
        if (name == "__metadata__") continue;
        Tensor t;
        t.name = name;
        t.dtype = ParseDtype(v.At("dtype", name).str);
        if (const json::Value *s = v.Find("scale"); s && s->IsNumber()) t.scale = float(s->num);
        const json::Value &shape = v.At("shape", name);
        OPURE_CHECK(shape.IsArray(), "tensor '" + name + "' has a non-array shape");
        for (const json::Value &d : shape.arr) {
            OPURE_CHECK(d.IsNumber() && d.integral, "tensor '" + name + "' has a non-integer dim");
            t.shape.push_back(d.inum);
        }
        const json::Value &off = v.At("data_offsets", name);
        OPURE_CHECK(off.IsArray() && off.arr.size() == 2,
                    "data_offsets of '" + name + "' is not a [begin, end] pair");
        const uint64_t b = uint64_t(off.arr[0].inum), e = uint64_t(off.arr[1].inum);
        OPURE_CHECK(b <= e, "data_offsets of '" + name + "' end before they begin");
        OPURE_CHECK(e <= payloadBytes_, "bytes of '" + name + "' extend beyond the file's data section");
        const uint64_t expect = StorageBytes(t.dtype, t.ElementCount());
        OPURE_CHECK(e - b == expect, "'" + name + "' spans " + std::to_string(e - b) + " bytes, but " +
                                         std::to_string(t.ElementCount()) + " elements of " + DtypeName(t.dtype) +
                                         " take " + std::to_string(expect));
        t.byteBegin = payloadBegin_ + b;
        t.byteEnd = payloadBegin_ + e;
        tensors_.push_back(std::move(t));
    }
    OPURE_CHECK(!tensors_.empty(), "the safetensors header lists no tensor");
}

const Tensor *WeightStreamer::TryFind(std::string_view name) const {
    for (const Tensor &t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

const Tensor &WeightStreamer::Find(std::string_view name) const {
    const Tensor *t = TryFind(name);
    if (!t) ThrowError("tensor '" + std::string(name) + "' not found in the model");
    return *t;
}

const void *WeightStreamer::Data(const Tensor &t) const {
    OPURE_CHECK(base_ != nullptr, "WeightStreamer::Data on a closed streamer");
    OPURE_CHECK(t.byteEnd <= totalBytes_, "tensor '" + t.name + "' is out of range");
    return base_ + t.byteBegin;
}

float Bf16ToF32(uint16_t v) {
    const uint32_t bits = uint32_t(v) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float F16ToF32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            // Subnormal: value man * 2^-24. Normalise; e shifts make the exponent 1-e.
            uint32_t e = 0;
            while ((man & 0x400u) == 0) { man <<= 1; ++e; }
            bits = sign | ((127u - 15u + 1u - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t F32ToF16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    const uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return uint16_t(sign | (man ? 0x7E00u : 0x7C00u));
    const int e = int(exp) - 112;
    if (e >= 31) return uint16_t(sign | 0x7C00u);
    if (e <= 0) {
        const int s = 14 - e;
        if (s > 24) return uint16_t(sign);
        const uint32_t M = man | 0x800000u;
        uint32_t q = M >> s;
        const uint32_t rem = M & ((1u << s) - 1u), half = 1u << (s - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return uint16_t(sign | q);
    }
    uint32_t q = (uint32_t(e) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return uint16_t(sign | q);
}

uint64_t WidenToF32(Dtype dt, const void *src, uint64_t n, float *out) {
    const auto *s = static_cast<const uint8_t *>(src);
    switch (dt) {
        case Dtype::F32:
            std::memcpy(out, s, n * 4);
            return n * 4;
        case Dtype::BF16:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, s + i * 2, 2);
                out[i] = Bf16ToF32(h);
            }
            return n * 4;
        case Dtype::F16:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, s + i * 2, 2);
                out[i] = F16ToF32(h);
            }
            return n * 4;
        case Dtype::U8:
        case Dtype::I8:
            std::memcpy(out, s, n);
            return n;
        case Dtype::U4:
        case Dtype::I4: {
            // Two elements per byte, high nibble first (Opure_Streamer.cpp:404-424).
            const bool sgn = dt == Dtype::I4;
            for (uint64_t i = 0; i < n; ++i) {
                const uint8_t byte = s[i >> 1];
                const int nib = (i & 1) ? (byte & 0x0F) : (byte >> 4);
                out[i] = float(sgn && (nib & 8) ? nib - 16 : nib);
            }
            return n * 4;
        }
        default: ThrowError("WidenToF32 cannot widen this dtype");
    }
}

void NarrowToF16(Dtype dt, const void *src, uint64_t n, uint16_t *out) {
    const auto *s = static_cast<const uint8_t *>(src);
    switch (dt) {
        case Dtype::F16:
            std::memcpy(out, s, n * 2);
            return;
        case Dtype::BF16:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, s + i * 2, 2);
                out[i] = F32ToF16(Bf16ToF32(h));
            }
            return;
        case Dtype::F32:
            for (uint64_t i = 0; i < n; ++i) {
                float f;
                std::memcpy(&f, s + i * 4, 4);
                out[i] = F32ToF16(f);
            }
            return;
        default: ThrowError(std::string("cannot convert ") + DtypeName(dt) + " to fp16");
    }
}

}  // namespace opure::safetensors
