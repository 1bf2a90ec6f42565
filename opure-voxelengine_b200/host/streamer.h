// streamer.h -- zero-copy .safetensors reader (POSIX mmap).
// Keeps the API of the reference's safetensors::WeightStreamer
// (src/core/Opure_Streamer.h:47-153): Dtype, Tensor, WeightStreamer::{Open, Close, Find,
// TryFind, Data, ...}, Bf16ToF32, WidenToF32. Two reference bugs are not carried over:
// ElementBytes(F16/BF16) = 4 made the header cross-check reject every real F16/BF16 file
// (Opure_Streamer.cpp:110,318-322), and F16ToF32 halved fp16 subnormals (:66).
#pragma once

#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

namespace opure::safetensors {

enum class Dtype : uint8_t { F32, F16, BF16, U8, I8, U4, I4, Count };

const char *DtypeName(Dtype d);
Dtype ParseDtype(std::string_view s);
// Bytes a tensor of `elements` occupies in the file (4-bit types pack two per byte).
uint64_t StorageBytes(Dtype d, uint64_t elements);

struct Tensor {
    std::string name;
    Dtype dtype = Dtype::F32;
    std::vector<int64_t> shape;
    uint64_t byteBegin = 0;  // absolute offset into the mapped file
    uint64_t byteEnd = 0;
    float scale = 1.0f;      // per-tensor scale of quantised tensors ("scale" header key)

    uint64_t ElementCount() const;
    uint64_t ByteCount() const { return byteEnd - byteBegin; }
    uint64_t Rows() const;   // product of all dims but the last
    uint64_t Cols() const;   // last dim
};

class WeightStreamer {
public:
    WeightStreamer() = default;
    ~WeightStreamer() { Close(); }
    WeightStreamer(const WeightStreamer &) = delete;
    WeightStreamer &operator=(const WeightStreamer &) = delete;

    void Open(const std::string &path);  // throws opure::Error
    void Close();

    bool IsOpen() const { return base_ != nullptr; }
    size_t TensorCount() const { return tensors_.size(); }
    const Tensor &TensorAt(size_t i) const { return tensors_[i]; }
    const std::vector<Tensor> &Tensors() const { return tensors_; }
    const Tensor &Find(std::string_view name) const;     // throws when absent
    const Tensor *TryFind(std::string_view name) const;
    const void *Data(const Tensor &t) const;
    uint64_t ByteOffset(const Tensor &t) const { return t.byteBegin; }
    uint64_t PayloadBegin() const { return payloadBegin_; }
    uint64_t PayloadBytes() const { return payloadBytes_; }
    uint64_t TotalBytes() const { return totalBytes_; }

private:
    void ParseHeader(const uint8_t *header, uint64_t len);

    uint8_t *base_ = nullptr;
    size_t mappingBytes_ = 0;
    uint64_t payloadBegin_ = 0, payloadBytes_ = 0, totalBytes_ = 0;
    std::vector<Tensor> tensors_;
};

float Bf16ToF32(uint16_t v);
float F16ToF32(uint16_t v);
uint16_t F32ToF16(float f);  // IEEE round to nearest even

// F32/F16/BF16 -> fp32 words; U8/I8 copied raw; U4/I4 widened. Returns bytes written.
uint64_t WidenToF32(Dtype dt, const void *src, uint64_t elements, float *out);
// F32/F16/BF16 -> fp16 (the engine's resident weight format).
void NarrowToF16(Dtype dt, const void *src, uint64_t elements, uint16_t *out);

}  // namespace opure::safetensors
