// CPU stand-in for brotensor::Tensor, used only to compile the reference's own
// decoder sources (src/kokoro_decoder_backward.cpp, src/decoder_lora.cpp) as a
// checker of this repository's oracle. Test infrastructure: host memory, fp32,
// value semantics. The members are those the reference's call sites use.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace brotensor {

enum class Device { CPU, CUDA, METAL };
enum class Dtype { FP32 };

struct Tensor {
    int rows = 0;
    int cols = 0;
    Device device = Device::CPU;
    Dtype dtype = Dtype::FP32;
    void* data = nullptr;

    Tensor() = default;
    Tensor(const Tensor& o) : rows(o.rows), cols(o.cols), device(o.device), dtype(o.dtype), buf_(o.buf_) {
        data = buf_.empty() ? nullptr : buf_.data();
    }
    Tensor(Tensor&& o) noexcept
        : rows(o.rows), cols(o.cols), device(o.device), dtype(o.dtype), buf_(std::move(o.buf_)) {
        data = buf_.empty() ? nullptr : buf_.data();
        o.rows = o.cols = 0;
        o.data = nullptr;
    }
    Tensor& operator=(const Tensor& o) {
        if (this != &o) {
            rows = o.rows; cols = o.cols; device = o.device; dtype = o.dtype; buf_ = o.buf_;
            data = buf_.empty() ? nullptr : buf_.data();
        }
        return *this;
    }
    Tensor& operator=(Tensor&& o) noexcept {
        if (this != &o) {
            rows = o.rows; cols = o.cols; device = o.device; dtype = o.dtype; buf_ = std::move(o.buf_);
            data = buf_.empty() ? nullptr : buf_.data();
            o.rows = o.cols = 0;
            o.data = nullptr;
        }
        return *this;
    }

    static Tensor zeros_on(Device dev, int r, int c, Dtype dt = Dtype::FP32) {
        Tensor t;
        t.rows = r; t.cols = c; t.device = dev; t.dtype = dt;
        t.buf_.assign((size_t)r * c, 0.0f);
        t.data = t.buf_.empty() ? nullptr : t.buf_.data();
        return t;
    }
    static Tensor empty_on(Device dev, int r, int c, Dtype dt = Dtype::FP32) { return zeros_on(dev, r, c, dt); }
    static Tensor from_host_on(Device dev, const float* src, int r, int c) {
        Tensor t = zeros_on(dev, r, c);
        if (t.size()) std::memcpy(t.buf_.data(), src, sizeof(float) * (size_t)t.size());
        return t;
    }
    static Tensor mat(int r, int c) { return zeros_on(Device::CPU, r, c); }

    std::int64_t size() const { return (std::int64_t)rows * cols; }
    float* f() { return buf_.data(); }
    const float* f() const { return buf_.data(); }
    float& operator[](std::int64_t i) { return buf_[(size_t)i]; }
    float operator[](std::int64_t i) const { return buf_[(size_t)i]; }
    std::vector<float> to_host_vector() const { return buf_; }
    Tensor clone() const { return *this; }
    Tensor to(Device dev) const { Tensor t(*this); t.device = dev; return t; }
    // (r, c) zero-filled
    void reset(int r, int c) { *this = zeros_on(device, r, c); }

   private:
    std::vector<float> buf_;
};

}  // namespace brotensor
