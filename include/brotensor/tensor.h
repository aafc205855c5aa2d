// brotensor/tensor.h — the tensor type of the reference's C++ entry points, as
// this build provides it. The reference composes the ops of its sibling library
// brotensor (absent here), whose `brotensor::Tensor` is a row-major fp32 matrix
// (rows, cols) tagged with a device (call sites throughout
// src/kokoro_decoder_backward.cpp and src/decoder_lora.cpp). This is a
// self-owned stand-in with the members and constructors those call sites and the
// reference's tests use, so code written against the reference compiles
// unchanged.
//
// Storage: CUDA managed memory, whatever the device tag. Every computation of
// this build runs on the GPU (there is no CPU path); managed memory keeps each
// element host-addressable as well, which the reference's callers rely on
// (element access through operator[], e.g. in finite-difference tests). The entry
// points synchronise before returning, so results may be read on the host at
// once. Value semantics: a copy owns a copy of the data.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace brotensor {

enum class Device { CPU, CUDA };
enum class Dtype { FP32 };

struct Tensor {
    int rows = 0;
    int cols = 0;
    Device device = Device::CPU;
    Dtype dtype = Dtype::FP32;
    void* data = nullptr;    // rows * cols floats (nullptr when empty)

    Tensor() = default;
    Tensor(const Tensor& o);
    Tensor(Tensor&& o) noexcept;
    Tensor& operator=(const Tensor& o);
    Tensor& operator=(Tensor&& o) noexcept;
    ~Tensor();

    // (r, c) zero-filled on `dev`
    static Tensor zeros_on(Device dev, int r, int c, Dtype dt = Dtype::FP32);
    // (r, c) on `dev`; this build zero-fills it too
    static Tensor empty_on(Device dev, int r, int c, Dtype dt = Dtype::FP32);
    // (r, c) copied from `src` (r * c host floats)
    static Tensor from_host_on(Device dev, const float* src, int r, int c);
    // (r, c) zero-filled, device tag CPU
    static Tensor mat(int r, int c);

    std::int64_t size() const { return (std::int64_t)rows * cols; }
    bool empty() const { return size() == 0; }
    float* f32() { return static_cast<float*>(data); }
    const float* f32() const { return static_cast<const float*>(data); }
    float& operator[](std::int64_t i) { return f32()[i]; }
    float operator[](std::int64_t i) const { return f32()[i]; }
    std::vector<float> to_host_vector() const;
    Tensor clone() const { return *this; }
    // a copy tagged with another device (the storage is reachable from both)
    Tensor to(Device dev) const;
    // reshape in place to (r, c), reallocating only when the element count changes;
    // the contents are zero after a reallocation and kept otherwise
    void resize(int r, int c);

   private:
    std::size_t cap_ = 0;    // allocated floats
    void alloc(std::int64_t n);
    void release();
};

}  // namespace brotensor
