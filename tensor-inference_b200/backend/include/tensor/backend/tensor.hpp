#pragma once
// tensor::backend::Tensor over libti_b200 — same public interface as the
// reference's include/tensor/backend/tensor.hpp:21-72 (move-only, factories,
// metadata, raw pointer, host read-back).  Storage is shared between a tensor
// and the zero-copy views ops::reshape / ops::slice return (the reference copies
// there, ops.cu:550-557,648-665), so `q = ops::reshape(q, ...)` keeps the bytes
// alive.  Device memory comes from libti_b200's stream-ordered pool
// (ti_malloc / ti_free), so per-op temporaries never hit cudaMalloc/cudaFree.
#include <tensor/backend/device.hpp>
#include <tensor/core/dtype.hpp>
#include <tensor/core/shape.hpp>
#include <tensor/core/tensor_view.hpp>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

namespace tensor::backend {

using core::DType;
using core::Shape;
using core::TensorView;

class Tensor {
public:
    Tensor() = default;
    ~Tensor() = default;

    Tensor(const Tensor&)            = delete;
    Tensor& operator=(const Tensor&) = delete;
    Tensor(Tensor&&) noexcept;
    Tensor& operator=(Tensor&&) noexcept;

    static Tensor empty(const Shape& shape, DType dtype, const Device& device);
    static Tensor zeros(const Shape& shape, DType dtype, const Device& device);
    static Tensor from_view(const TensorView& view, const Device& device);

    DType         dtype()  const noexcept { return dtype_; }
    const Shape&  shape()  const noexcept { return shape_; }
    std::size_t   rank()   const noexcept { return shape_.rank(); }
    std::size_t   numel()  const noexcept { return shape_.numel(); }
    std::size_t   nbytes() const noexcept;
    const Device& device() const noexcept { return device_; }
    bool          valid()  const noexcept { return ptr_ != nullptr; }

    void*       data_ptr()       noexcept { return ptr_; }
    const void* data_ptr() const noexcept { return ptr_; }

    template <typename T> T* data_as() noexcept { return static_cast<T*>(ptr_); }
    template <typename T> const T* data_as() const noexcept { return static_cast<const T*>(ptr_); }

    std::vector<float>   to_host_f32() const;
    std::vector<int32_t> to_host_i32() const;

    // zero-copy alias of `base` bytes [byte_offset, byte_offset + nbytes(shape, dtype))
    static Tensor alias(const Tensor& base, std::size_t byte_offset, Shape shape, DType dtype);

private:
    std::shared_ptr<void> storage_;
    void*   ptr_   = nullptr;
    DType   dtype_ = DType::F32;
    Shape   shape_ = {};
    Device  device_;
};

}  // namespace tensor::backend
