// backend.cpp — tensor::backend::{Device, Tensor, ops} implemented over the
// libti_b200 C ABI (include/ti_b200.h).  This is the reference-side binding:
// built together with the reference's unchanged src/models, src/adapter and
// src/inference, it replaces src/backend/cuda/{device,tensor,ops}.cu.
#include <tensor/backend/ops.hpp>

#include <cstring>
#include <stdexcept>
#include <string>

#include "ti_b200.h"

namespace tensor::backend {

namespace {

[[noreturn]] void raise(ti_status st, const std::string& what) {
    const std::string msg = what + ": " + ti_last_error();
    if (st == TI_ERR_INVALID || st == TI_ERR_UNSUPPORTED) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}
void check(ti_status st, const char* what) {
    if (st != TI_OK) raise(st, what);
}

std::shared_ptr<void> device_alloc(const Device& d, std::size_t bytes) {
    void* p = nullptr;
    check(ti_malloc(d.index(), bytes, &p), "Tensor: device allocation");
    const int dev = d.index();
    return std::shared_ptr<void>(p, [dev](void* q) { ti_free(dev, q); });
}

std::shared_ptr<void> host_alloc(std::size_t bytes) {
    void* p = std::malloc(bytes ? bytes : 1);
    if (!p) throw std::bad_alloc();
    return std::shared_ptr<void>(p, [](void* q) { std::free(q); });
}

}  // namespace

// ------------------------------------------------------------------ Device
Device Device::cpu() { return Device(DeviceType::CPU, 0, "CPU", 0); }

Device Device::cuda(int index) {
    int count = 0;
    ti_device_count(&count);
    if (count == 0) throw std::runtime_error("Device::cuda: no CUDA devices available");
    if (index < 0 || index >= count)
        throw std::runtime_error("Device::cuda: index " + std::to_string(index) + " out of range (found " +
                                 std::to_string(count) + " devices)");
    char name[256] = {0};
    std::size_t mem = 0;
    check(ti_device_info(index, name, sizeof name, &mem), "Device::cuda");
    return Device(DeviceType::CUDA, index, name, mem);
}

void Device::make_current() const {
    if (type_ == DeviceType::CUDA) ti_set_device(index_);
}

// ------------------------------------------------------------------ Tensor
Tensor::Tensor(Tensor&& o) noexcept
    : storage_(std::move(o.storage_)), ptr_(o.ptr_), dtype_(o.dtype_), shape_(std::move(o.shape_)),
      device_(o.device_) {
    o.ptr_ = nullptr;
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this != &o) {
        storage_ = std::move(o.storage_);
        ptr_ = o.ptr_;
        dtype_ = o.dtype_;
        shape_ = std::move(o.shape_);
        device_ = o.device_;
        o.ptr_ = nullptr;
    }
    return *this;
}

std::size_t Tensor::nbytes() const noexcept { return numel() * core::dtype_size(dtype_); }

Tensor Tensor::empty(const Shape& shape, DType dtype, const Device& device) {
    Tensor t;
    const std::size_t bytes = shape.numel() * core::dtype_size(dtype);
    t.storage_ = device.is_cuda() ? device_alloc(device, bytes) : host_alloc(bytes);
    t.ptr_ = t.storage_.get();
    t.dtype_ = dtype;
    t.shape_ = shape;
    t.device_ = device;
    return t;
}

Tensor Tensor::zeros(const Shape& shape, DType dtype, const Device& device) {
    Tensor t = empty(shape, dtype, device);
    if (device.is_cuda()) {
        check(ti_memset(t.ptr_, 0, t.nbytes(), nullptr), "Tensor::zeros");
        check(ti_stream_sync(nullptr), "Tensor::zeros");
    } else {
        std::memset(t.ptr_, 0, t.nbytes());
    }
    return t;
}

Tensor Tensor::from_view(const TensorView& view, const Device& device) {
    Tensor t = empty(view.shape, view.dtype, device);
    if (device.is_cuda()) check(ti_memcpy_h2d(t.ptr_, view.data, view.nbytes(), nullptr), "Tensor::from_view");
    else std::memcpy(t.ptr_, view.data, view.nbytes());
    return t;
}

Tensor Tensor::alias(const Tensor& base, std::size_t byte_offset, Shape shape, DType dtype) {
    Tensor t;
    t.storage_ = base.storage_;
    t.ptr_ = static_cast<uint8_t*>(base.ptr_) + byte_offset;
    t.dtype_ = dtype;
    t.shape_ = std::move(shape);
    t.device_ = base.device_;
    return t;
}

std::vector<float> Tensor::to_host_f32() const {
    if (dtype_ != DType::F32) throw std::invalid_argument("Tensor::to_host_f32: dtype is not F32");
    std::vector<float> out(numel());
    if (device_.is_cuda()) check(ti_memcpy_d2h(out.data(), ptr_, nbytes(), nullptr), "Tensor::to_host_f32");
    else std::memcpy(out.data(), ptr_, nbytes());
    return out;
}

std::vector<int32_t> Tensor::to_host_i32() const {
    if (dtype_ != DType::I32) throw std::invalid_argument("Tensor::to_host_i32: dtype is not I32");
    std::vector<int32_t> out(numel());
    if (device_.is_cuda()) check(ti_memcpy_d2h(out.data(), ptr_, nbytes(), nullptr), "Tensor::to_host_i32");
    else std::memcpy(out.data(), ptr_, nbytes());
    return out;
}

// ------------------------------------------------------------------ ops
namespace ops {

namespace {
int dt(DType d) {
    switch (d) {
        case DType::F32: return TI_DTYPE_F32;
        case DType::BF16: return TI_DTYPE_BF16;
        default: throw std::invalid_argument("unsupported dtype " + core::to_string(d));
    }
}
void need_bf16(const Tensor& t, const char* op) {
    if (t.dtype() != DType::BF16) throw std::invalid_argument(std::string(op) + ": BF16 expected");
}
void need_cuda(const Tensor& t, const char* op) {
    if (!t.device().is_cuda()) throw std::invalid_argument(std::string(op) + ": CUDA tensor expected");
}
int as_int(std::size_t v) { return static_cast<int>(v); }
}  // namespace

Tensor embedding(const Tensor& w, const std::vector<int32_t>& ids) {
    need_cuda(w, "embedding");
    const int n = as_int(ids.size()), hidden = as_int(w.shape()[1]);
    w.device().make_current();
    Tensor out = Tensor::empty({ids.size(), w.shape()[1]}, w.dtype(), w.device());
    check(ti_op_embedding(w.data_ptr(), as_int(w.shape()[0]), hidden, ids.data(), n, out.data_ptr(), nullptr),
          "embedding");
    return out;
}

Tensor matmul_t(const Tensor& a, const Tensor& b) {
    need_cuda(a, "matmul_t");
    if (a.rank() != 2 || b.rank() != 2 || a.shape()[1] != b.shape()[1] || a.dtype() != b.dtype())
        throw std::invalid_argument("matmul_t: shapes [M,K] x [N,K] of one dtype expected");
    a.device().make_current();
    Tensor c = Tensor::empty({a.shape()[0], b.shape()[0]}, a.dtype(), a.device());
    check(ti_op_matmul_t(dt(a.dtype()), a.data_ptr(), b.data_ptr(), c.data_ptr(), as_int(a.shape()[0]),
                         as_int(b.shape()[0]), as_int(a.shape()[1]), nullptr),
          "matmul_t");
    return c;
}

static Tensor norm(const Tensor& x, const Tensor& w, float eps, int offset, const char* op) {
    need_bf16(x, op);
    x.device().make_current();
    Tensor out = Tensor::empty(x.shape(), x.dtype(), x.device());
    const int hidden = as_int(x.shape().back());
    check(ti_op_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), as_int(x.numel()) / hidden, hidden, eps, offset,
                         nullptr),
          op);
    return out;
}
Tensor rms_norm(const Tensor& x, const Tensor& w, float eps) { return norm(x, w, eps, 0, "rms_norm"); }
Tensor rms_norm_offset(const Tensor& x, const Tensor& w, float eps) { return norm(x, w, eps, 1, "rms_norm_offset"); }

Tensor rope(const Tensor& x, int seq_offset, float theta, const RopeScaling& sc) {
    need_bf16(x, "rope");
    if (x.rank() != 3) throw std::invalid_argument("rope: [seq, heads, head_dim] expected");
    x.device().make_current();
    Tensor out = Tensor::empty(x.shape(), x.dtype(), x.device());
    ti_rope_scaling s = {sc.apply_scaling ? 1 : 0, sc.factor, sc.low_freq_factor, sc.high_freq_factor,
                         sc.original_max_pos};
    check(ti_op_rope(x.data_ptr(), out.data_ptr(), as_int(x.shape()[0]), as_int(x.shape()[1]), as_int(x.shape()[2]),
                     seq_offset, theta, &s, nullptr),
          "rope");
    return out;
}
Tensor rope(const Tensor& x, int seq_offset, float theta) { return rope(x, seq_offset, theta, RopeScaling{}); }

static Tensor ew(int kind, const Tensor& a, const Tensor* b, float scalar, const char* op) {
    need_bf16(a, op);
    if (b && b->numel() != a.numel()) throw std::invalid_argument(std::string(op) + ": size mismatch");
    a.device().make_current();
    Tensor out = Tensor::empty(a.shape(), a.dtype(), a.device());
    check(ti_op_elementwise(kind, a.data_ptr(), b ? b->data_ptr() : nullptr, scalar, out.data_ptr(), a.numel(),
                            nullptr),
          op);
    return out;
}
Tensor silu(const Tensor& x) { return ew(TI_EW_SILU, x, nullptr, 0.f, "silu"); }
Tensor gelu(const Tensor& x) { return ew(TI_EW_GELU, x, nullptr, 0.f, "gelu"); }
Tensor mul(const Tensor& a, const Tensor& b) { return ew(TI_EW_MUL, a, &b, 0.f, "mul"); }
Tensor add(const Tensor& a, const Tensor& b) { return ew(TI_EW_ADD, a, &b, 0.f, "add"); }
Tensor mul(const Tensor& x, float s) { return ew(TI_EW_MUL_SCALAR, x, nullptr, s, "mul"); }

Tensor add_bias(const Tensor& x, const Tensor& bias) {
    need_bf16(x, "add_bias");
    x.device().make_current();
    Tensor out = Tensor::empty(x.shape(), x.dtype(), x.device());
    const int hidden = as_int(x.shape().back());
    check(ti_op_add_bias(x.data_ptr(), bias.data_ptr(), out.data_ptr(), as_int(x.numel()) / hidden, hidden, nullptr),
          "add_bias");
    return out;
}

Tensor softmax(const Tensor& x) {
    x.device().make_current();
    Tensor out = Tensor::empty(x.shape(), DType::F32, x.device());
    const int cols = as_int(x.shape().back());
    check(ti_op_softmax(dt(x.dtype()), x.data_ptr(), out.data_as<float>(), as_int(x.numel()) / cols, cols, nullptr),
          "softmax");
    return out;
}

Tensor attention(const Tensor& q, const Tensor& k, const Tensor& v, bool causal, int sliding_window) {
    need_bf16(q, "attention");
    if (q.rank() != 3 || k.rank() != 3 || v.rank() != 3) throw std::invalid_argument("attention: rank-3 q/k/v");
    q.device().make_current();
    Tensor out = Tensor::empty(q.shape(), q.dtype(), q.device());
    check(ti_op_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), as_int(q.shape()[0]),
                          as_int(q.shape()[1]), as_int(k.shape()[0]), as_int(k.shape()[1]), as_int(q.shape()[2]),
                          causal ? 1 : 0, sliding_window, nullptr),
          "attention");
    return out;
}

Tensor reshape(const Tensor& x, const Shape& shape) {
    if (shape.numel() != x.numel()) throw std::invalid_argument("reshape: numel mismatch");  // ops.cu:551
    return Tensor::alias(x, 0, shape, x.dtype());
}

Tensor transpose(const Tensor& x, std::size_t, std::size_t) {
    if (x.rank() != 2) throw std::invalid_argument("transpose: only 2D supported currently");  // ops.cu:561
    x.device().make_current();
    Tensor out = Tensor::empty({x.shape()[1], x.shape()[0]}, x.dtype(), x.device());
    check(ti_op_transpose2d(dt(x.dtype()), x.data_ptr(), out.data_ptr(), as_int(x.shape()[0]), as_int(x.shape()[1]),
                            nullptr),
          "transpose");
    return out;
}

Tensor cast(const Tensor& x, DType target) {
    x.device().make_current();
    Tensor out = Tensor::empty(x.shape(), target, x.device());
    check(ti_op_cast(dt(x.dtype()), dt(target), x.data_ptr(), out.data_ptr(), x.numel(), nullptr), "cast");
    return out;
}

Tensor cat(const std::vector<const Tensor*>& ts, std::size_t dim) {
    if (ts.empty()) throw std::invalid_argument("cat: empty tensor list");
    if (dim != 0) throw std::invalid_argument("cat: only dim=0 supported currently");  // ops.cu:642
    Shape s = ts[0]->shape();
    for (std::size_t i = 1; i < ts.size(); ++i) s[0] += ts[i]->shape()[0];
    ts[0]->device().make_current();
    Tensor out = Tensor::empty(s, ts[0]->dtype(), ts[0]->device());
    std::size_t off = 0;
    for (const Tensor* t : ts) {
        check(ti_memcpy_d2d(static_cast<uint8_t*>(out.data_ptr()) + off, t->data_ptr(), t->nbytes(), nullptr), "cat");
        off += t->nbytes();
    }
    return out;
}

Tensor slice(const Tensor& x, std::size_t dim, std::size_t begin, std::size_t end) {
    if (dim != 0) throw std::invalid_argument("slice: only dim=0 supported currently");  // ops.cu:649
    if (begin > end || end > x.shape()[0]) throw std::invalid_argument("slice: range out of bounds");
    Shape s = x.shape();
    s[0] = end - begin;
    const std::size_t row = x.shape()[0] ? x.nbytes() / x.shape()[0] : 0;
    return Tensor::alias(x, begin * row, s, x.dtype());
}

}  // namespace ops
}  // namespace tensor::backend
