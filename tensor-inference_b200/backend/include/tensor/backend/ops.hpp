#pragma once
// tensor::backend::ops over libti_b200 — the same free functions and default
// arguments as the reference's include/tensor/backend/ops.hpp:19-117, so the
// reference's model code compiles against this header unchanged.  Each call
// validates shapes, allocates the result from libti_b200's pool and runs one
// sm_100a kernel (ti_op_*) on the legacy default stream, matching the
// reference's "synchronous with respect to the default stream" contract.
// Errors: std::invalid_argument for bad shapes/dtypes, std::runtime_error for
// device failures (as ops.cu:19-27 and :144,552,561,613,642,649).
#include <tensor/backend/tensor.hpp>

#include <cstdint>
#include <vector>

namespace tensor::backend::ops {

Tensor embedding(const Tensor& weight, const std::vector<int32_t>& indices);
Tensor matmul_t(const Tensor& a, const Tensor& b);
Tensor rms_norm(const Tensor& x, const Tensor& weight, float eps = 1e-5f);

struct RopeScaling {
    bool  apply_scaling    = false;
    float factor           = 1.0f;
    float low_freq_factor  = 1.0f;
    float high_freq_factor = 1.0f;
    int   original_max_pos = 8192;
};

Tensor rope(const Tensor& x, int seq_offset, float theta, const RopeScaling& scaling);
Tensor rope(const Tensor& x, int seq_offset, float theta = 500000.0f);
Tensor silu(const Tensor& x);
Tensor mul(const Tensor& a, const Tensor& b);
Tensor add(const Tensor& a, const Tensor& b);
Tensor softmax(const Tensor& x);
Tensor attention(const Tensor& q, const Tensor& k, const Tensor& v, bool causal = true, int sliding_window = -1);
Tensor reshape(const Tensor& x, const Shape& shape);
Tensor transpose(const Tensor& x, std::size_t dim_a, std::size_t dim_b);
Tensor cast(const Tensor& x, DType target);
Tensor cat(const std::vector<const Tensor*>& tensors, std::size_t dim);
Tensor slice(const Tensor& x, std::size_t dim, std::size_t begin, std::size_t end);
Tensor add_bias(const Tensor& x, const Tensor& bias);
Tensor gelu(const Tensor& x);
Tensor rms_norm_offset(const Tensor& x, const Tensor& weight, float eps = 1e-6f);
Tensor mul(const Tensor& x, float scalar);

}  // namespace tensor::backend::ops
