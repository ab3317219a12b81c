// Stable-LibTorch-ABI registration of the ops, a thin shim over the C ABI in ipl_b200.h.
//
// Namespace, schemas and in-place signatures are those of the reference
// (csrc/torch_ops.cpp:12-22): fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual,
// Tensor weight, float epsilon) -> (), silu_and_mul(Tensor(a!) output, Tensor input) -> (),
// silu_and_mul_packed(Tensor(a!) output, Tensor input) -> (). The tensor checks repeat the
// reference's (csrc/fused_add_rms_norm_kernel.cu:277-301, csrc/silu_and_mul_kernel.cu:86-106,
// :130-158) with the same messages, so callers see the same RuntimeError texts. The kernel runs
// on the current stream of the tensors' device, under a device guard; nothing synchronises.
#include <torch/csrc/stable/accelerator.h>
#include <torch/csrc/stable/library.h>
#include <torch/csrc/stable/tensor.h>
#include <torch/headeronly/core/ScalarType.h>
#include <torch/headeronly/util/Exception.h>

#include <cstdint>
#include <limits>

#include "ipl_b200.h"

// Declared by torch's C shim under USE_CUDA; the symbol lives in libtorch_cuda.
extern "C" AOTITorchError aoti_torch_get_current_cuda_stream(int32_t device_index, void** ret_stream);

namespace ts = torch::stable;

namespace {

void* current_stream(int32_t device_index) {
    void* stream = nullptr;
    const AOTITorchError err = aoti_torch_get_current_cuda_stream(device_index, &stream);
    STD_TORCH_CHECK(err == AOTI_TORCH_SUCCESS, "failed to query the current CUDA stream");
    return stream;
}

void raise_on_error(ipl_status status) {
    STD_TORCH_CHECK(status == IPL_SUCCESS, ipl_last_error());
}

void check_silu_tensors(const ts::Tensor& output, const ts::Tensor& input) {
    STD_TORCH_CHECK(input.is_cuda() && output.is_cuda(), "input and output must be CUDA tensors");
    STD_TORCH_CHECK(input.scalar_type() == torch::headeronly::ScalarType::BFloat16 &&
                        output.scalar_type() == torch::headeronly::ScalarType::BFloat16,
                    "input and output must use bfloat16");
    STD_TORCH_CHECK(input.is_contiguous() && output.is_contiguous(), "input and output must be contiguous");
    STD_TORCH_CHECK(input.device() == output.device(), "input and output must be on the same device");
    STD_TORCH_CHECK(input.dim() >= 1 && input.size(-1) % 2 == 0, "the final input dimension must be even");
    STD_TORCH_CHECK(output.dim() == input.dim(), "input and output must have the same rank");
    const int64_t intermediate_size = input.size(-1) / 2;
    STD_TORCH_CHECK(output.size(-1) == intermediate_size, "the output width must be half the input width");
    for (int64_t dimension = 0; dimension < input.dim() - 1; ++dimension) {
        STD_TORCH_CHECK(output.size(dimension) == input.size(dimension),
                        "input and output leading dimensions must match");
    }
}

void run_silu(ts::Tensor& output, const ts::Tensor& input, bool packed) {
    check_silu_tensors(output, input);
    if (output.numel() == 0) {
        return;
    }
    const int64_t intermediate_size = input.size(-1) / 2;
    const int64_t rows = output.numel() / intermediate_size;
    const int32_t device = input.get_device_index();
    const ts::accelerator::DeviceGuard device_guard(device);
    void* stream = current_stream(device);
    void* out = output.mutable_data_ptr();
    const void* in = input.const_data_ptr();
    raise_on_error(packed ? ipl_silu_and_mul_packed_bf16(out, in, rows, intermediate_size, stream)
                          : ipl_silu_and_mul_bf16(out, in, rows, intermediate_size, stream));
}

}  // namespace

void fused_add_rms_norm_cuda(ts::Tensor& x, ts::Tensor& residual, const ts::Tensor& weight, double epsilon) {
    STD_TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor");
    STD_TORCH_CHECK(residual.is_cuda(), "residual must be a CUDA tensor");
    STD_TORCH_CHECK(weight.is_cuda(), "weight must be a CUDA tensor");

    STD_TORCH_CHECK(x.scalar_type() == torch::headeronly::ScalarType::BFloat16, "x must use bfloat16");
    STD_TORCH_CHECK(residual.scalar_type() == torch::headeronly::ScalarType::BFloat16, "residual must use bfloat16");
    STD_TORCH_CHECK(weight.scalar_type() == torch::headeronly::ScalarType::BFloat16, "weight must use bfloat16");

    STD_TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
    STD_TORCH_CHECK(residual.is_contiguous(), "residual must be contiguous");
    STD_TORCH_CHECK(weight.is_contiguous(), "weight must be contiguous");

    STD_TORCH_CHECK(x.sizes().equals(residual.sizes()), "x and residual must have identical shapes");
    STD_TORCH_CHECK(x.device() == residual.device() && x.device() == weight.device(),
                    "x, residual, and weight must be on the same device");
    STD_TORCH_CHECK(x.dim() >= 1, "x must have at least one dimension");
    STD_TORCH_CHECK(weight.dim() == 1, "weight must be one-dimensional");
    STD_TORCH_CHECK(weight.size(0) == x.size(-1), "weight must match the final tensor dimension");
    STD_TORCH_CHECK(epsilon > 0.0, "epsilon must be positive");

    const int64_t hidden_size = x.size(-1);
    if (x.numel() == 0) {
        // Nothing to normalise (the reference launches an empty grid here and fails).
        return;
    }
    const int64_t rows = x.numel() / hidden_size;

    STD_TORCH_CHECK(hidden_size <= std::numeric_limits<int>::max(), "hidden dimension is too large");
    STD_TORCH_CHECK(rows <= std::numeric_limits<int>::max(), "number of rows is too large");

    const int32_t device = x.get_device_index();
    const ts::accelerator::DeviceGuard device_guard(device);
    void* stream = current_stream(device);
    raise_on_error(ipl_fused_add_rms_norm_bf16(x.mutable_data_ptr(), residual.mutable_data_ptr(),
                                               weight.const_data_ptr(), rows, hidden_size, epsilon, stream));
}

void rms_norm_cuda(ts::Tensor& output, const ts::Tensor& input, const ts::Tensor& weight, double epsilon) {
    STD_TORCH_CHECK(output.is_cuda() && input.is_cuda() && weight.is_cuda(),
                    "output, input, and weight must be CUDA tensors");
    STD_TORCH_CHECK(output.scalar_type() == torch::headeronly::ScalarType::BFloat16 &&
                        input.scalar_type() == torch::headeronly::ScalarType::BFloat16 &&
                        weight.scalar_type() == torch::headeronly::ScalarType::BFloat16,
                    "output, input, and weight must use bfloat16");
    STD_TORCH_CHECK(output.is_contiguous() && input.is_contiguous() && weight.is_contiguous(),
                    "output, input, and weight must be contiguous");
    STD_TORCH_CHECK(output.sizes().equals(input.sizes()), "output and input must have identical shapes");
    STD_TORCH_CHECK(output.device() == input.device() && input.device() == weight.device(),
                    "output, input, and weight must be on the same device");
    STD_TORCH_CHECK(input.dim() >= 1, "input must have at least one dimension");
    STD_TORCH_CHECK(weight.dim() == 1, "weight must be one-dimensional");
    STD_TORCH_CHECK(weight.size(0) == input.size(-1), "weight must match the final tensor dimension");
    STD_TORCH_CHECK(epsilon > 0.0, "epsilon must be positive");
    if (input.numel() == 0) {
        return;
    }
    const int64_t hidden_size = input.size(-1);
    const int64_t rows = input.numel() / hidden_size;
    const int32_t device = input.get_device_index();
    const ts::accelerator::DeviceGuard device_guard(device);
    void* stream = current_stream(device);
    raise_on_error(ipl_rms_norm_bf16(output.mutable_data_ptr(), input.const_data_ptr(), weight.const_data_ptr(),
                                     rows, hidden_size, epsilon, stream));
}

void fused_add_rms_norm_static_fp8_quant_cuda(ts::Tensor& result, const ts::Tensor& input, ts::Tensor& residual,
                                              const ts::Tensor& weight, const ts::Tensor& scale, double epsilon) {
    STD_TORCH_CHECK(result.is_cuda() && input.is_cuda() && residual.is_cuda() && weight.is_cuda() && scale.is_cuda(),
                    "result, input, residual, weight, and scale must be CUDA tensors");
    STD_TORCH_CHECK(result.scalar_type() == torch::headeronly::ScalarType::Float8_e4m3fn,
                    "result must use float8_e4m3fn");
    STD_TORCH_CHECK(input.scalar_type() == torch::headeronly::ScalarType::BFloat16 &&
                        residual.scalar_type() == torch::headeronly::ScalarType::BFloat16 &&
                        weight.scalar_type() == torch::headeronly::ScalarType::BFloat16,
                    "input, residual, and weight must use bfloat16");
    STD_TORCH_CHECK(scale.scalar_type() == torch::headeronly::ScalarType::Float && scale.numel() == 1,
                    "scale must be a single float32");
    STD_TORCH_CHECK(result.is_contiguous() && input.is_contiguous() && residual.is_contiguous() &&
                        weight.is_contiguous(),
                    "result, input, residual, and weight must be contiguous");
    STD_TORCH_CHECK(input.sizes().equals(residual.sizes()) && input.sizes().equals(result.sizes()),
                    "result, input, and residual must have identical shapes");
    STD_TORCH_CHECK(input.device() == residual.device() && input.device() == weight.device() &&
                        input.device() == result.device() && input.device() == scale.device(),
                    "all tensors must be on the same device");
    STD_TORCH_CHECK(input.dim() >= 1, "input must have at least one dimension");
    STD_TORCH_CHECK(weight.dim() == 1, "weight must be one-dimensional");
    STD_TORCH_CHECK(weight.size(0) == input.size(-1), "weight must match the final tensor dimension");
    STD_TORCH_CHECK(epsilon > 0.0, "epsilon must be positive");
    if (input.numel() == 0) {
        return;
    }
    const int64_t hidden_size = input.size(-1);
    const int64_t rows = input.numel() / hidden_size;
    const int32_t device = input.get_device_index();
    const ts::accelerator::DeviceGuard device_guard(device);
    void* stream = current_stream(device);
    raise_on_error(ipl_fused_add_rms_norm_static_fp8_quant(
        result.mutable_data_ptr(), input.const_data_ptr(), residual.mutable_data_ptr(), weight.const_data_ptr(),
        static_cast<const float*>(scale.const_data_ptr()), rows, hidden_size, epsilon, stream));
}

void silu_and_mul_cuda(ts::Tensor& output, const ts::Tensor& input) { run_silu(output, input, false); }

void silu_and_mul_packed_cuda(ts::Tensor& output, const ts::Tensor& input) { run_silu(output, input, true); }

STABLE_TORCH_LIBRARY(inference_performance_lab, library) {
    library.def("fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual, Tensor weight, float epsilon) -> ()");
    library.def("silu_and_mul(Tensor(a!) output, Tensor input) -> ()");
    library.def("silu_and_mul_packed(Tensor(a!) output, Tensor input) -> ()");
    // Not in the reference library: plain RMSNorm (vLLM's _C.rms_norm argument order).
    library.def("rms_norm(Tensor(a!) output, Tensor input, Tensor weight, float epsilon) -> ()");
    // Not in the reference library: add+RMSNorm with a static fp8 output (vLLM's argument order).
    library.def(
        "fused_add_rms_norm_static_fp8_quant(Tensor(a!) result, Tensor input, Tensor(b!) residual, "
        "Tensor weight, Tensor scale, float epsilon) -> ()");
}

STABLE_TORCH_LIBRARY_IMPL(inference_performance_lab, CUDA, library) {
    library.impl("fused_add_rms_norm", TORCH_BOX(&fused_add_rms_norm_cuda));
    library.impl("silu_and_mul", TORCH_BOX(&silu_and_mul_cuda));
    library.impl("silu_and_mul_packed", TORCH_BOX(&silu_and_mul_packed_cuda));
    library.impl("rms_norm", TORCH_BOX(&rms_norm_cuda));
    library.impl("fused_add_rms_norm_static_fp8_quant", TORCH_BOX(&fused_add_rms_norm_static_fp8_quant_cuda));
}
