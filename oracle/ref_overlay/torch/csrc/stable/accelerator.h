// Include overlay used only to compile the reference's own CUDA sources for sm_100a against this
// image's torch (test infrastructure; see oracle/build_ref_kernels.py). It is found before torch's
// include directory, pulls in torch's real header with #include_next, and adds the one accessor the
// reference's wrappers call that torch 2.11's stable Stream lacks: nativeHandle(), the raw
// cudaStream_t of the device's current stream (reference csrc/fused_add_rms_norm_kernel.cu:305,
// csrc/silu_and_mul_kernel.cu:121,174). Nothing else of the reference's code path changes.
#pragma once

#include_next <torch/csrc/stable/accelerator.h>

#include <cstdint>

extern "C" AOTITorchError aoti_torch_get_current_cuda_stream(int32_t device_index, void** ret_stream);

namespace torch::stable::accelerator {

// The current CUDA stream of a device, as the reference's `getCurrentStream(i).nativeHandle()`.
struct RefCurrentStream {
    void* handle;
    void* nativeHandle() const { return handle; }
};

inline RefCurrentStream ref_current_stream(DeviceIndex device_index) {
    void* stream = nullptr;
    TORCH_ERROR_CODE_CHECK(aoti_torch_get_current_cuda_stream(device_index, &stream));
    return RefCurrentStream{stream};
}

}  // namespace torch::stable::accelerator

// From here on, the reference's `ts::accelerator::getCurrentStream(i)` names the accessor above.
#define getCurrentStream(device_index) ref_current_stream(device_index)
