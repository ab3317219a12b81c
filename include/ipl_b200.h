/*
 * ipl_b200.h - C ABI of the B200 (sm_100a) fused add+RMSNorm and SiLU-and-mul library.
 *
 * Plain pointers and sizes only; no torch types cross this boundary. Every entry point is
 * stream-ordered: it validates its arguments on the host, enqueues at most one kernel on
 * `stream` (a cudaStream_t; NULL means the legacy default stream) of the CURRENT device and
 * returns without synchronising. Device pointers must be memory of the current device.
 * Nothing is allocated on the device.
 *
 * Element type is bfloat16 (passed as raw 16-bit words); arithmetic is fp32.
 *
 * Errors: every function returns IPL_SUCCESS (0) or a nonzero ipl_status. The message of the
 * last failure on the calling thread is available from ipl_last_error(); the messages repeat
 * the reference's STD_TORCH_CHECK texts where an equivalent check exists.
 *
 * Shared library: libipl_b200.so (link with -lipl_b200, or dlopen it).
 */
#ifndef IPL_B200_H_
#define IPL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IPL_ABI_VERSION 1

#if defined(__GNUC__)
#define IPL_API __attribute__((visibility("default")))
#else
#define IPL_API
#endif

typedef int ipl_status;

#define IPL_SUCCESS 0
#define IPL_ERROR_INVALID_VALUE 1 /* bad size, null pointer, non-positive epsilon */
#define IPL_ERROR_MISALIGNED 2    /* packed entry point given a pointer or width it cannot vectorise */
#define IPL_ERROR_TOO_LARGE 3     /* a dimension beyond what the kernels index */
#define IPL_ERROR_CUDA 4          /* a CUDA runtime call or kernel launch failed */

/*
 * Fused residual add + RMSNorm, in place, over `rows` rows of `hidden_size` bf16 elements:
 *
 *   v        = fp32(x) + fp32(residual)                (fp32, round to nearest)
 *   residual = bf16(v)                                 (bit-exact with the reference)
 *   x        = bf16(v * rsqrt(mean(v^2) + epsilon) * fp32(weight))
 *
 * x, residual: [rows, hidden_size] contiguous, distinct; weight: [hidden_size].
 * Any alignment of the three pointers is accepted. rows == 0 is a no-op.
 *
 * Replaces fused_add_rms_norm_cuda(Tensor& x, Tensor& residual, const Tensor& weight,
 * double epsilon) at csrc/fused_add_rms_norm_kernel.cu:276-329 of the reference, the body of
 * torch.ops.inference_performance_lab.fused_add_rms_norm (csrc/torch_ops.cpp:13,19).
 */
IPL_API ipl_status ipl_fused_add_rms_norm_bf16(void* x, void* residual, const void* weight, int64_t rows,
                                       int64_t hidden_size, double epsilon, void* stream);

/*
 * RMSNorm without a residual, out of place (output may equal input):
 *
 *   output = bf16((fp32(input) * rsqrt(mean(fp32(input)^2) + epsilon)) * fp32(weight))
 *
 * input, output: [rows, hidden_size] contiguous; weight: [hidden_size]. Any alignment is
 * accepted (output sharing input's offset modulo 16 bytes keeps the vectorised kernels).
 *
 * No counterpart in the reference's C++ sources: it is the plain rms_norm of the vLLM IR that
 * the reference's plugin targets (vllm/ir/ops/layernorm.py:9-21 of vLLM 0.22, the op before the
 * first and after the last decoder layer), with vLLM's torch.ops._C.rms_norm(out, input, weight,
 * epsilon) argument order and the reference oracle's fp32 arithmetic
 * (src/inference_performance_lab/kernels/reference.py:18-23 with a zero residual).
 */
IPL_API ipl_status ipl_rms_norm_bf16(void* output, const void* input, const void* weight, int64_t rows,
                                     int64_t hidden_size, double epsilon, void* stream);

/*
 * Fused residual add + RMSNorm with a statically scaled fp8 (e4m3) output:
 *
 *   v        = fp32(input) + fp32(residual)
 *   residual = bf16(v)                                            (bit-exact, in place)
 *   output   = e4m3(((v * rsqrt(mean(v^2) + epsilon)) * fp32(weight)) / *scale)
 *
 * e4m3 is OCP E4M3FN (bias 7, max 448, no infinities), round to nearest even, saturating to
 * +-448. input is read only. output: [rows, hidden_size] bytes; scale: one fp32 on the device.
 *
 * No counterpart in the reference's C++ sources: it is the fused variant the reference's scope
 * lists next (add+RMSNorm feeding an fp8 GEMM), with vLLM's
 * torch.ops._C.fused_add_rms_norm_static_fp8_quant(result, input, residual, weight, scale,
 * epsilon) argument order and the reference oracle's arithmetic up to the quantisation
 * (src/inference_performance_lab/kernels/reference.py:18-21).
 */
IPL_API ipl_status ipl_fused_add_rms_norm_static_fp8_quant(void* output, const void* input, void* residual,
                                                           const void* weight, const float* scale, int64_t rows,
                                                           int64_t hidden_size, double epsilon, void* stream);

/*
 * SiLU-and-multiply: output[r, c] = bf16(silu(fp32(input[r, c])) * fp32(input[r, I + c])),
 * I = intermediate_size, input [rows, 2*I] and output [rows, I], both contiguous. Any width and
 * alignment is accepted; aligned widths take the vector path. rows * I == 0 is a no-op.
 *
 * Replaces silu_and_mul_cuda(Tensor& output, const Tensor& input) at
 * csrc/silu_and_mul_kernel.cu:85-127 (torch.ops.inference_performance_lab.silu_and_mul,
 * csrc/torch_ops.cpp:14,20).
 */
IPL_API ipl_status ipl_silu_and_mul_bf16(void* output, const void* input, int64_t rows,
                                 int64_t intermediate_size, void* stream);

/*
 * Same computation with the reference's packed contract: intermediate_size must be a multiple
 * of 8 and both pointers 16-byte aligned, else IPL_ERROR_MISALIGNED with the reference's
 * message ("the output width must be divisible by 8", "input and output must be 16-byte
 * aligned"); no fallback path is taken.
 *
 * Replaces silu_and_mul_packed_cuda(Tensor& output, const Tensor& input) at
 * csrc/silu_and_mul_kernel.cu:129-180 (torch.ops.inference_performance_lab.silu_and_mul_packed,
 * csrc/torch_ops.cpp:15,21).
 */
IPL_API ipl_status ipl_silu_and_mul_packed_bf16(void* output, const void* input, int64_t rows,
                                        int64_t intermediate_size, void* stream);

/* Message of the last failing call on this thread ("" if none). Valid until the next call. */
IPL_API const char* ipl_last_error(void);

/* Static name of a status code. */
IPL_API const char* ipl_status_string(ipl_status status);

/* IPL_ABI_VERSION of the loaded library. */
IPL_API int ipl_abi_version(void);

/*
 * Device-side fault word of `device`: bit flags that a kernel sets when one of its bounded
 * waits on a shared-memory barrier runs out (the kernel then stops early and its outputs are
 * incomplete). 0 means no kernel of this library has given up on that device. Reading it
 * synchronises the device. These waits never run out on a healthy GPU.
 */
IPL_API ipl_status ipl_device_fault_flags(int device, uint32_t* flags);

/* Clears the fault word of `device` (synchronous). */
IPL_API ipl_status ipl_clear_device_fault_flags(int device);

/*
 * Name of the kernel that ipl_fused_add_rms_norm_bf16 / ipl_rms_norm_bf16 /
 * ipl_fused_add_rms_norm_static_fp8_quant / ipl_silu_and_mul_bf16 would launch for these
 * arguments on the current device (no launch; the device's SM count and shared-memory limit are
 * read as a call reads them). Where no CUDA device can be queried, a B200's limits are assumed
 * (148 SMs, 232448 bytes of opt-in shared memory per block). Static string; "none" for an empty
 * batch, "invalid" when the arguments would be rejected.
 */
IPL_API const char* ipl_fused_add_rms_norm_plan(const void* x, const void* residual, const void* weight,
                                        int64_t rows, int64_t hidden_size);
IPL_API const char* ipl_rms_norm_plan(const void* output, const void* input, const void* weight,
                                      int64_t rows, int64_t hidden_size);
IPL_API const char* ipl_fused_add_rms_norm_static_fp8_quant_plan(const void* output, const void* input,
                                                                 const void* residual, const void* weight,
                                                                 int64_t rows, int64_t hidden_size);
IPL_API const char* ipl_silu_and_mul_plan(const void* output, const void* input, int64_t rows,
                                  int64_t intermediate_size);

#ifdef __cplusplus
}
#endif

#endif /* IPL_B200_H_ */
