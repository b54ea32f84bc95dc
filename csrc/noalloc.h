// C interface of the allocation-free entry points (noalloc.cu). No counterpart in the reference implementation.
//
// For callers that may not allocate device memory: every buffer is passed in, and the only scratch space is a
// fixed-size static device array (QW_NOALLOC_SCRATCH_FLOATS floats) that each GPU loading the library keeps until
// the process exits. Two rules follow from that array: calls that can overlap on the GPU (streams with no order
// between them) race on it, and the first call on each device looks up the array's device address, so it must
// come before any stream capture. dy, x and dx must be 16-byte aligned. See noalloc.cu for the full contract.
#pragma once

#define QW_NOALLOC_API __attribute__((visibility("default")))

#define QW_NOALLOC_SCRATCH_FLOATS 4194304  // 16 MiB of fp32 partial sums

#define QW_NOALLOC_OK 0
#define QW_NOALLOC_BAD_ARGUMENT 1
#define QW_NOALLOC_TOO_LARGE 2
#define QW_NOALLOC_CUDA_ERROR 3
#define QW_NOALLOC_PENDING_ERROR 4

#ifdef __cplusplus
extern "C" {
#endif

// RMSNorm backward without any allocation. Returns QW_NOALLOC_OK or one of the error codes above.
QW_NOALLOC_API int qw_rmsnorm_backward_noalloc(const void* dy, const void* x, const float* weight, const float* rstd,
                                               void* dx, float* dweight, long long rows, int hidden, void* stream);

// Human-readable text for a return code of the functions above.
QW_NOALLOC_API const char* qw_noalloc_error_message(int code);

// Capacity of the static scratch array, in floats.
QW_NOALLOC_API long long qw_noalloc_scratch_floats(void);

#ifdef __cplusplus
}
#endif
