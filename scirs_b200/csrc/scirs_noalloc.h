// C declarations of the no-allocation entry points of the scirs_b200 kernel
// library (exported with C linkage from scirs_b200/_C*.so).
//
// These entry points have no counterpart in the reference (krharrison/scirs):
// they exist for callers that cannot allocate device memory at the point of
// the call, such as C or other-language hosts that drive the kernels inside a
// fixed device-memory budget and have no allocator of their own, or code that
// must not call cudaMalloc where it runs (cudaMalloc can synchronise the
// device). Their scratch memory is a fixed-size array inside the library
// instead of a caller-provided buffer.
//
// Common rules:
//   * No call allocates or frees memory: no cudaMalloc / cudaFree and no
//     allocating library routine (PyTorch's allocator included).
//   * Every GPU that loads the library holds the scratch array
//     (SCIRS_NOALLOC_SCRATCH_BYTES) until the process exits.
//   * The first call on a device looks up the array's device address (with
//     cudaGetSymbolAddress, that device current). Make that first call before
//     any stream capture on the device; later calls do no set-up.
//   * All calls on a device share the one array and it keeps the last call's
//     contents. Calls whose executions overlap on the GPU (unordered streams,
//     or several host threads) race on it: serialise them.
//   * The calling thread's current device and the stream passed in select
//     where the work runs; all pointers are device pointers on that device.
//   * If an error from earlier, unrelated work is already pending on the
//     calling thread (cudaPeekAtLastError() != cudaSuccess), the call returns
//     that error code without launching anything and leaves it pending.
//
// Return value: 0 on success; a negative SCIRS_NOALLOC_E* code on invalid
// arguments (scirs_noalloc_last_error() then returns a message); or a positive
// cudaError_t value from the CUDA runtime.
#ifndef SCIRS_NOALLOC_H_
#define SCIRS_NOALLOC_H_

#ifdef __cplusplus
extern "C" {
#endif

// Size of the shared scratch array: 2^20 fp32 values (4 MiB) per device.
#define SCIRS_NOALLOC_SCRATCH_FLOATS (1L << 20)
#define SCIRS_NOALLOC_SCRATCH_BYTES (SCIRS_NOALLOC_SCRATCH_FLOATS * 4L)
// Widest LayerNorm row the scratch can serve (one block needs 3 * D floats).
#define SCIRS_NOALLOC_LN_MAX_D ((int)(SCIRS_NOALLOC_SCRATCH_FLOATS / 3))

#define SCIRS_NOALLOC_EARG (-1)       // rows <= 0, rows > INT_MAX, or D not a positive multiple of 8
#define SCIRS_NOALLOC_ETOOBIG (-2)    // D > SCIRS_NOALLOC_LN_MAX_D
#define SCIRS_NOALLOC_ENULL (-3)      // a required pointer is NULL
#define SCIRS_NOALLOC_EDEVICE (-4)    // current device index outside 0..63
#define SCIRS_NOALLOC_EALIGN (-5)     // a bf16 pointer is not 2-byte or an fp32 pointer not 4-byte aligned

// LayerNorm backward over `rows` rows of width D (bf16 data, fp32 statistics):
//   dx   [rows, D] bf16 (written)  = d loss / d x (+ dresid if not NULL)
//   dw   [D] fp32 (accumulated)    += sum over rows of dy * x_hat
//   db   [D] fp32 (accumulated)    += sum over rows of dy
//   dsum [D] fp32 (accumulated, optional, may be NULL) += column sums of dx
// dy, x, dresid: [rows, D] bf16, row-major, contiguous; w: [D] bf16;
// mean, rstd: [rows] fp32 (the forward's row statistics). Pointers that are
// not 16-byte aligned are served by a scalar-load kernel (slower, same
// result). Same math and kernels as the library's regular layernorm_bwd.
int scirs_layernorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* mean,
                                const float* rstd, const void* dresid, void* dx, float* dw, float* db,
                                float* dsum, long long rows, int D, void* stream);

// Message describing the last negative return code on the calling thread
// ("" after a successful call).
const char* scirs_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif

#endif  // SCIRS_NOALLOC_H_
