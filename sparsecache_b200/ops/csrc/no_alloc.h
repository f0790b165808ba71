// Allocation-free C entry point of the LM-head + greedy argmax kernel.
//
// This entry point has no counterpart in the reference (forlight123/SparseCache
// allocates everything through PyTorch); it exists for callers of this
// library that cannot allocate device memory themselves.
//
// Who needs it: code that runs where cudaMalloc is unavailable or forbidden:
// a host application that embeds the kernel in a pre-planned memory budget
// (every byte reserved up front, no allocator linked in), a plugin loaded
// into another runtime that owns the device allocator, or a latency-critical
// loop that must never enter the driver's allocation path.  Such callers
// still own their inputs and outputs; what they cannot provide is the
// kernel's scratch space (per-CTA argmax partials and a completion counter).
// That scratch therefore lives in a file-scope device array of fixed size
// inside the library.
//
// Contract:
//   * Inputs: x [M, K] bf16 row-major (row stride K), w [N, K] bf16 row-major,
//     norm_w [K] bf16 or NULL (then x is used without RMSNorm), eps.
//     Output: out_token [M] int32 (device memory), the index of the largest
//     bf16-rounded logit of each row, lowest index on ties (0 for a row none
//     of whose logits compares, i.e. all NaN).
//   * Pointers: x, w and norm_w (when given) must be 16-byte aligned device
//     addresses (the kernel reads them with 16-byte vector loads; a row-major
//     view that starts at a multiple of 8 elements of an aligned buffer
//     qualifies); out_token must be a non-NULL, 4-byte aligned device
//     address.  A NULL or misaligned pointer returns SC_NOALLOC_EBADPOINTER
//     before anything is launched.
//   * Limits: 1 <= M <= SC_NOALLOC_MAX_ROWS, K a multiple of 8, N even,
//     M * K * 2 <= 200 KiB (x is staged in shared memory), and the launch
//     grid (<= 8 CTAs per SM) times M must fit SC_NOALLOC_MAX_PARTIALS.
//     Violations return a non-zero code before anything is launched.
//   * Set-up: the first call on a device (with that device current) looks up
//     the device address of the scratch array with cudaGetSymbolAddress; do
//     this first call before any CUDA stream capture.  The set-up runs once
//     per device under a lock, so host threads may make their first calls at
//     the same time; it is the GPU-side scratch, not the host state, that
//     concurrent calls share (see below).
//   * The scratch array is shared by every call on a device and keeps the
//     last call's contents; the completion counter is cleared (memset on
//     `stream`) at the start of every call.  Calls that overlap on the GPU
//     (different streams without ordering) race on the scratch: order them.
//   * Nothing is allocated: no cudaMalloc, cudaFree or allocating library
//     routine is called.  The scratch costs every GPU that loads the library
//     about 129 KiB of device memory until process exit.
#pragma once

#include <cuda_runtime.h>

#define SC_NOALLOC_MAX_ROWS 8
#define SC_NOALLOC_MAX_PARTIALS 16384

#ifdef __cplusplus
extern "C" {
#endif

// Returns 0 on success, or one of the SC_NOALLOC_E* codes.
int sc_lm_head_argmax_noalloc(const void* x, const void* w, const void* norm_w, float eps, int M,
                              int N, int K, int* out_token, cudaStream_t stream);

// Human-readable message for a return code of sc_lm_head_argmax_noalloc.
const char* sc_noalloc_error_string(int code);

#define SC_NOALLOC_OK 0
#define SC_NOALLOC_EBADSHAPE 1      // M, N or K outside the documented limits
#define SC_NOALLOC_ETOOLARGE 2      // grid * M exceeds SC_NOALLOC_MAX_PARTIALS
#define SC_NOALLOC_ESYMBOL 3        // cudaGetSymbolAddress failed
#define SC_NOALLOC_ELAUNCH 4        // memset or kernel launch failed
#define SC_NOALLOC_EBADPOINTER 5    // NULL or misaligned x / w / norm_w / out_token

#ifdef __cplusplus
}
#endif
