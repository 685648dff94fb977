/* Allocation-free entry points of the dtrain_b200 library (plain C interface).
 *
 * These functions have no counterpart in the reference project.  They are for
 * callers that must not allocate device memory while they run: host runtimes
 * that reserve the whole GPU in their own memory pool before training starts
 * (a cudaMalloc would fail or fragment that pool), latency-sensitive loops that
 * cannot take the device-wide synchronisation cudaMalloc/cudaFree may cause, and
 * programs written in C that do not link torch.  Each such function uses a fixed
 * scratch array compiled into the library instead of allocating a workspace; the
 * caller passes every input and output.
 *
 * Link against the built extension (dtb_C*.so) and include this header.
 */
#ifndef DTB_NOALLOC_H_
#define DTB_NOALLOC_H_

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define DTB_NOALLOC_OK 0
#define DTB_NOALLOC_BAD_ARGUMENT (-1) /* null or misaligned pointer, or an unsupported size */
#define DTB_NOALLOC_TOO_LARGE (-2)    /* the call needs more scratch than the fixed array holds */
#define DTB_NOALLOC_SETUP_FAILED (-3) /* the scratch array's device address could not be found */
#define DTB_NOALLOC_LAUNCH_FAILED (-4) /* a kernel launch failed (the CUDA error is cleared) */
#define DTB_NOALLOC_PRIOR_ERROR (-5)   /* a CUDA error was already pending on entry (left as is) */

/* Capacity of the LayerNorm-backward scratch array, in floats (4 MiB per device).
 * A call needs 2 * ceil(rows / 64) * C floats: at C = 768 up to 43,648 rows. */
#define DTB_LN_NOALLOC_SCRATCH_FLOATS (1L << 20)

/* LayerNorm backward without allocation.
 *
 * dx[r, c] = rstd[r] * (g - mean_c(g) - xhat * mean_c(g * xhat)) + dresid[r, c], with
 * g = dy * w and xhat = (x - mean) * rstd; dw = sum_r dy * xhat, db = sum_r dy
 * (written, or added to dw/db when accumulate != 0), reduced in a fixed order so
 * the bits do not depend on scheduling.
 *
 * dy, x, dresid (may be NULL), dx: bf16 [rows, C], 16-byte aligned; w: bf16 [C],
 * 16-byte aligned; mean, rstd: fp32 [rows]; dw, db: fp32 [C].  C is a multiple
 * of 8 and at most 2048.  Work is enqueued on `stream`; the function returns
 * before it runs.
 *
 * Scratch: one array per device, shared by every call and keeping the previous
 * call's contents (each call writes every partial it reads, so nothing needs to
 * start at zero).  Calls that overlap on the GPU - on different streams, or from
 * host threads without ordering - race on it: serialise calls on a device.  The
 * first call on a device (with that device current) looks up the array's device
 * address and caches it per CUDA context; make that first call before any
 * stream capture.  The function calls no cudaMalloc, cudaFree or allocating
 * library routine.
 */
int dtb_layernorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* mean, const float* rstd,
                              const void* dresid, void* dx, float* dw, float* db, int rows, int C, int accumulate,
                              cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DTB_NOALLOC_H_ */
