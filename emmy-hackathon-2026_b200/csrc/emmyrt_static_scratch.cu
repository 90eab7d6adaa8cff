/*
 * Whole-array reductions without allocating anything.
 *
 * The whole-array reduction kernels (global sum, mean, max, sum of squares) need a
 * small scratch area beside their input and output: one partial per CTA plus the
 * ticket word the last CTA uses to finish the reduction.  The regular path has the
 * caller (the runner) allocate that scratch with the CUDA driver.
 *
 * Some callers cannot allocate device memory at the point where they want a
 * reduction: a process that hands all of HBM to its own pool at start-up and may
 * not call cudaMalloc afterwards, an error path that runs after an out-of-memory
 * failure (and wants a norm or a checksum of what is on the device), or a
 * latency-bound loop where cudaMalloc / cudaFree and the synchronisation they
 * imply are not acceptable.  For them this file provides one entry point that
 * launches the same reduction kernel with its scratch taken from a file-scope
 * device array instead:
 *
 *   - the array holds EMMY_RT_STATIC_SCRATCH_BYTES (64 KiB); it is zero-filled when
 *     the library is loaded, and every GPU that loads this library keeps its own
 *     copy until the process exits;
 *   - the kernel writes a 16-byte ticket and one 8-byte partial per CTA, so a launch
 *     of `grid` CTAs needs 16 + 8 * grid bytes whatever the caller claims in
 *     `scratch_bytes`; a launch whose need (the larger of the two) exceeds the array
 *     is rejected with EMMY_RT_ESCRATCH before anything is enqueued (at most 8190
 *     CTAs fit);
 *   - the array's device address is looked up once per device with
 *     cudaGetSymbolAddress on that device's first call (with that device current).
 *     That first call on a device therefore does the set-up; make it before any
 *     stream capture.  The address belongs to the device's primary context: after
 *     a reset of that context (cudaDeviceReset) the cached address is stale, so a
 *     process that resets a device must not call this entry point on it again;
 *   - every call shares the one array and it keeps the last call's contents.  The
 *     ticket word at its head must start at zero, so each call clears it on the
 *     stream (cudaMemsetAsync, which allocates nothing) before the launch.  Two
 *     calls whose kernels overlap on the GPU race on the array: serialise them
 *     (one stream, or events) when they run on the same device.
 *
 * Nothing here calls cudaMalloc, cudaFree or any other allocating routine.
 */
#include <cuda_runtime.h>
#include <stdint.h>

#include "emmyrt.h"

static __device__ __align__(256) unsigned char g_reduce_scratch[EMMY_RT_STATIC_SCRATCH_BYTES];

/* device address of g_reduce_scratch per device ordinal, filled on first use; host
 * threads that race on the first call store the same value, atomically */
static void *g_scratch_addr[64];

/* bytes the whole-array reduction kernel writes for a launch of `grid` CTAs */
static size_t scratch_need(unsigned grid) { return 16 + 8 * (size_t)grid; }

#define MAX_ARGS 62

extern "C" __attribute__((visibility("default")))
int emmy_rt_full_reduce_static_scratch(uint64_t function, unsigned grid, unsigned block,
                                       const uint64_t *args, int nargs, size_t scratch_bytes,
                                       uint64_t stream) {
    if (nargs < 0 || nargs > MAX_ARGS || (nargs > 0 && args == NULL) || grid == 0 || block == 0)
        return EMMY_RT_EINVAL;
    size_t need = scratch_need(grid);
    if (scratch_bytes > need) need = scratch_bytes;
    if (need > EMMY_RT_STATIC_SCRATCH_BYTES)
        return EMMY_RT_ESCRATCH;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return EMMY_RT_EINVAL;
    void *base = __atomic_load_n(&g_scratch_addr[dev], __ATOMIC_ACQUIRE);
    if (base == NULL) {
        e = cudaGetSymbolAddress(&base, g_reduce_scratch);
        if (e != cudaSuccess) return (int)e;
        __atomic_store_n(&g_scratch_addr[dev], base, __ATOMIC_RELEASE);
    }
    /* the ticket (first 16 bytes) must read zero when the kernel starts */
    e = cudaMemsetAsync(base, 0, 16, (cudaStream_t)(uintptr_t)stream);
    if (e != cudaSuccess) return (int)e;
    uint64_t vals[MAX_ARGS + 1];
    void *params[MAX_ARGS + 1];
    for (int i = 0; i < nargs; ++i) {
        vals[i] = args[i];
        params[i] = &vals[i];
    }
    vals[nargs] = (uint64_t)(uintptr_t)base;
    params[nargs] = &vals[nargs];
    const unsigned g[3] = {grid, 1, 1}, b[3] = {block, 1, 1};
    return emmy_rt_launch(function, g, b, NULL, 0, stream, params);
}
