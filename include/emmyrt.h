/*
 * emmyrt -- the native launch runtime of the B200 back end for Emmy Kernel IR.
 *
 * The reference compiler (prathamesh-chavan-22/emmy-hackathon-2026) hands its PTX to
 * a remote HTTP runner (submit.py; docs/API.md) that assembles it with ptxas, fills
 * the arguments, launches the kernel once and returns the outputs.  This library is
 * the local replacement for that runner: a plain C ABI over the CUDA driver API (and
 * NCCL for the one collective), loaded with ctypes by the Python host side.
 *
 * Conventions
 *   - every entry point returns an int status: 0 on success, a CUresult / ncclResult
 *     value (> 0) from the failing driver call, or a negative EMMY_RT_E* code;
 *     emmy_rt_last_error() then describes the failure (per thread);
 *   - device pointers, modules, functions, streams, events and communicators are
 *     opaque 64-bit handles; no C++ or torch types cross the boundary;
 *   - libcuda and libnccl are opened lazily with dlopen, so the library loads (and
 *     its symbols can be listed) on a host without a GPU.
 *
 * Citations name the reference file and line range each entry point replaces.
 */
#ifndef EMMYRT_H
#define EMMYRT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMMY_RT_VERSION 1

/* negative status codes (positive ones are CUresult / ncclResult_t values) */
#define EMMY_RT_ENOLIB    (-1)   /* libcuda / libnccl could not be opened        */
#define EMMY_RT_ENOSYM    (-2)   /* a required driver symbol is missing           */
#define EMMY_RT_EINVAL    (-3)   /* bad argument                                  */
#define EMMY_RT_ETIMEOUT  (-4)   /* emmy_rt_stream_wait deadline passed           */
#define EMMY_RT_ENOINIT   (-5)   /* emmy_rt_init was not called                   */
#define EMMY_RT_ESCRATCH  (-6)   /* scratch larger than the static array          */

/* ---- errors ------------------------------------------------------------------ */

/* Text of the last failure on this thread ("" when none).
 * Replaces the runner's `stderr` field of a failed /compile or /run
 * (docs/API.md:12-24, submit.py:101-103). */
const char *emmy_rt_last_error(void);

/* EMMY_RT_VERSION of the loaded library. */
int emmy_rt_version(void);

/* ---- device / context ------------------------------------------------------------ */

/* Open libcuda, cuInit, retain `device`'s primary context and make it current on the
 * calling thread.  The runner's GET /health (docs/API.md:5-9) reported its GPU; this is
 * the local equivalent and must precede every other call below except the NCCL loader. */
int emmy_rt_init(int device);

/* Number of visible devices (after emmy_rt_init). */
int emmy_rt_device_count(int *count);

/* cuDeviceGetAttribute(attr) of `device` (e.g. 16 = multiprocessor count,
 * 75/76 = compute capability major/minor). */
int emmy_rt_device_attribute(int attr, int device, int *value);

/* Make `device`'s primary context current on the calling thread. */
int emmy_rt_set_device(int device);

/* Block until all work on the current context has finished. */
int emmy_rt_synchronize(void);

/* ---- modules (replaces POST /compile: submit.py:99-110, docs/API.md:12-24) ------ */

/* Load a module image: a NUL-terminated PTX text (JIT-assembled by the driver) or a
 * cubin written by ptxas.  *module receives an opaque handle. */
int emmy_rt_module_load(const void *image, size_t nbytes, uint64_t *module);
int emmy_rt_module_unload(uint64_t module);

/* Look up an .entry by name (the runner's entry_points check, submit.py:107-110). */
int emmy_rt_module_function(uint64_t module, const char *entry, uint64_t *function);

/* Address and size of a module-scope .global variable. */
int emmy_rt_module_global(uint64_t module, const char *name, uint64_t *dptr, size_t *bytes);

/* cuFuncGetAttribute(attr) (4 = registers per thread, the runner's `registers`
 * field, docs/API.md:23-24; 1 = static shared bytes; 0 = max threads per block). */
int emmy_rt_function_attribute(uint64_t function, int attr, int *value);

/* Allow up to `bytes` of dynamic shared memory for `function` (> 48 KB needs this). */
int emmy_rt_function_set_max_dynamic_smem(uint64_t function, int bytes);

/* ---- launch (replaces POST /run's launch: submit.py:126-135, docs/API.md:26-53) -- */

/* Launch `function` on `stream` (0 = the legacy default stream) with the given grid,
 * block, thread-block-cluster shape (cluster = NULL or {1,1,1} for none) and dynamic
 * shared memory.  `params[i]` points at the value of kernel parameter i, exactly as
 * cuLaunchKernel takes them (a tensor map parameter points at its 128 bytes). */
int emmy_rt_launch(uint64_t function, const unsigned grid[3], const unsigned block[3],
                   const unsigned cluster[3], unsigned smem_bytes, uint64_t stream,
                   void **params);

/* Launch flags of emmy_rt_launch_ex. */
#define EMMY_RT_LAUNCH_PDL 1u   /* programmatic dependent launch (see below) */

/* emmy_rt_launch with flags (same role: the reference runner's POST /run launch,
 * docs/API.md:26-53).  EMMY_RT_LAUNCH_PDL lets the kernel start while the stream's previous
 * kernel finishes (CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION): only for modules
 * whose launch descriptor says "pdl": true, which wait for the previous kernel
 * (griddepcontrol.wait) before their first global memory access.  Unknown flags:
 * EMMY_RT_EINVAL. */
int emmy_rt_launch_ex(uint64_t function, const unsigned grid[3], const unsigned block[3],
                      const unsigned cluster[3], unsigned smem_bytes, uint64_t stream,
                      void **params, unsigned flags);

/* ---- TMA descriptors (new: the reference never emits TMA, TASK.md:130-136) ------- */

/* cuTensorMapEncodeTiled into the 128-byte, 64-byte-aligned buffer `out`.
 * dims/box/elem_strides have `rank` entries (innermost first); strides_bytes has
 * rank-1 entries (the byte stride of dims 1..rank-1).  dtype, interleave, swizzle,
 * l2promo and oobfill take the CUtensorMap* enum values. */
int emmy_rt_tensor_map_encode_tiled(void *out, int dtype, unsigned rank, uint64_t gaddr,
                                    const uint64_t *dims, const uint64_t *strides_bytes,
                                    const unsigned *box, const unsigned *elem_strides,
                                    int interleave, int swizzle, int l2promo, int oobfill);

/* ---- memory (the runner allocated, filled and returned buffers itself:
 *      docs/API.md:40-53, submit.py:113-122) ---------------------------------------- */

int emmy_rt_mem_alloc(uint64_t *dptr, size_t bytes);
int emmy_rt_mem_free(uint64_t dptr);
int emmy_rt_mem_info(size_t *free_bytes, size_t *total_bytes);
/* page-locked host memory, so copies are asynchronous and run at full PCIe rate */
int emmy_rt_host_alloc(void **ptr, size_t bytes);
int emmy_rt_host_free(void *ptr);
int emmy_rt_memcpy_htod(uint64_t dst, const void *src, size_t bytes, uint64_t stream);
int emmy_rt_memcpy_dtoh(void *dst, uint64_t src, size_t bytes, uint64_t stream);
int emmy_rt_memcpy_dtod(uint64_t dst, uint64_t src, size_t bytes, uint64_t stream);
/* the runner's zero_outputs re-zeroing before every launch (docs/API.md:51-53) */
int emmy_rt_memset(uint64_t dst, unsigned char value, size_t bytes, uint64_t stream);

/* ---- streams and events (the runner's median_us timing, docs/API.md:36,77) -------- */

int emmy_rt_stream_create(uint64_t *stream);
int emmy_rt_stream_destroy(uint64_t stream);
int emmy_rt_stream_synchronize(uint64_t stream);
/* Poll the stream until it is idle or `timeout_s` seconds pass (EMMY_RT_ETIMEOUT):
 * the runner's 20 s launch limit (docs/API.md:69) without blocking forever. */
int emmy_rt_stream_wait(uint64_t stream, double timeout_s);
/* Work queued on `stream` after this call starts once `event`'s latest recording has
 * completed (cuStreamWaitEvent): copies of the next step overlap the current kernel.
 * The runner ran one launch at a time (submit.py:126-135); this orders streams of a
 * pipelined run instead. */
int emmy_rt_stream_wait_event(uint64_t stream, uint64_t event);
int emmy_rt_event_create(uint64_t *event);
int emmy_rt_event_destroy(uint64_t event);
int emmy_rt_event_record(uint64_t event, uint64_t stream);
int emmy_rt_event_synchronize(uint64_t event);
int emmy_rt_event_elapsed_ms(uint64_t start, uint64_t end, float *ms);

/* ---- CUDA graphs (new: the runner launched one kernel per request, submit.py:126-135;
 *      a sequence of short launches replays as one graph without per-launch host cost) */

/* Start capturing the work queued on `stream` (not the legacy stream 0; thread-local
 * capture mode).  Launches made on it until emmy_rt_graph_end are recorded, not run. */
int emmy_rt_graph_begin(uint64_t stream);
/* Stop capturing and instantiate the recorded work: *graph receives the executable. */
int emmy_rt_graph_end(uint64_t stream, uint64_t *graph);
/* Run the captured work on `stream` (any stream, 0 included). */
int emmy_rt_graph_launch(uint64_t graph, uint64_t stream);
/* Stage the graph on the device ahead of its first launch (nothing runs). */
int emmy_rt_graph_upload(uint64_t graph, uint64_t stream);
int emmy_rt_graph_destroy(uint64_t graph);

/* ---- NCCL (new: the reference has no collective; one all-reduce finishes the
 *      sharded global sum) ------------------------------------------------------- */

/* dlopen libnccl (path NULL = "libnccl.so.2" from the loader path). */
int emmy_rt_nccl_load(const char *path);
/* ncclGetUniqueId into the 128-byte buffer `id` (rank 0 shares it with the others). */
int emmy_rt_nccl_unique_id(void *id);
int emmy_rt_nccl_comm_init(uint64_t *comm, int nranks, const void *id, int rank);
/* ncclAllReduce; dtype / op take ncclDataType_t / ncclRedOp_t values
 * (7 = ncclFloat32, 8 = ncclFloat64; 0 = ncclSum). */
int emmy_rt_nccl_allreduce(uint64_t comm, uint64_t sendbuf, uint64_t recvbuf, size_t count,
                           int dtype, int op, uint64_t stream);
int emmy_rt_nccl_comm_destroy(uint64_t comm);

/* ---- whole-array reduction with static scratch (libemmyrt_static.so) ------------- */

/* Size of the device array emmy_rt_full_reduce_static_scratch takes scratch from. */
#define EMMY_RT_STATIC_SCRATCH_BYTES (64 * 1024)

/* No counterpart in the reference: an addition for callers that cannot allocate device
 * memory where they need a reduction (a process whose HBM is all handed to its own pool,
 * an error path after an out-of-memory failure, a latency-bound loop that must not pay
 * for cudaMalloc).  Launches a whole-array reduction kernel compiled by this back end
 * (`function`, from emmy_rt_module_function; grid and block from its launch descriptor)
 * with `args` = its nargs pointer arguments in meta.json arg_order and its scratch taken
 * from a file-scope device array of EMMY_RT_STATIC_SCRATCH_BYTES instead of an allocation.
 * The kernel writes 16 + 8 * grid bytes of scratch; a launch whose need (that, or
 * scratch_bytes if larger) exceeds the array is rejected with EMMY_RT_ESCRATCH.  The first
 * call on a device looks the array up (cudaGetSymbolAddress) and should come before any
 * stream capture; the address is cached for the life of the process, so a device whose
 * primary context was reset (cudaDeviceReset) must not be passed here again.  Calls share the array: each clears its ticket word on `stream` first, and
 * calls whose kernels overlap on the GPU race.  Returns 0, EMMY_RT_EINVAL /
 * EMMY_RT_ESCRATCH, a cudaError_t from the set-up or the clear, or emmy_rt_launch's
 * status. */
int emmy_rt_full_reduce_static_scratch(uint64_t function, unsigned grid, unsigned block,
                                       const uint64_t *args, int nargs, size_t scratch_bytes,
                                       uint64_t stream);

#ifdef __cplusplus
}
#endif

#endif /* EMMYRT_H */
