/*
 * emmyrt: C-ABI launch runtime over the CUDA driver API and NCCL.
 * The interface and its reference citations are in include/emmyrt.h.
 *
 * libcuda.so.1 and libnccl.so.2 are opened with dlopen on first use, and every driver
 * entry point is resolved through cuGetProcAddress for the CUDA 12 ABI, so the shared
 * object has no link-time dependency on either and loads on a GPU-less host.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include <cuda.h>

#include "emmyrt.h"

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ errors */

static __thread char g_err[1024];

static int fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return status;
}

EXPORT const char *emmy_rt_last_error(void) { return g_err; }
EXPORT int emmy_rt_version(void) { return EMMY_RT_VERSION; }

/* ------------------------------------------------------------ driver table */

typedef CUresult (*pfn_getproc)(const char *, void **, int, cuuint64_t,
                                CUdriverProcAddressQueryResult *);

static struct {
    void *lib;
    int ready;
    CUresult (*Init)(unsigned);
    CUresult (*GetErrorString)(CUresult, const char **);
    CUresult (*GetErrorName)(CUresult, const char **);
    CUresult (*DeviceGet)(CUdevice *, int);
    CUresult (*DeviceGetCount)(int *);
    CUresult (*DeviceGetAttribute)(int *, CUdevice_attribute, CUdevice);
    CUresult (*DevicePrimaryCtxRetain)(CUcontext *, CUdevice);
    CUresult (*CtxSetCurrent)(CUcontext);
    CUresult (*CtxSynchronize)(void);
    CUresult (*ModuleLoadDataEx)(CUmodule *, const void *, unsigned, CUjit_option *, void **);
    CUresult (*ModuleUnload)(CUmodule);
    CUresult (*ModuleGetFunction)(CUfunction *, CUmodule, const char *);
    CUresult (*ModuleGetGlobal)(CUdeviceptr *, size_t *, CUmodule, const char *);
    CUresult (*FuncGetAttribute)(int *, CUfunction_attribute, CUfunction);
    CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
    CUresult (*LaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **, void **);
    CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                     const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                     const cuuint32_t *, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion,
                                     CUtensorMapFloatOOBfill);
    CUresult (*MemAlloc)(CUdeviceptr *, size_t);
    CUresult (*MemFree)(CUdeviceptr);
    CUresult (*MemGetInfo)(size_t *, size_t *);
    CUresult (*MemHostAlloc)(void **, size_t, unsigned);
    CUresult (*MemFreeHost)(void *);
    CUresult (*MemcpyHtoDAsync)(CUdeviceptr, const void *, size_t, CUstream);
    CUresult (*MemcpyDtoHAsync)(void *, CUdeviceptr, size_t, CUstream);
    CUresult (*MemcpyDtoDAsync)(CUdeviceptr, CUdeviceptr, size_t, CUstream);
    CUresult (*MemsetD8Async)(CUdeviceptr, unsigned char, size_t, CUstream);
    CUresult (*StreamCreate)(CUstream *, unsigned);
    CUresult (*StreamDestroy)(CUstream);
    CUresult (*StreamSynchronize)(CUstream);
    CUresult (*StreamQuery)(CUstream);
    CUresult (*StreamWaitEvent)(CUstream, CUevent, unsigned);
    CUresult (*StreamBeginCapture)(CUstream, CUstreamCaptureMode);
    CUresult (*StreamEndCapture)(CUstream, CUgraph *);
    CUresult (*GraphInstantiateWithFlags)(CUgraphExec *, CUgraph, unsigned long long);
    CUresult (*GraphLaunch)(CUgraphExec, CUstream);
    CUresult (*GraphUpload)(CUgraphExec, CUstream);
    CUresult (*GraphExecDestroy)(CUgraphExec);
    CUresult (*GraphDestroy)(CUgraph);
    CUresult (*EventCreate)(CUevent *, unsigned);
    CUresult (*EventDestroy)(CUevent);
    CUresult (*EventRecord)(CUevent, CUstream);
    CUresult (*EventSynchronize)(CUevent);
    CUresult (*EventElapsedTime)(float *, CUevent, CUevent);
} cu;

static CUcontext g_ctx[64];

static int cu_fail(CUresult r, const char *what) {
    const char *name = "?", *text = "?";
    if (cu.GetErrorName) cu.GetErrorName(r, &name);
    if (cu.GetErrorString) cu.GetErrorString(r, &text);
    return fail((int)r, "%s failed: %s (%s)", what, name ? name : "?", text ? text : "?");
}

#define CU(call, what)                              \
    do {                                            \
        CUresult r_ = (call);                       \
        if (r_ != CUDA_SUCCESS) return cu_fail(r_, what); \
    } while (0)

#define NEED_INIT()                                                   \
    do {                                                              \
        if (!cu.ready) return fail(EMMY_RT_ENOINIT, "emmy_rt_init was not called"); \
    } while (0)

static int load_driver(void) {
    if (cu.ready) return 0;
    if (!cu.lib) cu.lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!cu.lib) return fail(EMMY_RT_ENOLIB, "cannot open libcuda.so.1: %s", dlerror());
    pfn_getproc getproc = (pfn_getproc)dlsym(cu.lib, "cuGetProcAddress_v2");
    if (!getproc) return fail(EMMY_RT_ENOSYM, "libcuda has no cuGetProcAddress_v2 (driver too old)");
    struct { const char *name; void **slot; } table[] = {
#define E(sym, field) {#sym, (void **)&cu.field}
        E(cuInit, Init), E(cuGetErrorString, GetErrorString), E(cuGetErrorName, GetErrorName),
        E(cuDeviceGet, DeviceGet), E(cuDeviceGetCount, DeviceGetCount),
        E(cuDeviceGetAttribute, DeviceGetAttribute),
        E(cuDevicePrimaryCtxRetain, DevicePrimaryCtxRetain), E(cuCtxSetCurrent, CtxSetCurrent),
        E(cuCtxSynchronize, CtxSynchronize), E(cuModuleLoadDataEx, ModuleLoadDataEx),
        E(cuModuleUnload, ModuleUnload), E(cuModuleGetFunction, ModuleGetFunction),
        E(cuModuleGetGlobal, ModuleGetGlobal), E(cuFuncGetAttribute, FuncGetAttribute),
        E(cuFuncSetAttribute, FuncSetAttribute), E(cuLaunchKernelEx, LaunchKernelEx),
        E(cuTensorMapEncodeTiled, TensorMapEncodeTiled), E(cuMemAlloc, MemAlloc),
        E(cuMemFree, MemFree), E(cuMemGetInfo, MemGetInfo), E(cuMemHostAlloc, MemHostAlloc),
        E(cuMemFreeHost, MemFreeHost), E(cuMemcpyHtoDAsync, MemcpyHtoDAsync),
        E(cuMemcpyDtoHAsync, MemcpyDtoHAsync), E(cuMemcpyDtoDAsync, MemcpyDtoDAsync),
        E(cuMemsetD8Async, MemsetD8Async), E(cuStreamCreate, StreamCreate),
        E(cuStreamDestroy, StreamDestroy), E(cuStreamSynchronize, StreamSynchronize),
        E(cuStreamQuery, StreamQuery), E(cuStreamWaitEvent, StreamWaitEvent),
        E(cuStreamBeginCapture, StreamBeginCapture), E(cuStreamEndCapture, StreamEndCapture),
        E(cuGraphInstantiateWithFlags, GraphInstantiateWithFlags), E(cuGraphLaunch, GraphLaunch),
        E(cuGraphUpload, GraphUpload),
        E(cuGraphExecDestroy, GraphExecDestroy), E(cuGraphDestroy, GraphDestroy),
        E(cuEventCreate, EventCreate),
        E(cuEventDestroy, EventDestroy), E(cuEventRecord, EventRecord),
        E(cuEventSynchronize, EventSynchronize), E(cuEventElapsedTime, EventElapsedTime),
#undef E
    };
    for (size_t i = 0; i < sizeof table / sizeof table[0]; ++i) {
        CUdriverProcAddressQueryResult q;
        CUresult r = getproc(table[i].name, table[i].slot, 12000, CU_GET_PROC_ADDRESS_DEFAULT, &q);
        if (r != CUDA_SUCCESS || *table[i].slot == NULL)
            return fail(EMMY_RT_ENOSYM, "driver symbol %s not found", table[i].name);
    }
    CU(cu.Init(0), "cuInit");
    cu.ready = 1;
    return 0;
}

/* ------------------------------------------------------------- device/ctx */

EXPORT int emmy_rt_set_device(int device) {
    NEED_INIT();
    if (device < 0 || device >= 64) return fail(EMMY_RT_EINVAL, "device %d out of range", device);
    if (!g_ctx[device]) {
        CUdevice dev;
        CU(cu.DeviceGet(&dev, device), "cuDeviceGet");
        CU(cu.DevicePrimaryCtxRetain(&g_ctx[device], dev), "cuDevicePrimaryCtxRetain");
    }
    CU(cu.CtxSetCurrent(g_ctx[device]), "cuCtxSetCurrent");
    return 0;
}

EXPORT int emmy_rt_init(int device) {
    int s = load_driver();
    if (s) return s;
    return emmy_rt_set_device(device);
}

EXPORT int emmy_rt_device_count(int *count) {
    NEED_INIT();
    CU(cu.DeviceGetCount(count), "cuDeviceGetCount");
    return 0;
}

EXPORT int emmy_rt_device_attribute(int attr, int device, int *value) {
    NEED_INIT();
    CUdevice dev;
    CU(cu.DeviceGet(&dev, device), "cuDeviceGet");
    CU(cu.DeviceGetAttribute(value, (CUdevice_attribute)attr, dev), "cuDeviceGetAttribute");
    return 0;
}

EXPORT int emmy_rt_synchronize(void) {
    NEED_INIT();
    CU(cu.CtxSynchronize(), "cuCtxSynchronize");
    return 0;
}

/* ---------------------------------------------------------------- modules */

EXPORT int emmy_rt_module_load(const void *image, size_t nbytes, uint64_t *module) {
    NEED_INIT();
    (void)nbytes;
    if (!image || !module) return fail(EMMY_RT_EINVAL, "null image or module");
    char info[4096] = {0}, err[8192] = {0};
    CUjit_option opts[] = {CU_JIT_INFO_LOG_BUFFER, CU_JIT_INFO_LOG_BUFFER_SIZE_BYTES,
                           CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
    void *vals[] = {info, (void *)(uintptr_t)sizeof info, err, (void *)(uintptr_t)sizeof err};
    CUmodule m;
    CUresult r = cu.ModuleLoadDataEx(&m, image, 4, opts, vals);
    if (r != CUDA_SUCCESS) {
        const char *name = "?";
        if (cu.GetErrorName) cu.GetErrorName(r, &name);
        return fail((int)r, "cuModuleLoadDataEx failed: %s\n%s", name, err);
    }
    *module = (uint64_t)(uintptr_t)m;
    return 0;
}

EXPORT int emmy_rt_module_unload(uint64_t module) {
    NEED_INIT();
    CU(cu.ModuleUnload((CUmodule)(uintptr_t)module), "cuModuleUnload");
    return 0;
}

EXPORT int emmy_rt_module_function(uint64_t module, const char *entry, uint64_t *function) {
    NEED_INIT();
    CUfunction f;
    CUresult r = cu.ModuleGetFunction(&f, (CUmodule)(uintptr_t)module, entry);
    if (r != CUDA_SUCCESS) return cu_fail(r, entry ? entry : "cuModuleGetFunction");
    *function = (uint64_t)(uintptr_t)f;
    return 0;
}

EXPORT int emmy_rt_module_global(uint64_t module, const char *name, uint64_t *dptr, size_t *bytes) {
    NEED_INIT();
    CUdeviceptr p;
    size_t n;
    CU(cu.ModuleGetGlobal(&p, &n, (CUmodule)(uintptr_t)module, name), "cuModuleGetGlobal");
    if (dptr) *dptr = (uint64_t)p;
    if (bytes) *bytes = n;
    return 0;
}

EXPORT int emmy_rt_function_attribute(uint64_t function, int attr, int *value) {
    NEED_INIT();
    CU(cu.FuncGetAttribute(value, (CUfunction_attribute)attr, (CUfunction)(uintptr_t)function),
       "cuFuncGetAttribute");
    return 0;
}

EXPORT int emmy_rt_function_set_max_dynamic_smem(uint64_t function, int bytes) {
    NEED_INIT();
    CU(cu.FuncSetAttribute((CUfunction)(uintptr_t)function,
                           CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, bytes),
       "cuFuncSetAttribute(max dynamic smem)");
    return 0;
}

/* ----------------------------------------------------------------- launch */

EXPORT int emmy_rt_launch_ex(uint64_t function, const unsigned grid[3], const unsigned block[3],
                             const unsigned cluster[3], unsigned smem_bytes, uint64_t stream,
                             void **params, unsigned flags) {
    NEED_INIT();
    if (!grid || !block) return fail(EMMY_RT_EINVAL, "null grid or block");
    if (flags & ~(unsigned)EMMY_RT_LAUNCH_PDL) return fail(EMMY_RT_EINVAL, "unknown launch flags %#x", flags);
    CUlaunchConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDimX = grid[0]; cfg.gridDimY = grid[1]; cfg.gridDimZ = grid[2];
    cfg.blockDimX = block[0]; cfg.blockDimY = block[1]; cfg.blockDimZ = block[2];
    cfg.sharedMemBytes = smem_bytes;
    cfg.hStream = (CUstream)(uintptr_t)stream;
    CUlaunchAttribute attr[2];
    memset(attr, 0, sizeof attr);
    unsigned n = 0;
    if (cluster && (cluster[0] * cluster[1] * cluster[2]) > 1) {
        attr[n].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        attr[n].value.clusterDim.x = cluster[0];
        attr[n].value.clusterDim.y = cluster[1];
        attr[n].value.clusterDim.z = cluster[2];
        ++n;
    }
    if (flags & EMMY_RT_LAUNCH_PDL) {
        /* the kernel may start while the previous kernel of the stream finishes; it waits
         * for that kernel (griddepcontrol.wait) before its first global memory access */
        attr[n].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attr[n].value.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (n) {
        cfg.attrs = attr;
        cfg.numAttrs = n;
    }
    CU(cu.LaunchKernelEx(&cfg, (CUfunction)(uintptr_t)function, params, NULL), "cuLaunchKernelEx");
    return 0;
}

EXPORT int emmy_rt_launch(uint64_t function, const unsigned grid[3], const unsigned block[3],
                          const unsigned cluster[3], unsigned smem_bytes, uint64_t stream,
                          void **params) {
    return emmy_rt_launch_ex(function, grid, block, cluster, smem_bytes, stream, params, 0);
}

/* -------------------------------------------------------------------- TMA */

EXPORT int emmy_rt_tensor_map_encode_tiled(void *out, int dtype, unsigned rank, uint64_t gaddr,
                                           const uint64_t *dims, const uint64_t *strides_bytes,
                                           const unsigned *box, const unsigned *elem_strides,
                                           int interleave, int swizzle, int l2promo, int oobfill) {
    NEED_INIT();
    if (!out || ((uintptr_t)out & 63)) return fail(EMMY_RT_EINVAL, "tensor map buffer must be 64-byte aligned");
    if (rank < 1 || rank > 5) return fail(EMMY_RT_EINVAL, "tensor map rank %u", rank);
    if (gaddr & 15) return fail(EMMY_RT_EINVAL, "tensor base address is not 16-byte aligned");
    for (unsigned i = 0; i + 1 < rank; ++i)
        if (strides_bytes[i] & 15)
            return fail(EMMY_RT_EINVAL, "tensor stride %u (%llu bytes) is not a multiple of 16", i + 1,
                        (unsigned long long)strides_bytes[i]);
    cuuint64_t gd[5], gs[5];
    cuuint32_t bx[5], es[5];
    for (unsigned i = 0; i < rank; ++i) {
        gd[i] = dims[i];
        bx[i] = box[i];
        es[i] = elem_strides ? elem_strides[i] : 1;
        if (i + 1 < rank) gs[i] = strides_bytes[i];
    }
    CU(cu.TensorMapEncodeTiled((CUtensorMap *)out, (CUtensorMapDataType)dtype, rank,
                               (void *)(uintptr_t)gaddr, gd, gs, bx, es,
                               (CUtensorMapInterleave)interleave, (CUtensorMapSwizzle)swizzle,
                               (CUtensorMapL2promotion)l2promo, (CUtensorMapFloatOOBfill)oobfill),
       "cuTensorMapEncodeTiled");
    return 0;
}

/* ----------------------------------------------------------------- memory */

EXPORT int emmy_rt_mem_alloc(uint64_t *dptr, size_t bytes) {
    NEED_INIT();
    CUdeviceptr p;
    CU(cu.MemAlloc(&p, bytes ? bytes : 1), "cuMemAlloc");
    *dptr = (uint64_t)p;
    return 0;
}

EXPORT int emmy_rt_mem_free(uint64_t dptr) {
    NEED_INIT();
    CU(cu.MemFree((CUdeviceptr)dptr), "cuMemFree");
    return 0;
}

EXPORT int emmy_rt_mem_info(size_t *free_bytes, size_t *total_bytes) {
    NEED_INIT();
    CU(cu.MemGetInfo(free_bytes, total_bytes), "cuMemGetInfo");
    return 0;
}

EXPORT int emmy_rt_host_alloc(void **ptr, size_t bytes) {
    NEED_INIT();
    CU(cu.MemHostAlloc(ptr, bytes ? bytes : 1, CU_MEMHOSTALLOC_PORTABLE), "cuMemHostAlloc");
    return 0;
}

EXPORT int emmy_rt_host_free(void *ptr) {
    NEED_INIT();
    CU(cu.MemFreeHost(ptr), "cuMemFreeHost");
    return 0;
}

EXPORT int emmy_rt_memcpy_htod(uint64_t dst, const void *src, size_t bytes, uint64_t stream) {
    NEED_INIT();
    CU(cu.MemcpyHtoDAsync((CUdeviceptr)dst, src, bytes, (CUstream)(uintptr_t)stream), "cuMemcpyHtoDAsync");
    return 0;
}

EXPORT int emmy_rt_memcpy_dtoh(void *dst, uint64_t src, size_t bytes, uint64_t stream) {
    NEED_INIT();
    CU(cu.MemcpyDtoHAsync(dst, (CUdeviceptr)src, bytes, (CUstream)(uintptr_t)stream), "cuMemcpyDtoHAsync");
    return 0;
}

EXPORT int emmy_rt_memcpy_dtod(uint64_t dst, uint64_t src, size_t bytes, uint64_t stream) {
    NEED_INIT();
    CU(cu.MemcpyDtoDAsync((CUdeviceptr)dst, (CUdeviceptr)src, bytes, (CUstream)(uintptr_t)stream),
       "cuMemcpyDtoDAsync");
    return 0;
}

EXPORT int emmy_rt_memset(uint64_t dst, unsigned char value, size_t bytes, uint64_t stream) {
    NEED_INIT();
    CU(cu.MemsetD8Async((CUdeviceptr)dst, value, bytes, (CUstream)(uintptr_t)stream), "cuMemsetD8Async");
    return 0;
}

/* ------------------------------------------------------- streams / events */

EXPORT int emmy_rt_stream_create(uint64_t *stream) {
    NEED_INIT();
    CUstream s;
    CU(cu.StreamCreate(&s, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    *stream = (uint64_t)(uintptr_t)s;
    return 0;
}

EXPORT int emmy_rt_stream_destroy(uint64_t stream) {
    NEED_INIT();
    CU(cu.StreamDestroy((CUstream)(uintptr_t)stream), "cuStreamDestroy");
    return 0;
}

EXPORT int emmy_rt_stream_synchronize(uint64_t stream) {
    NEED_INIT();
    CU(cu.StreamSynchronize((CUstream)(uintptr_t)stream), "cuStreamSynchronize");
    return 0;
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

EXPORT int emmy_rt_stream_wait(uint64_t stream, double timeout_s) {
    NEED_INIT();
    double deadline = now_s() + timeout_s;
    for (;;) {
        CUresult r = cu.StreamQuery((CUstream)(uintptr_t)stream);
        if (r == CUDA_SUCCESS) return 0;
        if (r != CUDA_ERROR_NOT_READY) return cu_fail(r, "cuStreamQuery");
        if (now_s() > deadline)
            return fail(EMMY_RT_ETIMEOUT, "stream still busy after %.1f s", timeout_s);
        struct timespec ts = {0, 200000};
        nanosleep(&ts, NULL);
    }
}

EXPORT int emmy_rt_stream_wait_event(uint64_t stream, uint64_t event) {
    NEED_INIT();
    CU(cu.StreamWaitEvent((CUstream)(uintptr_t)stream, (CUevent)(uintptr_t)event, 0), "cuStreamWaitEvent");
    return 0;
}

/* ------------------------------------------------------------------ graphs */

EXPORT int emmy_rt_graph_begin(uint64_t stream) {
    NEED_INIT();
    if (stream == 0) return fail(EMMY_RT_EINVAL, "the legacy default stream cannot be captured");
    CU(cu.StreamBeginCapture((CUstream)(uintptr_t)stream, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL),
       "cuStreamBeginCapture");
    return 0;
}

EXPORT int emmy_rt_graph_end(uint64_t stream, uint64_t *graph) {
    NEED_INIT();
    CUgraph g = NULL;
    CUgraphExec e = NULL;
    CU(cu.StreamEndCapture((CUstream)(uintptr_t)stream, &g), "cuStreamEndCapture");
    CUresult r = cu.GraphInstantiateWithFlags(&e, g, 0);
    cu.GraphDestroy(g);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuGraphInstantiateWithFlags");
    *graph = (uint64_t)(uintptr_t)e;
    return 0;
}

EXPORT int emmy_rt_graph_launch(uint64_t graph, uint64_t stream) {
    NEED_INIT();
    CU(cu.GraphLaunch((CUgraphExec)(uintptr_t)graph, (CUstream)(uintptr_t)stream), "cuGraphLaunch");
    return 0;
}

EXPORT int emmy_rt_graph_upload(uint64_t graph, uint64_t stream) {
    NEED_INIT();
    CU(cu.GraphUpload((CUgraphExec)(uintptr_t)graph, (CUstream)(uintptr_t)stream), "cuGraphUpload");
    return 0;
}

EXPORT int emmy_rt_graph_destroy(uint64_t graph) {
    NEED_INIT();
    CU(cu.GraphExecDestroy((CUgraphExec)(uintptr_t)graph), "cuGraphExecDestroy");
    return 0;
}

EXPORT int emmy_rt_event_create(uint64_t *event) {
    NEED_INIT();
    CUevent e;
    CU(cu.EventCreate(&e, CU_EVENT_DEFAULT), "cuEventCreate");
    *event = (uint64_t)(uintptr_t)e;
    return 0;
}

EXPORT int emmy_rt_event_destroy(uint64_t event) {
    NEED_INIT();
    CU(cu.EventDestroy((CUevent)(uintptr_t)event), "cuEventDestroy");
    return 0;
}

EXPORT int emmy_rt_event_record(uint64_t event, uint64_t stream) {
    NEED_INIT();
    CU(cu.EventRecord((CUevent)(uintptr_t)event, (CUstream)(uintptr_t)stream), "cuEventRecord");
    return 0;
}

EXPORT int emmy_rt_event_synchronize(uint64_t event) {
    NEED_INIT();
    CU(cu.EventSynchronize((CUevent)(uintptr_t)event), "cuEventSynchronize");
    return 0;
}

EXPORT int emmy_rt_event_elapsed_ms(uint64_t start, uint64_t end, float *ms) {
    NEED_INIT();
    CU(cu.EventElapsedTime(ms, (CUevent)(uintptr_t)start, (CUevent)(uintptr_t)end), "cuEventElapsedTime");
    return 0;
}

/* ------------------------------------------------------------------- NCCL */

typedef struct { char internal[128]; } nccl_unique_id;

static struct {
    void *lib;
    int (*GetUniqueId)(nccl_unique_id *);
    int (*CommInitRank)(void **, int, nccl_unique_id, int);
    int (*AllReduce)(const void *, void *, size_t, int, int, void *, CUstream);
    int (*CommDestroy)(void *);
    const char *(*GetErrorString)(int);
} nc;

static int nccl_fail(int r, const char *what) {
    return fail(r, "%s failed: %s", what, nc.GetErrorString ? nc.GetErrorString(r) : "?");
}

EXPORT int emmy_rt_nccl_load(const char *path) {
    if (nc.lib) return 0;
    void *lib = dlopen(path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!lib) return fail(EMMY_RT_ENOLIB, "cannot open %s: %s", path ? path : "libnccl.so.2", dlerror());
    nc.GetUniqueId = (int (*)(nccl_unique_id *))dlsym(lib, "ncclGetUniqueId");
    nc.CommInitRank = (int (*)(void **, int, nccl_unique_id, int))dlsym(lib, "ncclCommInitRank");
    nc.AllReduce = (int (*)(const void *, void *, size_t, int, int, void *, CUstream))dlsym(lib, "ncclAllReduce");
    nc.CommDestroy = (int (*)(void *))dlsym(lib, "ncclCommDestroy");
    nc.GetErrorString = (const char *(*)(int))dlsym(lib, "ncclGetErrorString");
    if (!nc.GetUniqueId || !nc.CommInitRank || !nc.AllReduce || !nc.CommDestroy) {
        dlclose(lib);
        memset(&nc, 0, sizeof nc);
        return fail(EMMY_RT_ENOSYM, "libnccl lacks a required symbol");
    }
    nc.lib = lib;
    return 0;
}

EXPORT int emmy_rt_nccl_unique_id(void *id) {
    if (!nc.lib) return fail(EMMY_RT_ENOLIB, "emmy_rt_nccl_load was not called");
    nccl_unique_id u;
    int r = nc.GetUniqueId(&u);
    if (r) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id, &u, sizeof u);
    return 0;
}

EXPORT int emmy_rt_nccl_comm_init(uint64_t *comm, int nranks, const void *id, int rank) {
    if (!nc.lib) return fail(EMMY_RT_ENOLIB, "emmy_rt_nccl_load was not called");
    nccl_unique_id u;
    memcpy(&u, id, sizeof u);
    void *c = NULL;
    int r = nc.CommInitRank(&c, nranks, u, rank);
    if (r) return nccl_fail(r, "ncclCommInitRank");
    *comm = (uint64_t)(uintptr_t)c;
    return 0;
}

EXPORT int emmy_rt_nccl_allreduce(uint64_t comm, uint64_t sendbuf, uint64_t recvbuf, size_t count,
                                  int dtype, int op, uint64_t stream) {
    if (!nc.lib) return fail(EMMY_RT_ENOLIB, "emmy_rt_nccl_load was not called");
    int r = nc.AllReduce((const void *)(uintptr_t)sendbuf, (void *)(uintptr_t)recvbuf, count, dtype, op,
                         (void *)(uintptr_t)comm, (CUstream)(uintptr_t)stream);
    if (r) return nccl_fail(r, "ncclAllReduce");
    return 0;
}

EXPORT int emmy_rt_nccl_comm_destroy(uint64_t comm) {
    if (!nc.lib) return fail(EMMY_RT_ENOLIB, "emmy_rt_nccl_load was not called");
    int r = nc.CommDestroy((void *)(uintptr_t)comm);
    if (r) return nccl_fail(r, "ncclCommDestroy");
    return 0;
}
