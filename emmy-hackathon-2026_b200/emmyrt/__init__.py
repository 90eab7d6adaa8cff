"""ctypes binding of the native launch runtime (``libemmyrt.so``, C ABI in include/emmyrt.h).

This replaces the reference's remote runner client (``submit.py:99-135``): PTX is
assembled locally with ``ptxas -arch=sm_100a`` (the runner ran ptxas remotely,
``docs/API.md:12-24``), loaded through the driver, and launched with the launch
descriptor the compiler wrote into the module.

The extension is required: importing this package on a machine where the shared
library was not built raises ``ImportError`` -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import shutil
import subprocess
import tempfile
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libemmyrt.so"

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                      "(or python emmy-hackathon-2026_b200/build.py)")

lib = ctypes.CDLL(str(LIB_PATH))

_u64, _u32, _int, _sz = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t
_P = ctypes.POINTER

# every symbol declared in include/emmyrt.h, with its ctypes signature
SIGNATURES = {
    "emmy_rt_last_error": ([], ctypes.c_char_p),
    "emmy_rt_version": ([], _int),
    "emmy_rt_init": ([_int], _int),
    "emmy_rt_device_count": ([_P(_int)], _int),
    "emmy_rt_device_attribute": ([_int, _int, _P(_int)], _int),
    "emmy_rt_set_device": ([_int], _int),
    "emmy_rt_synchronize": ([], _int),
    "emmy_rt_module_load": ([ctypes.c_void_p, _sz, _P(_u64)], _int),
    "emmy_rt_module_unload": ([_u64], _int),
    "emmy_rt_module_function": ([_u64, ctypes.c_char_p, _P(_u64)], _int),
    "emmy_rt_module_global": ([_u64, ctypes.c_char_p, _P(_u64), _P(_sz)], _int),
    "emmy_rt_function_attribute": ([_u64, _int, _P(_int)], _int),
    "emmy_rt_function_set_max_dynamic_smem": ([_u64, _int], _int),
    "emmy_rt_launch": ([_u64, _P(ctypes.c_uint), _P(ctypes.c_uint), _P(ctypes.c_uint), ctypes.c_uint,
                        _u64, _P(ctypes.c_void_p)], _int),
    "emmy_rt_launch_ex": ([_u64, _P(ctypes.c_uint), _P(ctypes.c_uint), _P(ctypes.c_uint), ctypes.c_uint,
                           _u64, _P(ctypes.c_void_p), ctypes.c_uint], _int),
    "emmy_rt_tensor_map_encode_tiled": ([ctypes.c_void_p, _int, ctypes.c_uint, _u64, _P(_u64), _P(_u64),
                                         _P(ctypes.c_uint), _P(ctypes.c_uint), _int, _int, _int, _int], _int),
    "emmy_rt_mem_alloc": ([_P(_u64), _sz], _int),
    "emmy_rt_mem_free": ([_u64], _int),
    "emmy_rt_mem_info": ([_P(_sz), _P(_sz)], _int),
    "emmy_rt_host_alloc": ([_P(ctypes.c_void_p), _sz], _int),
    "emmy_rt_host_free": ([ctypes.c_void_p], _int),
    "emmy_rt_memcpy_htod": ([_u64, ctypes.c_void_p, _sz, _u64], _int),
    "emmy_rt_memcpy_dtoh": ([ctypes.c_void_p, _u64, _sz, _u64], _int),
    "emmy_rt_memcpy_dtod": ([_u64, _u64, _sz, _u64], _int),
    "emmy_rt_memset": ([_u64, ctypes.c_ubyte, _sz, _u64], _int),
    "emmy_rt_stream_create": ([_P(_u64)], _int),
    "emmy_rt_stream_destroy": ([_u64], _int),
    "emmy_rt_stream_synchronize": ([_u64], _int),
    "emmy_rt_stream_wait": ([_u64, ctypes.c_double], _int),
    "emmy_rt_stream_wait_event": ([_u64, _u64], _int),
    "emmy_rt_graph_begin": ([_u64], _int),
    "emmy_rt_graph_end": ([_u64, _P(_u64)], _int),
    "emmy_rt_graph_launch": ([_u64, _u64], _int),
    "emmy_rt_graph_upload": ([_u64, _u64], _int),
    "emmy_rt_graph_destroy": ([_u64], _int),
    "emmy_rt_event_create": ([_P(_u64)], _int),
    "emmy_rt_event_destroy": ([_u64], _int),
    "emmy_rt_event_record": ([_u64, _u64], _int),
    "emmy_rt_event_synchronize": ([_u64], _int),
    "emmy_rt_event_elapsed_ms": ([_u64, _u64, _P(ctypes.c_float)], _int),
    "emmy_rt_nccl_load": ([ctypes.c_char_p], _int),
    "emmy_rt_nccl_unique_id": ([ctypes.c_void_p], _int),
    "emmy_rt_nccl_comm_init": ([_P(_u64), _int, ctypes.c_void_p, _int], _int),
    "emmy_rt_nccl_allreduce": ([_u64, _u64, _u64, _sz, _int, _int, _u64], _int),
    "emmy_rt_nccl_comm_destroy": ([_u64], _int),
}

for _name, (_args, _res) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res


class EmmyRTError(RuntimeError):
    def __init__(self, status: int, what: str):
        msg = lib.emmy_rt_last_error().decode(errors="replace")
        super().__init__(f"{what}: status {status}: {msg}")
        self.status = status


def check(status: int, what: str) -> None:
    if status != 0:
        raise EmmyRTError(status, what)


# ---------------------------------------------------------------------------
# device

_initialised: dict[int, bool] = {}

CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT = 16
CU_DEVICE_ATTRIBUTE_CC_MAJOR = 75
CU_DEVICE_ATTRIBUTE_CC_MINOR = 76


def init(device: int = 0) -> None:
    """Open the driver and make ``device``'s primary context current (idempotent)."""
    if _initialised.get(device):
        check(lib.emmy_rt_set_device(device), "emmy_rt_set_device")
        return
    check(lib.emmy_rt_init(device), "emmy_rt_init")
    _initialised[device] = True


def device_attribute(attr: int, device: int = 0) -> int:
    v = ctypes.c_int()
    check(lib.emmy_rt_device_attribute(attr, device, ctypes.byref(v)), "device attribute")
    return v.value


def sm_count(device: int = 0) -> int:
    return device_attribute(CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, device)


def synchronize() -> None:
    check(lib.emmy_rt_synchronize(), "synchronize")


# ---------------------------------------------------------------------------
# memory


class DeviceBuffer:
    """An owned device allocation."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        p = _u64()
        check(lib.emmy_rt_mem_alloc(ctypes.byref(p), max(1, self.nbytes)), f"alloc {nbytes} B")
        self.ptr = p.value

    def free(self) -> None:
        if self.ptr:
            lib.emmy_rt_mem_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def upload(self, array, stream: int = 0) -> None:
        import numpy as np
        a = np.ascontiguousarray(array)
        if a.nbytes > self.nbytes:
            raise ValueError("upload larger than the buffer")
        check(lib.emmy_rt_memcpy_htod(self.ptr, a.ctypes.data, a.nbytes, stream), "htod")
        if stream == 0:
            check(lib.emmy_rt_stream_synchronize(0), "sync")

    def download(self, array, stream: int = 0):
        import numpy as np
        if not array.flags["C_CONTIGUOUS"]:
            raise ValueError("download target must be contiguous")
        check(lib.emmy_rt_memcpy_dtoh(array.ctypes.data, self.ptr, array.nbytes, stream), "dtoh")
        check(lib.emmy_rt_stream_synchronize(stream), "sync")
        return array

    def zero(self, stream: int = 0) -> None:
        check(lib.emmy_rt_memset(self.ptr, 0, self.nbytes, stream), "memset")


class HostBuffer:
    """Page-locked host memory viewed as a numpy array."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib.emmy_rt_host_alloc(ctypes.byref(p), max(1, nbytes)), f"host alloc {nbytes} B")
        self.ptr, self.nbytes = p.value, nbytes

    def array(self, dtype, shape):
        import numpy as np
        buf = (ctypes.c_char * self.nbytes).from_address(self.ptr)
        return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)

    def free(self):
        if self.ptr:
            lib.emmy_rt_host_free(ctypes.c_void_p(self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Stream:
    """A non-blocking stream of the current context (its handle is ``.handle``)."""

    def __init__(self):
        s = _u64()
        check(lib.emmy_rt_stream_create(ctypes.byref(s)), "stream create")
        self.handle = s.value

    def wait(self, event: "Event") -> None:
        """Later work on this stream waits for ``event``'s latest recording."""
        check(lib.emmy_rt_stream_wait_event(self.handle, event.handle), "stream wait event")

    def __del__(self):
        try:
            lib.emmy_rt_stream_destroy(self.handle)
        except Exception:
            pass


class Graph:
    """Launches captured from a stream once and replayed as one CUDA graph::

        g = Graph.capture(stream, lambda: [fire(stream.handle) for fire in launches])
        g.launch(0)
    """

    def __init__(self, handle: int):
        self.handle = handle

    @classmethod
    def capture(cls, stream: "Stream", enqueue, keep=()) -> "Graph":
        """The captured launches refer to their buffers, scratch and modules by device
        address only, so whatever owns them (``DeviceBuffer``, ``CompiledKernel``) must live
        as long as the graph is replayed: a replay after they are freed reads freed memory.
        The graph holds ``enqueue`` and the objects in ``keep`` for that purpose."""
        check(lib.emmy_rt_graph_begin(stream.handle), "graph begin")
        try:
            enqueue()
        finally:
            g = _u64()
            check(lib.emmy_rt_graph_end(stream.handle, ctypes.byref(g)), "graph end")
        graph = cls(g.value)
        graph._keep = (enqueue, tuple(keep))
        return graph

    def launch(self, stream: int = 0) -> None:
        check(lib.emmy_rt_graph_launch(self.handle, stream), "graph launch")

    def upload(self, stream: int = 0) -> None:
        """Stage the graph on the device without running it."""
        check(lib.emmy_rt_graph_upload(self.handle, stream), "graph upload")

    def __del__(self):
        try:
            lib.emmy_rt_graph_destroy(self.handle)
        except Exception:
            pass


class Event:
    def __init__(self):
        e = _u64()
        check(lib.emmy_rt_event_create(ctypes.byref(e)), "event create")
        self.handle = e.value

    def record(self, stream: int = 0):
        check(lib.emmy_rt_event_record(self.handle, stream), "event record")

    def synchronize(self):
        check(lib.emmy_rt_event_synchronize(self.handle), "event sync")

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        check(lib.emmy_rt_event_elapsed_ms(self.handle, end.handle, ctypes.byref(ms)), "elapsed")
        return ms.value

    def __del__(self):
        try:
            lib.emmy_rt_event_destroy(self.handle)
        except Exception:
            pass


def stream_wait(stream: int, timeout_s: float = 60.0) -> None:
    """Wait for ``stream`` with a deadline (the runner's 20 s launch limit, docs/API.md:69)."""
    check(lib.emmy_rt_stream_wait(stream, timeout_s), "stream wait")


# ---------------------------------------------------------------------------
# ptxas + modules

PTXAS = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
_CACHE = Path(os.environ.get("EMMY_CUBIN_CACHE", os.path.join(tempfile.gettempdir(), "emmy_cubin")))


def assemble(ptx: str, arch: str = "sm_100a", extra: tuple = ()) -> tuple[bytes, str]:
    """``ptxas -arch=sm_100a -v`` -> (cubin bytes, ptxas -v log); cached by content."""
    key = hashlib.sha256((ptx + arch + " ".join(extra)).encode()).hexdigest()[:24]
    _CACHE.mkdir(parents=True, exist_ok=True)
    cub, log = _CACHE / f"{key}.cubin", _CACHE / f"{key}.log"
    if cub.exists() and log.exists():
        return cub.read_bytes(), log.read_text()
    with tempfile.TemporaryDirectory() as td:
        src, out = Path(td) / "k.ptx", Path(td) / "k.cubin"
        src.write_text(ptx)
        r = subprocess.run([PTXAS, f"-arch={arch}", "-v", *extra, str(src), "-o", str(out)],
                           capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"ptxas rejected the module:\n{r.stderr}")
        data = out.read_bytes()
    # per-process temporary names and renames, the cubin last: processes assembling the
    # same module at once (one per GPU) never read a half-written entry
    tmp = log.with_name(f".{log.name}.{os.getpid()}.tmp")
    tmp.write_text(r.stderr)
    tmp.replace(log)
    tmp = cub.with_name(f".{cub.name}.{os.getpid()}.tmp")
    tmp.write_bytes(data)
    tmp.replace(cub)
    return data, r.stderr


class Module:
    def __init__(self, ptx: str):
        self.ptx = ptx
        self.cubin, self.ptxas_log = assemble(ptx)
        m = _u64()
        buf = ctypes.create_string_buffer(self.cubin, len(self.cubin))
        check(lib.emmy_rt_module_load(buf, len(self.cubin), ctypes.byref(m)), "module load")
        self.handle = m.value

    def function(self, entry: str) -> int:
        f = _u64()
        check(lib.emmy_rt_module_function(self.handle, entry.encode(), ctypes.byref(f)),
              f"entry {entry}")
        return f.value

    def global_ptr(self, name: str) -> tuple[int, int]:
        p, n = _u64(), _sz()
        check(lib.emmy_rt_module_global(self.handle, name.encode(), ctypes.byref(p), ctypes.byref(n)),
              f"global {name}")
        return p.value, n.value


CU_FUNC_ATTRIBUTE_NUM_REGS = 4


def function_attribute(fn: int, attr: int) -> int:
    v = ctypes.c_int()
    check(lib.emmy_rt_function_attribute(fn, attr, ctypes.byref(v)), "function attribute")
    return v.value


class PreparedLaunch:
    """A launch whose argument arrays are built once: each call is one C call (no
    per-launch Python marshalling), so back-to-back launches keep the GPU fed."""

    def __init__(self, fn: int, grid, block, cluster, smem: int, params: list, flags: int = 0):
        self.fn, self.smem, self.flags = fn, smem, flags
        self.g = (ctypes.c_uint * 3)(*grid)
        self.b = (ctypes.c_uint * 3)(*block)
        self.c = (ctypes.c_uint * 3)(*(cluster or (1, 1, 1)))
        self.params = params
        self.arr = (ctypes.c_void_p * max(1, len(params)))(
            *[ctypes.cast(ctypes.pointer(p), ctypes.c_void_p) if not isinstance(p, ctypes.Array)
              else ctypes.cast(p, ctypes.c_void_p) for p in params])
        self._launch = lib.emmy_rt_launch_ex

    def __call__(self, stream: int = 0) -> None:
        st = self._launch(self.fn, self.g, self.b, self.c, self.smem, stream, self.arr, self.flags)
        if st:
            check(st, "launch")


LAUNCH_PDL = 1      # EMMY_RT_LAUNCH_PDL


def launch(fn: int, grid, block, cluster, smem: int, stream: int, params: list, flags: int = 0) -> None:
    """``params``: one ctypes object per kernel parameter (c_uint64 pointers, tensor
    map byte arrays, scalars), in signature order."""
    g = (ctypes.c_uint * 3)(*grid)
    b = (ctypes.c_uint * 3)(*block)
    c = (ctypes.c_uint * 3)(*(cluster or (1, 1, 1)))
    arr = (ctypes.c_void_p * max(1, len(params)))(
        *[ctypes.cast(ctypes.pointer(p), ctypes.c_void_p) if not isinstance(p, ctypes.Array)
          else ctypes.cast(p, ctypes.c_void_p) for p in params])
    check(lib.emmy_rt_launch_ex(fn, g, b, c, smem, stream, arr, flags), "launch")


# ---------------------------------------------------------------------------
# TMA descriptors

TMA_DTYPE = {"u8": 0, "e4m3": 0, "u16": 1, "u32": 2, "i32": 3, "u64": 4, "i64": 5, "f16": 6,
             "f32": 7, "f64": 8, "bf16": 9}
TMA_SWIZZLE = {0: 0, 32: 1, 64: 2, 128: 3}


def tensor_map(gaddr: int, dtype: str, dims, strides_bytes, box, swizzle: int = 128,
               l2promo: int = 2, oobfill: int = 0):
    """A CUtensorMap (128 bytes, 64-byte aligned) as a ctypes array ready to pass as a
    kernel parameter.  ``dims``/``box`` innermost first; ``strides_bytes`` rank-1."""
    rank = len(dims)
    raw = (ctypes.c_ubyte * 192)()
    off = (-ctypes.addressof(raw)) % 64
    view = (ctypes.c_ubyte * 128).from_buffer(raw, off)
    d = (_u64 * rank)(*dims)
    s = (_u64 * max(1, rank - 1))(*strides_bytes)
    bx = (ctypes.c_uint * rank)(*box)
    es = (ctypes.c_uint * rank)(*([1] * rank))
    check(lib.emmy_rt_tensor_map_encode_tiled(ctypes.addressof(view), TMA_DTYPE[dtype], rank, gaddr,
                                              d, s, bx, es, 0, TMA_SWIZZLE[swizzle], l2promo, oobfill),
          "tensor map encode")
    view._keepalive = raw
    return view


# ---------------------------------------------------------------------------
# whole-array reductions with static scratch (libemmyrt_static.so)

STATIC_LIB_PATH = _HERE / "libemmyrt_static.so"
STATIC_SIGNATURES = {
    "emmy_rt_full_reduce_static_scratch": ([_u64, ctypes.c_uint, ctypes.c_uint, _P(_u64), _int, _sz, _u64],
                                           _int),
}
EMMY_RT_ESCRATCH = -6
_static_lib = None


def static_scratch_lib():
    """The library whose single entry point launches a whole-array reduction with its
    scratch taken from a static device array (for callers that cannot allocate)."""
    global _static_lib
    if _static_lib is None:
        if not STATIC_LIB_PATH.exists():
            raise ImportError(f"{STATIC_LIB_PATH} is not built; run __graft_entry__.build()")
        lib2 = ctypes.CDLL(str(STATIC_LIB_PATH))
        for name, (args, res) in STATIC_SIGNATURES.items():
            fn = getattr(lib2, name)
            fn.argtypes = args
            fn.restype = res
        _static_lib = lib2
    return _static_lib
