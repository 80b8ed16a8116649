"""ctypes binding of the C ABI in ``include/nanoserve_sampler.h``.

This is the binding a Python maintainer of the reference would add to call
the library without torch's op registry: the structs mirror the header field
for field, and :func:`ns_sample` raises on a non-zero status with the
library's own message.  The library is loaded from this package directory;
a missing library raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libnanoserve_sampler.so"

NS_OK = 0
NS_ERR_INVALID_ARG = 1
NS_ERR_UNSUPPORTED = 2
NS_ERR_CUDA = 3

NS_DTYPE_F32 = 0
NS_DTYPE_BF16 = 1
NS_OUT_I64 = 0
NS_OUT_I32 = 1

NS_KERNEL_AUTO = 0
NS_KERNEL_CLUSTER = 1
NS_KERNEL_SPLIT = 2

NS_ROW_GREEDY = 0x1
NS_ROW_TOP_P = 0x2
NS_ROW_PENALTY = 0x4
NS_ROW_SEED = 0x8

NS_STATUS_BAD_SAMPLE_INDEX = 0x1
NS_STATUS_BAD_HISTORY_ID = 0x2
NS_STATUS_WAIT_TIMEOUT = 0x4
NS_STATUS_CAP_OVERFLOW = 0x8
NS_STATUS_BAD_ROW_ORDER = 0x10
NS_STATUS_BAD_POOL_RANGE = 0x20

# every entry point the header declares
EXPORTED_SYMBOLS = ("ns_sample", "ns_sample_noalloc", "ns_workspace_bytes", "ns_history_gather",
                    "ns_history_append", "ns_last_error", "ns_abi_version", "ns_max_vocab")
NS_ABI_VERSION = 3
NS_NOALLOC_WORKSPACE_BYTES = 128


class NsRowParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("seed_step", ctypes.c_uint32),
        ("seed", ctypes.c_uint64),
    ]


class NsSampleArgs(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p),
        ("logits_dtype", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("num_logit_rows", ctypes.c_int64),
        ("logits_row_stride", ctypes.c_int64),
        ("num_rows", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("sample_indices", ctypes.c_void_p),
        ("row_params", ctypes.c_void_p),
        ("history_offsets", ctypes.c_void_p),
        ("history_ids", ctypes.c_void_p),
        ("uniforms", ctypes.c_void_p),
        ("philox_seed", ctypes.c_uint64),
        ("philox_offset", ctypes.c_uint64),
        ("row_offset", ctypes.c_int64),
        ("out_tokens", ctypes.c_void_p),
        ("out_penalized", ctypes.c_void_p),
        ("out_filtered", ctypes.c_void_p),
        ("out_probs", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("row_order", ctypes.c_void_p),
        ("kernel", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
    ]


assert ctypes.sizeof(NsRowParams) == 32


class NativeLibraryMissing(RuntimeError):
    """The CUDA library was not built; there is no fallback implementation."""


_lib = None


def load_library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                "(there is no CPU fallback for the sampling op)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.ns_sample.argtypes = [ctypes.POINTER(NsSampleArgs), ctypes.c_void_p]
        lib.ns_sample.restype = ctypes.c_int
        lib.ns_sample_noalloc.argtypes = [ctypes.POINTER(NsSampleArgs), ctypes.c_void_p]
        lib.ns_sample_noalloc.restype = ctypes.c_int
        lib.ns_history_gather.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.ns_history_gather.restype = ctypes.c_int
        lib.ns_history_append.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
        lib.ns_history_append.restype = ctypes.c_int
        lib.ns_last_error.argtypes = []
        lib.ns_last_error.restype = ctypes.c_char_p
        lib.ns_abi_version.argtypes = []
        lib.ns_abi_version.restype = ctypes.c_int
        lib.ns_max_vocab.argtypes = [ctypes.c_int32]
        lib.ns_max_vocab.restype = ctypes.c_int32
        lib.ns_workspace_bytes.argtypes = [ctypes.c_int32]
        lib.ns_workspace_bytes.restype = ctypes.c_int64
        _lib = lib
    return _lib


class NsError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"ns_sample failed ({code}): {message}")
        self.code = code


def ns_sample(args: NsSampleArgs, stream: int = 0) -> None:
    lib = load_library()
    rc = lib.ns_sample(ctypes.byref(args), ctypes.c_void_p(stream))
    if rc != NS_OK:
        raise NsError(rc, lib.ns_last_error().decode(errors="replace"))


def ns_sample_noalloc(args: NsSampleArgs, stream: int = 0) -> None:
    """The entry point for callers that cannot allocate device memory: it
    ignores ``args.workspace`` and runs on the library's static workspace."""
    lib = load_library()
    rc = lib.ns_sample_noalloc(ctypes.byref(args), ctypes.c_void_p(stream))
    if rc != NS_OK:
        raise NsError(rc, lib.ns_last_error().decode(errors="replace"))


def ns_workspace_bytes(num_rows: int) -> int:
    """Bytes of ``NsSampleArgs.workspace`` for calls of up to ``num_rows`` rows."""
    return int(load_library().ns_workspace_bytes(int(num_rows)))


def ns_history_gather(pool: int, pool_size: int, row_src: int, offsets: int, num_rows: int, out_ids: int,
                      status: int = 0, stream: int = 0) -> None:
    """Build one step's CSR history ids from a device pool (device pointers as ints)."""
    lib = load_library()
    rc = lib.ns_history_gather(pool or None, pool_size, row_src or None, offsets or None, num_rows,
                               out_ids or None, status or None, ctypes.c_void_p(stream))
    if rc != NS_OK:
        raise NsError(rc, lib.ns_last_error().decode(errors="replace"))


def ns_history_append(pool: int, pool_size: int, row_dst: int, tokens: int, tokens_dtype: int, num_rows: int,
                      status: int = 0, stream: int = 0) -> None:
    """Append one sampled id per row to the device pool (device pointers as ints)."""
    lib = load_library()
    rc = lib.ns_history_append(pool or None, pool_size, row_dst or None, tokens or None, tokens_dtype, num_rows,
                               status or None, ctypes.c_void_p(stream))
    if rc != NS_OK:
        raise NsError(rc, lib.ns_last_error().decode(errors="replace"))
