"""zstd frames through the system libzstd (ctypes; the `zstandard` Python
package is not required).

Only the one-shot frame API is used: `ZSTD_compress`, `ZSTD_decompress` and
`ZSTD_getFrameContentSize`, which is what the reference container's
`zstandard.ZstdCompressor().compress` / `ZstdDecompressor().decompress` read
and write (single frames with the content size in the header). ctypes
releases the GIL for the duration of each call, so a thread pool
decompresses several segments in parallel.
"""

from __future__ import annotations

import ctypes as C
import ctypes.util
import threading

_lib = None
_lock = threading.Lock()
_CONTENTSIZE_UNKNOWN = (1 << 64) - 1
_CONTENTSIZE_ERROR = (1 << 64) - 2


def _load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            name = ctypes.util.find_library("zstd") or "libzstd.so.1"
            lib = C.CDLL(name)
            lib.ZSTD_compressBound.restype = C.c_size_t
            lib.ZSTD_compressBound.argtypes = [C.c_size_t]
            lib.ZSTD_compress.restype = C.c_size_t
            lib.ZSTD_compress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int]
            lib.ZSTD_decompress.restype = C.c_size_t
            lib.ZSTD_decompress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
            lib.ZSTD_getFrameContentSize.restype = C.c_ulonglong
            lib.ZSTD_getFrameContentSize.argtypes = [C.c_void_p, C.c_size_t]
            lib.ZSTD_isError.restype = C.c_uint
            lib.ZSTD_isError.argtypes = [C.c_size_t]
            lib.ZSTD_getErrorName.restype = C.c_char_p
            lib.ZSTD_getErrorName.argtypes = [C.c_size_t]
            _lib = lib
    return _lib


def _check(lib, rc: int, what: str) -> int:
    if lib.ZSTD_isError(rc):
        raise RuntimeError(f"{what}: {lib.ZSTD_getErrorName(rc).decode()}")
    return rc


def compress(data, level: int = 12) -> bytes:
    """One zstd frame holding `data` (bytes-like), content size recorded."""
    lib = _load()
    src = bytes(data)
    cap = lib.ZSTD_compressBound(len(src))
    dst = C.create_string_buffer(cap)
    n = _check(lib, lib.ZSTD_compress(dst, cap, src, len(src), int(level)), "ZSTD_compress")
    return dst.raw[:n]


def decompressed_size(frame) -> int:
    lib = _load()
    src = bytes(frame[:32]) if len(frame) > 32 else bytes(frame)
    n = lib.ZSTD_getFrameContentSize(src, len(src))
    if n in (_CONTENTSIZE_UNKNOWN, _CONTENTSIZE_ERROR):
        raise RuntimeError("zstd frame without a content size")
    return int(n)


def decompress_into(frame, out) -> int:
    """Decompress one frame into the writable buffer `out` (a ctypes array,
    bytearray or numpy array); returns the bytes written."""
    lib = _load()
    src = bytes(frame)
    if isinstance(out, (bytearray, memoryview)):
        buf = (C.c_char * len(out)).from_buffer(out)
        cap = len(out)
    else:   # numpy
        buf = out.ctypes.data_as(C.c_void_p)
        cap = out.nbytes
    return _check(lib, lib.ZSTD_decompress(buf, cap, src, len(src)), "ZSTD_decompress")


def decompress(frame) -> bytes:
    out = bytearray(decompressed_size(frame))
    n = decompress_into(frame, out)
    if n != len(out):
        raise RuntimeError("zstd frame shorter than its content size")
    return bytes(out)
