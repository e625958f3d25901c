"""Host buffers that fault on out-of-bounds access (test infrastructure).

`guarded(a, side)` copies an array into anonymous memory placed against a
PROT_NONE page: side "end" puts the data's last byte (rounded up to 16 for
vector loads) next to the guard page after it, side "start" puts its first
byte right after the guard page before it. A kernel run on the host that
reads or writes past the end (or before the start) then stops the process
with SIGSEGV instead of touching a neighbour.
"""

import ctypes
import mmap

import numpy as np

_libc = ctypes.CDLL(None, use_errno=True)
_libc.mprotect.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
_keep = []  # mappings stay alive while any view into them may be used


def guarded(a, side: str = "end") -> np.ndarray:
    a = np.ascontiguousarray(a)
    page = mmap.PAGESIZE
    nbytes = max(a.nbytes, 1)
    span = -(-nbytes // 16) * 16
    pages = -(-span // page)
    m = mmap.mmap(-1, (pages + 2) * page)
    base = ctypes.addressof(ctypes.c_char.from_buffer(m))
    for at in (base, base + (pages + 1) * page):
        if _libc.mprotect(ctypes.c_void_p(at), page, 0) != 0:
            raise OSError(ctypes.get_errno(), "mprotect failed")
    off = page + (pages * page - span if side == "end" else 0)
    view = np.frombuffer(m, dtype=a.dtype, count=a.size, offset=off).reshape(a.shape)
    view[...] = a
    _keep.append(m)
    return view


def ptr(a) -> int:
    return 0 if a is None else a.ctypes.data
