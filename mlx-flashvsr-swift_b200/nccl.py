"""NCCL communicator over ctypes for the query-block partition of a chunk across the GPUs of one node.

The collectives run on streams the caller chooses (the library's compute stream, or a communication stream beside
it), so they order with the library's kernels by stream semantics and can be captured in a CUDA graph. The library
loaded is the one torch ships (the same NCCL the process group uses), else the system's. The unique id is handed from
rank 0 to the others through the process group that the launcher set up (torch.distributed).

Failure handling: every blocking point of a collective is on the device; `check()` reads the communicator's async
error (ncclCommGetAsyncError) so that a rank whose peer died ends with an exception, and `abort()` tears the
communicator down without waiting for peers.
"""
from __future__ import annotations

import ctypes
import glob
import os

NCCL_INT8 = 0
NCCL_FLOAT32 = 7
_RESULTS = {0: "ncclSuccess", 1: "ncclUnhandledCudaError", 2: "ncclSystemError", 3: "ncclInternalError",
            4: "ncclInvalidArgument", 5: "ncclInvalidUsage", 6: "ncclRemoteError", 7: "ncclInProgress"}


class NcclError(RuntimeError):
    pass


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_byte * 128)]


def library_path() -> str:
    """torch's bundled libnccl (site-packages/nvidia/nccl/lib) when present, else the system libnccl.so.2."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    if spec is not None and spec.submodule_search_locations:
        for base in spec.submodule_search_locations:
            hits = glob.glob(os.path.join(base, "nccl", "lib", "libnccl.so*"))
            if hits:
                return sorted(hits)[0]
    return "libnccl.so.2"


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = ctypes.CDLL(library_path())
        P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        L.ncclGetUniqueId.argtypes = [ctypes.POINTER(_UniqueId)]
        L.ncclCommInitRank.argtypes = [ctypes.POINTER(P), I, _UniqueId, I]
        L.ncclAllGather.argtypes = [P, P, SZ, I, P, P]
        L.ncclSend.argtypes = [P, SZ, I, I, P, P]
        L.ncclRecv.argtypes = [P, SZ, I, I, P, P]
        L.ncclGroupStart.argtypes = []
        L.ncclGroupEnd.argtypes = []
        L.ncclCommDestroy.argtypes = [P]
        L.ncclCommAbort.argtypes = [P]
        L.ncclCommGetAsyncError.argtypes = [P, ctypes.POINTER(I)]
        L.ncclGetErrorString.argtypes = [I]
        L.ncclGetErrorString.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _ok(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().ncclGetErrorString(rc)
        raise NcclError(f"{what}: {_RESULTS.get(rc, rc)} ({msg.decode() if msg else ''})")


class Comm:
    """One NCCL communicator over the ranks of the current torch.distributed process group (one GPU each)."""

    def __init__(self, rank: int, world: int, device):
        import torch
        import torch.distributed as dist
        self.rank, self.world = rank, world
        uid = _UniqueId()
        if rank == 0:
            _ok(lib().ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
        buf = torch.tensor(list(bytes(uid.internal)), dtype=torch.uint8, device=device)
        if world > 1:
            dist.broadcast(buf, src=0)
        raw = bytes(buf.cpu().tolist())
        ctypes.memmove(uid.internal, raw, 128)
        self.handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _ok(lib().ncclCommInitRank(ctypes.byref(self.handle), world, uid, rank), "ncclCommInitRank")

    def all_gather(self, send, recv, stream) -> None:
        """recv (world × send's bytes, rank order) ← every rank's send, on `stream` (a torch.cuda.Stream)."""
        n = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() < n * self.world:
            raise NcclError("all_gather: receive buffer too small")
        _ok(lib().ncclAllGather(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()), n, NCCL_INT8,
                                self.handle, ctypes.c_void_p(stream.cuda_stream)), "ncclAllGather")

    def group_start(self) -> None:
        _ok(lib().ncclGroupStart(), "ncclGroupStart")

    def group_end(self) -> None:
        _ok(lib().ncclGroupEnd(), "ncclGroupEnd")

    def check(self) -> None:
        """Raises NcclError if the communicator recorded an asynchronous error (e.g. a peer is gone)."""
        st = ctypes.c_int(0)
        _ok(lib().ncclCommGetAsyncError(self.handle, ctypes.byref(st)), "ncclCommGetAsyncError")
        if st.value not in (0, 7):
            raise NcclError(f"communicator error: {_RESULTS.get(st.value, st.value)}")

    def destroy(self) -> None:
        if self.handle:
            lib().ncclCommDestroy(self.handle)
            self.handle = None

    def abort(self) -> None:
        if self.handle:
            lib().ncclCommAbort(self.handle)
            self.handle = None
